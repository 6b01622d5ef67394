"""Compatibility module with the reference's name (utils_v2_1.py)."""

from hspmn_b200.utils import (  # noqa: F401
    HSPMNConfig,
    get_device,
    seed_everything,
    setup_env,
    setup_logging,
)
