"""hspmn_b200: the HSPMN v2.1 contextual-stream inference path on B200 (sm_100a).

Public API mirrors the reference modules: ``HSPMNBlock``, ``TopKRouter``,
``HSPMNConfig``, ``RouterOutput`` and ``sparse_query_dense_key_attention``.
The kernels live in ``libhspmn_sm100.so`` (built by ``build_native.py``)
and are exposed as ``torch.ops.hspmn.*`` custom ops through ``ops``.
"""

from . import ops  # noqa: F401
from ._native import available as native_available  # noqa: F401
from .kernels import sparse_query_dense_key_attention  # noqa: F401
from .model import (  # noqa: F401
    HSPMNBlock,
    ReflexiveStream,
    RotaryEmbedding,
    RouterOutput,
    TopKRouter,
    apply_rotary_pos_emb,
    rotate_half,
)
from .utils import HSPMNConfig, get_device, seed_everything, setup_env, setup_logging  # noqa: F401

__version__ = "0.1.0"
