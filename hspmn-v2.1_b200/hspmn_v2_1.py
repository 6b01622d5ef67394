"""Compatibility module with the reference's name (hspmn_v2_1.py).

``from hspmn_v2_1 import HSPMNBlock, TopKRouter, HSPMNConfig`` works unchanged;
the block's eval-mode contextual stream runs on the sm_100a library.
``HAS_TRITON_KERNELS`` keeps its name for scripts that read it and is True
when the native library is present (the path needs no Triton).
"""

from hspmn_b200._native import available as _available
from hspmn_b200.model import (  # noqa: F401
    HSPMNBlock,
    ReflexiveStream,
    RotaryEmbedding,
    RouterOutput,
    TopKRouter,
    apply_rotary_pos_emb,
    get_compiled_flex_attention,
    rotate_half,
)
from hspmn_b200.utils import HSPMNConfig  # noqa: F401

HAS_TRITON_KERNELS = _available()
HAS_NATIVE_KERNELS = HAS_TRITON_KERNELS

__all__ = ["HSPMNBlock", "TopKRouter", "HSPMNConfig"]
