"""The reference's SQDK entry point, backed by the sm_100a library.

Drop-in for ``kernels_v2_1.sparse_query_dense_key_attention``
(kernels_v2_1.py:141-180): same name, arguments, return convention (a new
tensor shaped and typed like ``q``) and shape assertions. Grouped K/V heads
(``k.shape[2] < q.shape[2]``) are supported with the Flex path's semantics
(hspmn_v2_1.py:212) instead of being indexed as query heads. When an input
requires grad, the result is differentiable (backward on the sm_100a kernels).
"""

from __future__ import annotations

import torch

from . import ops


def sparse_query_dense_key_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                     q_indices: torch.Tensor, block_m: int = 64,
                                     block_n: int = 64) -> torch.Tensor:
    """Sparse-Query Dense-Key attention.

    Args:
        q: [Batch, N_Active, Heads, Dim] gathered queries.
        k, v: [Batch, Seq_Len, KV_Heads, Dim], KV_Heads dividing Heads.
        q_indices: [Batch, N_Active] int64 original positions of the queries,
            sorted ascending per row (sortedness only affects speed).
        block_m, block_n: accepted for compatibility; the sm_100a kernel
            tiles 128 (query, head) rows by 64 keys.
    Returns:
        o: [Batch, N_Active, Heads, Dim], dtype of q.
    """
    Lq, Lk = q.shape[1], k.shape[1]  # noqa: F841 (mirrors the reference's checks)
    assert Lk == v.shape[1]
    assert q.shape[-1] == k.shape[-1] == v.shape[-1]
    head_dim = q.shape[-1]
    sm_scale = 1.0 / (head_dim ** 0.5)
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        # the reference's kernel has no backward; this one does (bf16 / f16)
        return ops.sqdk_attention(q, k, v, q_indices, sm_scale)
    return ops.sqdk_fwd(q, k, v, q_indices, sm_scale)
