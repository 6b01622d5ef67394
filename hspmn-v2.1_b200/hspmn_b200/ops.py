"""torch-facing operators over the native library.

Each operator is a ``torch.library`` custom op (namespace ``hspmn``) with a
fake implementation, so ``torch.compile`` traces through it without a graph
break. All of them run on the caller's current CUDA stream, allocate their
outputs with the PyTorch caching allocator and never synchronise. CPU
tensors, a missing library or a non-B200 device raise: there is no fallback.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _native as N

_DTYPE_CODE = {torch.float32: N.HSPMN_F32, torch.float16: N.HSPMN_F16, torch.bfloat16: N.HSPMN_BF16}
_CODE_DTYPE = {v: k for k, v in _DTYPE_CODE.items()}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"hspmn: unsupported dtype {dt}; expected float32, float16 or bfloat16") from None


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError(
                "hspmn: the sm_100a kernels need CUDA tensors (there is no CPU path); got a tensor on "
                f"{t.device}")
        if t.device != dev:
            raise RuntimeError(f"hspmn: tensors on different devices ({dev} vs {t.device})")
    return dev


def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


class _on_device:
    """Make ``dev`` current for the native call (the library launches on the
    current device)."""

    def __init__(self, dev: torch.device):
        self.dev = dev
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev.index:
            self.prev = cur
            torch.cuda.set_device(self.dev)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


class LaunchStats:
    """Counts native kernel launches and, while a ``KernelTimer`` is active,
    records CUDA events around each one on the launching stream."""

    launches = 0
    timer = None


class KernelTimer:
    """Context manager: per-op CUDA-event timing of the native launches made
    inside it. ``results()`` (after a synchronize) gives, per op name, the
    launch count and the summed device milliseconds."""

    def __init__(self):
        self.events = {}

    def __enter__(self):
        LaunchStats.timer = self
        return self

    def __exit__(self, *exc):
        LaunchStats.timer = None
        return False

    def _begin(self, name: str, dev: torch.device):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        return ev

    def _end(self, name: str, dev: torch.device, start):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        self.events.setdefault(name, []).append((start, ev))

    def results(self):
        out = {}
        for name, pairs in self.events.items():
            ms = sum(a.elapsed_time(b) for a, b in pairs)
            out[name] = {"launches": len(pairs), "ms": ms}
        return out


class _launch:
    """Wraps one native call: an NVTX range named ``hspmn::<op>`` around it
    (so a timeline attributes the kernels), a launch count, and CUDA-event
    timing when a ``KernelTimer`` is active."""

    __slots__ = ("name", "dev", "start")

    def __init__(self, name: str, dev: torch.device):
        self.name, self.dev, self.start = name, dev, None

    def __enter__(self):
        torch.cuda.nvtx.range_push("hspmn::" + self.name)
        t = LaunchStats.timer
        if t is not None:
            self.start = t._begin(self.name, self.dev)

    def __exit__(self, exc_type, *exc):
        try:
            if exc_type is None:
                LaunchStats.launches += 1
                t = LaunchStats.timer
                if t is not None and self.start is not None:
                    t._end(self.name, self.dev, self.start)
        finally:
            torch.cuda.nvtx.range_pop()
        return False


def _rows_view(t: torch.Tensor, lead: int) -> Tuple[torch.Tensor, int]:
    """View ``t`` as [lead dims..., row] with densely packed rows; copies when
    the trailing dims are not one dense block. Returns (tensor, row_bytes)."""
    row_elems = 1
    for d in t.shape[lead:]:
        row_elems *= d
    expect = 1
    dense = True
    for d, s in zip(reversed(t.shape[lead:]), reversed(t.stride()[lead:])):
        if d != 1 and s != expect:
            dense = False
            break
        expect *= d
    if not dense:
        t = t.contiguous()
    return t, row_elems * t.element_size()


# ---------------------------------------------------------------------------
# router top-K
# ---------------------------------------------------------------------------


@torch.library.custom_op("hspmn::router_topk", mutates_args=())
def router_topk(logits: torch.Tensor, temp: Optional[torch.Tensor], k: int,
                noisy_dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """Selection step of TopKRouter.forward (hspmn_v2_1.py:104-105,112-120).

    ``noisy = (logits / temp)`` rounded to ``noisy_dtype`` (``temp`` a
    one-element tensor, or None for no division); per row the ``k`` largest
    noisy values (NaN largest, equal values: lower position first). Returns
    (indices int64 [B,k] ascending, mask bool [B,S])."""
    dev = _require_cuda(logits) if temp is None else _require_cuda(logits, temp)
    if logits.dim() != 2:
        raise ValueError(f"router_topk: logits must be [B,S], got {tuple(logits.shape)}")
    B, S = logits.shape
    if not (1 <= k <= S):
        raise ValueError(f"router_topk: k={k} outside [1, S={S}]")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    if temp is not None and temp.numel() != 1:
        raise ValueError("router_topk: temp must hold one element")
    indices = torch.empty((B, k), dtype=torch.int64, device=dev)
    mask = torch.empty((B, S), dtype=torch.bool, device=dev)
    with _on_device(dev), _launch("router_topk", dev):
        rc = N.lib().hspmn_router_topk(
            ctypes.c_void_p(logits.data_ptr()), dtype_code(logits.dtype), logits.stride(0),
            ctypes.c_void_p(temp.data_ptr() if temp is not None else 0),
            dtype_code(temp.dtype) if temp is not None else 0, dtype_code(noisy_dtype),
            B, S, k, ctypes.c_void_p(indices.data_ptr()), k, ctypes.c_void_p(mask.data_ptr()), S,
            _stream(dev))
        N.check(rc, "hspmn_router_topk")
    return indices, mask


@router_topk.register_fake
def _(logits, temp, k, noisy_dtype):
    B, S = logits.shape
    return (logits.new_empty((B, k), dtype=torch.int64), logits.new_empty((B, S), dtype=torch.bool))


@torch.library.custom_op("hspmn::gate_logits", mutates_args=())
def gate_logits(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    """TopKRouter's gate (hspmn_v2_1.py:84,96) with float32 logits:
    ``logits[b,s] = x[b,s,:] . weight + bias`` summed in fp32 in a fixed order
    and not rounded to x's dtype. ``weight`` is the Linear(dim, 1) weight
    ([1,D] or [D]), ``bias`` its [1] bias or None; both in x's dtype.
    Returns float32 [B,S]."""
    tensors = (x, weight) if bias is None else (x, weight, bias)
    dev = _require_cuda(*tensors)
    if x.dim() != 3:
        raise ValueError(f"gate_logits: x must be [B,S,D], got {tuple(x.shape)}")
    B, S, D = x.shape
    if weight.numel() != D:
        raise ValueError(f"gate_logits: weight has {weight.numel()} elements, expected D={D}")
    if bias is not None and bias.numel() != 1:
        raise ValueError("gate_logits: bias must hold one element")
    if any(t.dtype != x.dtype for t in tensors):
        raise TypeError("gate_logits: x, weight and bias must share one dtype")
    es = x.element_size()
    if x.stride(2) != 1 or (x.stride(0) * es) % 16 or (x.stride(1) * es) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
        if x.data_ptr() % 16:
            x = x.clone()
    weight = weight.reshape(D)
    if not weight.is_contiguous() or weight.data_ptr() % 16:
        weight = weight.clone(memory_format=torch.contiguous_format)
    logits = torch.empty((B, S), dtype=torch.float32, device=dev)
    with _on_device(dev), _launch("gate_logits", dev):
        rc = N.lib().hspmn_gate_logits(
            ctypes.c_void_p(x.data_ptr()), dtype_code(x.dtype), x.stride(0), x.stride(1),
            ctypes.c_void_p(weight.data_ptr()), ctypes.c_void_p(bias.data_ptr() if bias is not None else 0),
            B, S, D, ctypes.c_void_p(logits.data_ptr()), S, _stream(dev))
        N.check(rc, "hspmn_gate_logits")
    return logits


@gate_logits.register_fake
def _(x, weight, bias):
    return x.new_empty(x.shape[:2], dtype=torch.float32)


# ---------------------------------------------------------------------------
# gather / scatter of selected rows
# ---------------------------------------------------------------------------


@torch.library.custom_op("hspmn::gather_rows", mutates_args=())
def gather_rows(src: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """``out[b,i,...] = src[b, indices[b,i], ...]`` (hspmn_v2_1.py:185-186).

    ``src`` is [B,S,...]; each position's trailing dims form one row. The
    result is a new contiguous [B,K,...] tensor."""
    dev = _require_cuda(src, indices)
    if indices.dim() != 2 or indices.dtype != torch.int64 or indices.shape[0] != src.shape[0]:
        raise ValueError("gather_rows: indices must be int64 [B,K] matching src's batch")
    if indices.stride(1) != 1:
        indices = indices.contiguous()
    B, S = src.shape[0], src.shape[1]
    K = indices.shape[1]
    src, row_bytes = _rows_view(src, 2)
    out = torch.empty((B, K) + tuple(src.shape[2:]), dtype=src.dtype, device=dev)
    es = src.element_size()
    with _on_device(dev), _launch("gather_rows", dev):
        rc = N.lib().hspmn_gather_rows(
            ctypes.c_void_p(src.data_ptr()), src.stride(0) * es, src.stride(1) * es,
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0),
            ctypes.c_void_p(out.data_ptr()), K * row_bytes, row_bytes, B, S, K, row_bytes, _stream(dev))
        N.check(rc, "hspmn_gather_rows")
    return out


@gather_rows.register_fake
def _(src, indices):
    return src.new_empty((src.shape[0], indices.shape[1]) + tuple(src.shape[2:]))


@torch.library.custom_op("hspmn::scatter_rows", mutates_args=())
def scatter_rows(src: torch.Tensor, indices: torch.Tensor, seq_len: int) -> torch.Tensor:
    """``out = zeros([B,seq_len,...]); out[b, indices[b,i]] = src[b,i]``
    (hspmn_v2_1.py:195-196) in a single pass over ``out``.

    ``indices`` rows must be strictly ascending, as the router emits them."""
    dev = _require_cuda(src, indices)
    if indices.dim() != 2 or indices.dtype != torch.int64 or tuple(indices.shape) != tuple(src.shape[:2]):
        raise ValueError("scatter_rows: indices must be int64 [B,K] matching src[:2]")
    if indices.stride(1) != 1:
        indices = indices.contiguous()
    B, K = indices.shape
    src, row_bytes = _rows_view(src, 2)
    out = torch.empty((B, seq_len) + tuple(src.shape[2:]), dtype=src.dtype, device=dev)
    es = src.element_size()
    with _on_device(dev), _launch("scatter_rows", dev):
        rc = N.lib().hspmn_scatter_rows(
            ctypes.c_void_p(src.data_ptr()), src.stride(0) * es, src.stride(1) * es,
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0),
            ctypes.c_void_p(out.data_ptr()), seq_len * row_bytes, row_bytes, B, seq_len, K, row_bytes,
            _stream(dev))
        N.check(rc, "hspmn_scatter_rows")
    return out


@scatter_rows.register_fake
def _(src, indices, seq_len):
    return src.new_empty((src.shape[0], seq_len) + tuple(src.shape[2:]))


@torch.library.custom_op("hspmn::rope_gather_rows", mutates_args=())
def rope_gather_rows(src: torch.Tensor, indices: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                     src_by_position: bool) -> torch.Tensor:
    """Selected query rows with the rotary embedding applied, bit-identical to
    ``gather(apply_rotary_pos_emb(q))`` (hspmn_v2_1.py:66-68,185-186).

    ``src`` is [B,S,H,hd] (all positions; ``src_by_position=True``) or
    [B,K,H,hd] (already the selected rows); ``cos``/``sin`` are the [S,hd]
    (or [1,1,S,hd]) tables in ``src``'s dtype; ``indices`` int64 [B,K] give
    the positions. Returns [B,K,H,hd]."""
    dev = _require_cuda(src, indices, cos, sin)
    if src.dim() != 4:
        raise ValueError("rope_gather_rows: src must be [B,S|K,H,hd]")
    B, _, H, hd = src.shape
    K = indices.shape[1]
    cos2, sin2 = cos.reshape(-1, hd), sin.reshape(-1, hd)
    if cos2.dtype != src.dtype or sin2.dtype != src.dtype:
        raise TypeError("rope_gather_rows: cos/sin must have src's dtype")
    if cos2.stride(1) != 1 or sin2.stride(1) != 1 or cos2.stride(0) != sin2.stride(0):
        cos2, sin2 = cos2.contiguous(), sin2.contiguous()
    S = cos2.shape[0]
    if indices.stride(1) != 1:
        indices = indices.contiguous()
    src, _ = _rows_view(src, 2)
    out = torch.empty((B, K, H, hd), dtype=src.dtype, device=dev)
    with _on_device(dev), _launch("rope_gather_rows", dev):
        rc = N.lib().hspmn_rope_gather_rows(
            ctypes.c_void_p(src.data_ptr()), src.stride(0), src.stride(1), int(src_by_position),
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0),
            ctypes.c_void_p(cos2.data_ptr()), ctypes.c_void_p(sin2.data_ptr()), cos2.stride(0),
            ctypes.c_void_p(out.data_ptr()), out.stride(0), out.stride(1), B, S, K, H, hd,
            dtype_code(src.dtype), _stream(dev))
        N.check(rc, "hspmn_rope_gather_rows")
    return out


@rope_gather_rows.register_fake
def _(src, indices, cos, sin, src_by_position):
    return src.new_empty((src.shape[0], indices.shape[1]) + tuple(src.shape[2:]))


@torch.library.custom_op("hspmn::rope_rows", mutates_args=())
def rope_rows(src: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos0: int) -> torch.Tensor:
    """Rotary embedding of every row of ``src`` [B,S,H,hd], row ``s`` at
    position ``pos0 + s``: bit-identical to the K side of
    ``apply_rotary_pos_emb`` (hspmn_v2_1.py:66-68,226-227) on the [B,S,H,hd]
    view, without an index array. ``cos``/``sin`` are the [L,hd] (or
    [1,1,L,hd]) tables in ``src``'s dtype with ``pos0 + S <= L``. Returns a
    new contiguous [B,S,H,hd] tensor."""
    dev = _require_cuda(src, cos, sin)
    if src.dim() != 4:
        raise ValueError("rope_rows: src must be [B,S,H,hd]")
    B, S, H, hd = src.shape
    cos2, sin2 = cos.reshape(-1, hd), sin.reshape(-1, hd)
    if cos2.dtype != src.dtype or sin2.dtype != src.dtype:
        raise TypeError("rope_rows: cos/sin must have src's dtype")
    if cos2.stride(1) != 1 or sin2.stride(1) != 1 or cos2.stride(0) != sin2.stride(0):
        cos2, sin2 = cos2.contiguous(), sin2.contiguous()
    if pos0 < 0 or pos0 + S > cos2.shape[0]:
        raise ValueError(f"rope_rows: positions [{pos0}, {pos0 + S}) outside the {cos2.shape[0]}-row table")
    src, _ = _rows_view(src, 2)
    out = torch.empty((B, S, H, hd), dtype=src.dtype, device=dev)
    with _on_device(dev), _launch("rope_rows", dev):
        rc = N.lib().hspmn_rope_rows(
            ctypes.c_void_p(src.data_ptr()), src.stride(0), src.stride(1),
            ctypes.c_void_p(cos2.data_ptr()), ctypes.c_void_p(sin2.data_ptr()), cos2.stride(0), cos2.shape[0],
            int(pos0), ctypes.c_void_p(out.data_ptr()), out.stride(0), out.stride(1), B, S, H, hd,
            dtype_code(src.dtype), _stream(dev))
        N.check(rc, "hspmn_rope_rows")
    return out


@rope_rows.register_fake
def _(src, cos, sin, pos0):
    return src.new_empty(src.shape)


@torch.library.custom_op("hspmn::scatter_add_rows_", mutates_args=("dst",))
def scatter_add_rows_(dst: torch.Tensor, indices: torch.Tensor, src: torch.Tensor) -> None:
    """In place ``dst[b, indices[b,i]] += src[b,i]`` in ``dst``'s dtype (the
    residual add of hspmn_v2_1.py:238 restricted to the selected rows).
    ``dst`` [B,S,...] with dense rows, ``src`` [B,K,...]."""
    dev = _require_cuda(dst, indices, src)
    if src.dtype != dst.dtype:
        raise TypeError("scatter_add_rows_: src and dst dtypes differ")
    B, S = dst.shape[0], dst.shape[1]
    K = indices.shape[1]
    row = 1
    for d in dst.shape[2:]:
        row *= d
    if not dst.is_contiguous():
        raise ValueError("scatter_add_rows_: dst must be contiguous")
    if indices.stride(1) != 1:
        indices = indices.contiguous()
    src = src.contiguous()
    with _on_device(dev), _launch("scatter_add_rows", dev):
        rc = N.lib().hspmn_scatter_add_rows(
            ctypes.c_void_p(src.data_ptr()), src.stride(0), src.stride(1),
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0),
            ctypes.c_void_p(dst.data_ptr()), dst.stride(0), dst.stride(1), B, S, K, row,
            dtype_code(dst.dtype), _stream(dev))
        N.check(rc, "hspmn_scatter_add_rows")


@scatter_add_rows_.register_fake
def _(dst, indices, src):
    return None


# ---------------------------------------------------------------------------
# SQDK attention
# ---------------------------------------------------------------------------


def _sqdk_operand(t: torch.Tensor) -> torch.Tensor:
    es = t.element_size()
    if t.stride(-1) != 1 or any((s * es) % 16 for s in t.stride()[:-1]) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _check_sqdk_shapes(name: str, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       indices: torch.Tensor) -> None:
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"{name}: q, k, v must be 4-D ([B,K,H,hd] / [B,S,Hkv,hd])")
    B, K, H, hd = q.shape
    Hkv = k.shape[2]
    if tuple(v.shape) != tuple(k.shape) or k.shape[0] != B or k.shape[3] != hd:
        raise ValueError(f"{name}: shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if tuple(indices.shape) != (B, K) or indices.dtype != torch.int64:
        raise ValueError(f"{name}: indices must be int64 [B,K]")
    if H % Hkv != 0:
        raise ValueError(f"{name}: num_heads {H} is not a multiple of num_kv_heads {Hkv}")


def _sqdk_workspace(dev: torch.device, B: int, K: int, S: int, H: int, Hkv: int, hd: int):
    with _on_device(dev):
        ws_bytes = int(N.lib().hspmn_sqdk_workspace_size(B, K, S, H, Hkv, hd))
    if ws_bytes < 0:
        raise N.HSPMNNativeError("hspmn_sqdk_workspace_size: device query failed")
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
    return ws, ws_bytes


@torch.library.custom_op("hspmn::sqdk_fwd", mutates_args=())
def sqdk_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
             sm_scale: float) -> torch.Tensor:
    """Sparse-query dense-key causal attention (kernels_v2_1.py:11-180).

    q [B,K,H,hd]; k, v [B,S,Hkv,hd] with H % Hkv == 0 (query head h reads
    K/V head h // (H // Hkv)); indices int64 [B,K] original positions. Returns
    o [B,K,H,hd] in q's dtype. bf16/f16 run natively; float32 operands are
    rounded to bf16 for the tensor cores and the result is returned as float32."""
    dev = _require_cuda(q, k, v, indices)
    _check_sqdk_shapes("sqdk_fwd", q, k, v, indices)
    B, K, H, hd = q.shape
    S, Hkv = k.shape[1], k.shape[2]
    out_dtype = q.dtype
    if q.dtype == torch.float32:
        q, k, v = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"sqdk_fwd: q/k/v dtypes {q.dtype}/{k.dtype}/{v.dtype} unsupported")
    q, k, v = _sqdk_operand(q), _sqdk_operand(k), _sqdk_operand(v)
    o = torch.empty((B, K, H, hd), dtype=q.dtype, device=dev)
    ws, ws_bytes = _sqdk_workspace(dev, B, K, S, H, Hkv, hd)
    with _on_device(dev), _launch("sqdk_fwd", dev):
        rc = N.lib().hspmn_sqdk_fwd(
            ctypes.c_void_p(q.data_ptr()), N.i64_array(q.stride()),
            ctypes.c_void_p(k.data_ptr()), N.i64_array(k.stride()),
            ctypes.c_void_p(v.data_ptr()), N.i64_array(v.stride()),
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0), indices.stride(1),
            ctypes.c_void_p(o.data_ptr()), N.i64_array(o.stride()),
            B, K, S, H, Hkv, hd, dtype_code(q.dtype), float(sm_scale),
            ctypes.c_void_p(ws.data_ptr() if ws is not None else 0), ws_bytes, _stream(dev))
        N.check(rc, "hspmn_sqdk_fwd")
    return o if o.dtype == out_dtype else o.to(out_dtype)


@sqdk_fwd.register_fake
def _(q, k, v, indices, sm_scale):
    return torch.empty_like(q, memory_format=torch.contiguous_format)


# ---------------------------------------------------------------------------
# SQDK attention, training: forward with log-sum-exp, backward
# ---------------------------------------------------------------------------


@torch.library.custom_op("hspmn::sqdk_fwd_lse", mutates_args=())
def sqdk_fwd_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                 sm_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """``sqdk_fwd`` that also returns each row's log-sum-exp of the scaled
    scores (float32 [B,K,H], natural log), which ``sqdk_bwd`` needs. q, k, v
    in bf16 or f16."""
    dev = _require_cuda(q, k, v, indices)
    _check_sqdk_shapes("sqdk_fwd_lse", q, k, v, indices)
    B, K, H, hd = q.shape
    S, Hkv = k.shape[1], k.shape[2]
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"sqdk_fwd_lse: q/k/v dtypes {q.dtype}/{k.dtype}/{v.dtype} unsupported (bf16 or f16)")
    o = torch.empty((B, K, H, hd), dtype=q.dtype, device=dev)
    lse = torch.empty((B, K, H), dtype=torch.float32, device=dev)
    if B == 0 or K == 0:
        return o, lse  # no selected query: nothing to attend
    q, k, v = _sqdk_operand(q), _sqdk_operand(k), _sqdk_operand(v)
    ws, ws_bytes = _sqdk_workspace(dev, B, K, S, H, Hkv, hd)
    with _on_device(dev), _launch("sqdk_fwd", dev):
        rc = N.lib().hspmn_sqdk_fwd_lse(
            ctypes.c_void_p(q.data_ptr()), N.i64_array(q.stride()),
            ctypes.c_void_p(k.data_ptr()), N.i64_array(k.stride()),
            ctypes.c_void_p(v.data_ptr()), N.i64_array(v.stride()),
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0), indices.stride(1),
            ctypes.c_void_p(o.data_ptr()), N.i64_array(o.stride()),
            ctypes.c_void_p(lse.data_ptr()), K * H, H,
            B, K, S, H, Hkv, hd, dtype_code(q.dtype), float(sm_scale),
            ctypes.c_void_p(ws.data_ptr() if ws is not None else 0), ws_bytes, _stream(dev))
        N.check(rc, "hspmn_sqdk_fwd_lse")
    return o, lse


@sqdk_fwd_lse.register_fake
def _(q, k, v, indices, sm_scale):
    B, K, H, _ = q.shape
    return torch.empty_like(q, memory_format=torch.contiguous_format), q.new_empty((B, K, H), dtype=torch.float32)


@torch.library.custom_op("hspmn::sqdk_bwd", mutates_args=())
def sqdk_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor, o: torch.Tensor,
             d_o: torch.Tensor, lse: torch.Tensor,
             sm_scale: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients (dq, dk, dv) of the SQDK attention for the output gradient
    ``d_o``, given the forward's output ``o`` and ``lse`` (``sqdk_fwd_lse``).
    The backward of the reference's training path (FlexAttention with the
    mask (q_idx >= kv_idx) & mask[b, q_idx], hspmn_v2_1.py:200-216).
    Each ``indices`` row must be ascending, as the router writes it (a key
    block finds its first query by binary search); a row out of order sets
    ``DEVERR_UNSORTED`` in ``device_errors()`` and its gradients are
    incomplete."""
    dev = _require_cuda(q, k, v, indices, o, d_o, lse)
    _check_sqdk_shapes("sqdk_bwd", q, k, v, indices)
    B, K, H, hd = q.shape
    S, Hkv = k.shape[1], k.shape[2]
    if not (q.dtype == k.dtype == v.dtype == o.dtype) or q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("sqdk_bwd: q, k, v and o must share one dtype, bf16 or f16")
    if tuple(o.shape) != tuple(q.shape) or tuple(d_o.shape) != tuple(q.shape) or tuple(lse.shape) != (B, K, H):
        raise ValueError("sqdk_bwd: o and d_o must be shaped like q, lse [B,K,H]")
    d_o = d_o.to(q.dtype)
    q, k, v, o, d_o = (_sqdk_operand(t) for t in (q, k, v, o, d_o))
    lse = lse.to(torch.float32).contiguous()
    dq = torch.empty((B, K, H, hd), dtype=q.dtype, device=dev)
    dk = torch.empty((B, S, Hkv, hd), dtype=q.dtype, device=dev)
    dv = torch.empty((B, S, Hkv, hd), dtype=q.dtype, device=dev)
    with _on_device(dev):
        ws_bytes = int(N.lib().hspmn_sqdk_bwd_workspace_size(B, K, H, hd))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
    with _on_device(dev), _launch("sqdk_bwd", dev):
        rc = N.lib().hspmn_sqdk_bwd(
            ctypes.c_void_p(q.data_ptr()), N.i64_array(q.stride()),
            ctypes.c_void_p(k.data_ptr()), N.i64_array(k.stride()),
            ctypes.c_void_p(v.data_ptr()), N.i64_array(v.stride()),
            ctypes.c_void_p(indices.data_ptr()), indices.stride(0), indices.stride(1),
            ctypes.c_void_p(o.data_ptr()), N.i64_array(o.stride()),
            ctypes.c_void_p(d_o.data_ptr()), N.i64_array(d_o.stride()),
            ctypes.c_void_p(lse.data_ptr()), K * H, H,
            ctypes.c_void_p(dq.data_ptr()), N.i64_array(dq.stride()),
            ctypes.c_void_p(dk.data_ptr()), N.i64_array(dk.stride()),
            ctypes.c_void_p(dv.data_ptr()), N.i64_array(dv.stride()),
            B, K, S, H, Hkv, hd, dtype_code(q.dtype), float(sm_scale),
            ctypes.c_void_p(ws.data_ptr() if ws is not None else 0), ws_bytes, _stream(dev))
        N.check(rc, "hspmn_sqdk_bwd")
    return dq, dk, dv


@sqdk_bwd.register_fake
def _(q, k, v, indices, o, d_o, lse, sm_scale):
    return (torch.empty_like(q, memory_format=torch.contiguous_format),
            torch.empty_like(k, memory_format=torch.contiguous_format),
            torch.empty_like(v, memory_format=torch.contiguous_format))


class _SqdkAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, indices, sm_scale):
        o, lse = sqdk_fwd_lse(q, k, v, indices, sm_scale)
        ctx.save_for_backward(q, k, v, indices, o, lse)
        ctx.sm_scale = sm_scale
        return o

    @staticmethod
    def backward(ctx, d_o):
        q, k, v, indices, o, lse = ctx.saved_tensors
        dq, dk, dv = sqdk_bwd(q, k, v, indices, o, d_o, lse, ctx.sm_scale)
        return dq, dk, dv, None, None


def sqdk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                   sm_scale: float) -> torch.Tensor:
    """Differentiable SQDK attention: ``sqdk_fwd_lse`` forward, ``sqdk_bwd``
    backward (bf16 / f16 operands). ``indices`` rows must be ascending for
    the backward (see ``sqdk_bwd``)."""
    return _SqdkAttention.apply(q, k, v, indices, sm_scale)


def device_errors(device: Optional[torch.device] = None, clear: bool = True) -> int:
    """Synchronise the current stream of ``device`` and return (and clear)
    the library's device flag word (``_native.DEVERR_*`` bits)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with _on_device(dev):
        return N.device_errors(torch.cuda.current_stream(dev).cuda_stream, clear)
