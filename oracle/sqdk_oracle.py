"""numpy restatement of the reference's contextual-stream inference path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): used by the tests, the
smoke check and the bench's CPU baseline, never by the product path.

Each function cites the reference file:line it restates. Dtypes: every
function computes in float32 (the "repo's own PyTorch reference SQDK evaluated
in fp32"), except where the reference itself rounds to a narrower type on the
path (the router's ``noisy_logits`` tensor, which lives in the module dtype),
which ``round_to`` reproduces bit for bit.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

# ----------------------------------------------------------------------------
# Rounding helpers (bit-exact IEEE round-to-nearest-even)
# ----------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round to nearest, ties to even) and
    return them as float32. NaN stays NaN (quieted), infinities stay."""
    a = np.ascontiguousarray(x, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    r = r.astype(np.uint32)
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, (a.view(np.uint32) | 0x00400000) & 0xFFFF0000, r).astype(np.uint32)
    return r.view(F32).reshape(a.shape)


def f16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to IEEE half (numpy's cast is RNE) and back."""
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` in {"f32", "bf16", "f16"}."""
    if dtype == "f32":
        return np.asarray(x, dtype=F32)
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "f16":
        return f16_round(x)
    raise ValueError(f"unknown dtype {dtype!r}")


# ----------------------------------------------------------------------------
# Router (hspmn_v2_1.py:95-122, eval branch)
# ----------------------------------------------------------------------------


def router_k(S: int, target_sparsity: float) -> int:
    """``k = max(1, int(S * self.target_sparsity.item()))`` (hspmn_v2_1.py:112).

    ``target_sparsity`` is the buffer's value *after* the module dtype cast
    (0.2 in a bf16 module is 0.2001953125, so S=4096 gives k=820)."""
    return max(1, int(S * float(target_sparsity)))


def noisy_logits(logits: np.ndarray, temp: float, dtype: str) -> np.ndarray:
    """``noisy_logits = logits / temp`` in eval mode (hspmn_v2_1.py:98,104-105).

    The division runs in float32 and is rounded to the result dtype, as
    PyTorch does for a bf16/f16 tensor divided by a one-element tensor."""
    q = np.asarray(logits, dtype=F32) / F32(temp)
    return round_to(q, dtype)


def gate_logits_fp32(x: np.ndarray, w: np.ndarray, bias: float | None, dtype: str) -> np.ndarray:
    """The router gate ``logits = x . w + b`` (hspmn_v2_1.py:84,96) with float32
    logits, in the summation order the library defines for it.

    ``x`` [..., D] and ``w`` [D] hold values of ``dtype`` (as float32 arrays);
    ``bias`` is the bias value or None. Order: the row is cut into vectors of
    E elements (E = 4 for "f32", 8 for 16-bit types); vector v belongs to
    lane v % 32, which keeps one float32 accumulator per slot e and adds
    ``x * w`` to it by a fused multiply-add over its vectors in ascending
    order; slots are summed as a pairwise tree, the 32 lanes by a xor
    butterfly (offsets 16, 8, 4, 2, 1), and the bias is added last.

    Each fused multiply-add is formed as a float64 product plus a float64 sum
    rounded once to float32. For 16-bit inputs that is the exact fma: the
    product is exact in float32, and the float64 sum is too close to the
    exact one for the final rounding to differ. For "f32" inputs the float64
    sum can round before the float32 rounding, so agreement there is to the
    summation error bound only."""
    x = np.asarray(x, dtype=F32)
    w = np.asarray(w, dtype=F32)
    D = x.shape[-1]
    E = 4 if dtype == "f32" else 8
    if D % E:
        raise ValueError(f"D={D} is not a multiple of {E}")
    lead = x.shape[:-1]
    xv = x.reshape(-1, D // E, E).astype(np.float64)
    wv = w.reshape(D // E, E).astype(np.float64)
    nvec = D // E
    R = xv.shape[0]
    acc = np.zeros((R, 32, E), dtype=F32)
    for j in range((nvec + 31) // 32):
        v0, v1 = 32 * j, min(32 * j + 32, nvec)
        n = v1 - v0
        prod = xv[:, v0:v1, :] * wv[v0:v1, :]
        acc[:, :n, :] = (acc[:, :n, :].astype(np.float64) + prod).astype(F32)
    a = acc
    if E == 4:
        t = (a[..., 0] + a[..., 1]) + (a[..., 2] + a[..., 3])
    else:
        t = ((a[..., 0] + a[..., 1]) + (a[..., 2] + a[..., 3])) + ((a[..., 4] + a[..., 5]) + (a[..., 6] + a[..., 7]))
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        t = t + t[:, lanes ^ o]
    out = t[:, 0] + F32(0.0 if bias is None else bias)
    return out.astype(F32).reshape(lead)


def gate_error_bound(x: np.ndarray, w: np.ndarray, bias: float | None) -> np.ndarray:
    """Upper bound on |fp32 gate logit - exact x . w + b| for any summation
    order: a sum of D + 1 terms formed by at most D + 1 roundings is off by
    at most gamma_(D+1) * (sum |x w| + |b|), gamma_n = n u / (1 - n u) with
    u = 2^-24 (1.01 n u covers it for n u < 0.01), plus 2^-149 per rounding
    for results in the subnormal range."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    n = x.shape[-1] + 1
    mag = np.abs(x) @ np.abs(w) + (0.0 if bias is None else abs(float(bias)))
    return 1.01 * n * 2.0 ** -24 * mag + n * 2.0 ** -149


def orderable_keys(noisy: np.ndarray, dtype: str) -> np.ndarray:
    """Map values to unsigned keys whose integer order is the selection order.

    Positive values get the sign bit set, negative values are bit-inverted and
    every NaN maps to the largest key (as torch.topk's radix select does).
    Keys are uint32; 16-bit dtypes use the low 16 bits only."""
    a = np.asarray(noisy, dtype=F32)
    if dtype == "f32":
        bits = a.view(np.uint32).astype(np.uint64)
        width = 32
    elif dtype == "bf16":
        bits = (a.view(np.uint32) >> 16).astype(np.uint64)
        width = 16
    elif dtype == "f16":
        bits = a.astype(np.float16).view(np.uint16).astype(np.uint64)
        width = 16
    else:
        raise ValueError(dtype)
    sign = np.uint64(1 << (width - 1))
    full = np.uint64((1 << width) - 1)
    key = np.where(bits & sign, (~bits) & full, bits | sign)
    key = np.where(np.isnan(a), full, key)
    return key.astype(np.uint32)


def router_topk(noisy: np.ndarray, k: int, dtype: str):
    """Top-k of each row of ``noisy`` [B,S], then indices sorted ascending and
    the boolean mask (hspmn_v2_1.py:113-120).

    Ranking: larger value first; among equal values (equal keys) the lower
    position first. ``torch.topk(sorted=False)`` leaves tie order unspecified;
    this rule is the library's definition and the CUDA kernel implements the
    same one. Returns (indices int64 [B,k], mask bool [B,S])."""
    noisy = np.asarray(noisy, dtype=F32)
    B, S = noisy.shape
    if not (1 <= k <= S):
        raise ValueError(f"k={k} outside [1, S={S}]")
    keys = orderable_keys(noisy, dtype).astype(np.int64)
    pos = np.arange(S, dtype=np.int64)
    idx = np.empty((B, k), dtype=np.int64)
    mask = np.zeros((B, S), dtype=bool)
    for b in range(B):
        order = np.lexsort((pos, -keys[b]))  # primary: key desc, then position asc
        sel = np.sort(order[:k])
        idx[b] = sel
        mask[b, sel] = True
    return idx, mask


# ----------------------------------------------------------------------------
# Gather / scatter (hspmn_v2_1.py:176-198)
# ----------------------------------------------------------------------------


def gather_rows(q_t: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """``q_sel[b,i,...] = q_t[b, idx[b,i], ...]`` (hspmn_v2_1.py:185-186)."""
    B = q_t.shape[0]
    return np.stack([q_t[b][idx[b]] for b in range(B)])


def scatter_rows(o: np.ndarray, idx: np.ndarray, S: int) -> np.ndarray:
    """``out = zeros_like(q_t); out.scatter_(1, idx, o)`` (hspmn_v2_1.py:195-196)."""
    B = o.shape[0]
    out = np.zeros((B, S) + o.shape[2:], dtype=o.dtype)
    for b in range(B):
        out[b, idx[b]] = o[b]
    return out


# ----------------------------------------------------------------------------
# SQDK attention (test_kernels_v2_1.py:34-65 generalised to GQA as the Flex
# path defines it, hspmn_v2_1.py:200-216 with enable_gqa)
# ----------------------------------------------------------------------------


def sqdk_fp32(q_sel, k, v, idx, sm_scale: float | None = None) -> np.ndarray:
    """Sparse-query dense-key causal attention in float32.

    q_sel [B,K,H,hd]; k, v [B,S,Hkv,hd]; idx [B,K] original query positions.
    Query head h reads key/value head ``h // (H // Hkv)``. Query i attends to
    key positions ``<= idx[b,i]`` with softmax scale ``hd ** -0.5``
    (kernels_v2_1.py:160, masked as at test_kernels_v2_1.py:54-59).
    Returns o [B,K,H,hd] float32."""
    q_sel = np.asarray(q_sel, dtype=F32)
    k = np.asarray(k, dtype=F32)
    v = np.asarray(v, dtype=F32)
    B, K, H, hd = q_sel.shape
    S, Hkv = k.shape[1], k.shape[2]
    G = H // Hkv
    scale = F32(1.0 / math.sqrt(hd)) if sm_scale is None else F32(sm_scale)
    out = np.empty((B, K, H, hd), dtype=F32)
    kpos = np.arange(S)
    for b in range(B):
        allowed = kpos[None, :] <= idx[b][:, None]  # [K,S]
        for h in range(H):
            g = h // G
            s = (q_sel[b, :, h, :] @ k[b, :, g, :].T) * scale
            s = np.where(allowed, s, -np.inf).astype(F32)
            m = s.max(axis=1, keepdims=True)
            with np.errstate(invalid="ignore"):
                p = np.exp(s - m)
            p = np.where(allowed, p, 0.0).astype(F32)
            l = p.sum(axis=1, keepdims=True)
            with np.errstate(invalid="ignore", divide="ignore"):
                out[b, :, h, :] = (p @ v[b, :, g, :]) / l
    return out


def sqdk_bwd_fp32(q_sel, k, v, idx, d_o, sm_scale: float | None = None):
    """Gradients of ``sqdk_fp32`` for the output gradient ``d_o`` [B,K,H,hd],
    in float32: the backward of the reference's training path, whose
    FlexAttention mask (q_idx >= kv_idx) & mask[b, q_idx] with enable_gqa
    (hspmn_v2_1.py:200-216) is this attention over the selected rows.

    Per (b, h): P = softmax of the masked scaled scores, O = P V,
    dP = dO V^T, D = rowsum(dO * O), dS = P (dP - D); dq = scale dS K,
    dk = scale dS^T Q and dv = P^T dO, dk and dv summed over the query heads
    that read each key/value head. Returns (dq [B,K,H,hd], dk, dv [B,S,Hkv,hd],
    lse [B,K,H]), lse the natural-log log-sum-exp of each row's scaled scores."""
    q_sel = np.asarray(q_sel, dtype=F32)
    k = np.asarray(k, dtype=F32)
    v = np.asarray(v, dtype=F32)
    d_o = np.asarray(d_o, dtype=F32)
    B, K, H, hd = q_sel.shape
    S, Hkv = k.shape[1], k.shape[2]
    G = H // Hkv
    scale = F32(1.0 / math.sqrt(hd)) if sm_scale is None else F32(sm_scale)
    dq = np.zeros_like(q_sel)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    lse = np.zeros((B, K, H), dtype=F32)
    kpos = np.arange(S)
    for b in range(B):
        allowed = kpos[None, :] <= idx[b][:, None]
        for h in range(H):
            g = h // G
            s = (q_sel[b, :, h, :] @ k[b, :, g, :].T) * scale
            s = np.where(allowed, s, -np.inf).astype(F32)
            m = s.max(axis=1, keepdims=True)
            p = np.where(allowed, np.exp(s - m), 0.0).astype(F32)
            l = p.sum(axis=1, keepdims=True)
            p = p / l
            lse[b, :, h] = (m + np.log(l))[:, 0]
            o = p @ v[b, :, g, :]
            dp = d_o[b, :, h, :] @ v[b, :, g, :].T
            delta = (d_o[b, :, h, :] * o).sum(axis=1, keepdims=True)
            ds = p * (dp - delta)
            dq[b, :, h, :] = scale * (ds @ k[b, :, g, :])
            dk[b, :, g, :] += scale * (ds.T @ q_sel[b, :, h, :])
            dv[b, :, g, :] += p.T @ d_o[b, :, h, :]
    return dq, dk, dv, lse


def attention_flops(idx: np.ndarray, H: int, hd: int) -> float:
    """Algorithmic SQDK FLOPs: 2*hd for q.k plus 2*hd for p.v per unmasked
    (query, key) pair, summed over heads: ``4*hd*H*sum(idx+1)``."""
    return float(4 * hd * H * (np.asarray(idx, dtype=np.int64) + 1).sum())


# ----------------------------------------------------------------------------
# Full HSPMNBlock eval forward (hspmn_v2_1.py:236-238), the block-level oracle
# ----------------------------------------------------------------------------


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """nn.RMSNorm with eps=None uses finfo(dtype).eps of the module dtype."""
    x = np.asarray(x, dtype=F32)
    ms = (x * x).mean(axis=-1, keepdims=True)
    return (x / np.sqrt(ms + F32(eps))) * np.asarray(w, dtype=F32)


def rope_tables(S: int, hd: int, base: float):
    """cos/sin tables [S,hd] (hspmn_v2_1.py:45-54)."""
    inv = F32(1.0) / (F32(base) ** (np.arange(0, hd, 2, dtype=F32) / F32(hd)))
    t = np.arange(S, dtype=F32)
    f = np.outer(t, inv).astype(F32)
    emb = np.concatenate([f, f], axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x [B,S,h,hd]; ``x*cos + rotate_half(x)*sin`` (hspmn_v2_1.py:34-38,66-68)."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * cos[None, :, None, :] + rot * sin[None, :, None, :]


def rope_rounded(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """``(x*cos) + (rotate_half(x)*sin)`` (hspmn_v2_1.py:34-38,66-68) evaluated
    as the reference's three tensor ops in ``dtype``: each product and the sum
    computed in float32 and rounded to ``dtype``. x [..., hd] with values of
    ``dtype``; cos/sin broadcastable, already rounded to ``dtype``."""
    x = np.asarray(x, dtype=F32)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    t1 = round_to(x * np.asarray(cos, F32), dtype)
    t2 = round_to(rot * np.asarray(sin, F32), dtype)
    return round_to(t1 + t2, dtype)


def _silu(x):
    return x / (F32(1.0) + np.exp(-x))


def block_forward(p: dict, x: np.ndarray, num_heads: int, num_kv_heads: int,
                  target_sparsity: float, rope_base: float, eps: float,
                  noisy_dtype: str = "f32", indices: np.ndarray | None = None):
    """HSPMNBlock.forward in eval mode, float32 arithmetic.

    ``p`` holds the block's state_dict entries as float32 numpy arrays.
    ``indices`` may be given to force the router's selection (used when the
    logits under test were computed by a different GEMM). Returns
    (out [B,S,D], indices, mask, logits)."""
    x = np.asarray(x, dtype=F32)
    B, S, D = x.shape
    H, Hkv = num_heads, num_kv_heads
    hd = D // H
    # router (hspmn_v2_1.py:95-122)
    logits = (x @ p["router.gate.weight"].T)[..., 0] + p["router.gate.bias"][0]
    temp = float(np.clip(np.exp(p["router.log_temp"][0]), 0.1, 2.0))
    k = router_k(S, target_sparsity)
    if indices is None:
        noisy = noisy_logits(logits, temp, noisy_dtype)
        indices, mask = router_topk(noisy, k, noisy_dtype)
    else:
        mask = np.zeros((B, S), dtype=bool)
        for b in range(B):
            mask[b, indices[b]] = True
    # reflexive stream (hspmn_v2_1.py:141-145)
    h = rms_norm(x, p["reflexive.norm.weight"], eps)
    cw = p["reflexive.conv.weight"][:, 0, :]  # [D,3]
    hp = np.pad(h, ((0, 0), (1, 1), (0, 0)))
    hc = hp[:, :-2] * cw[:, 0] + hp[:, 1:-1] * cw[:, 1] + hp[:, 2:] * cw[:, 2]
    mlp = (_silu(hc @ p["reflexive.gate_proj.weight"].T) * (hc @ p["reflexive.up_proj.weight"].T))
    refl = x + mlp @ p["reflexive.down_proj.weight"].T
    # attention (hspmn_v2_1.py:218-234, 176-198)
    xn = rms_norm(x, p["norm.weight"], eps)
    q = (xn @ p["q_proj.weight"].T).reshape(B, S, H, hd)
    kk = (xn @ p["k_proj.weight"].T).reshape(B, S, Hkv, hd)
    vv = (xn @ p["v_proj.weight"].T).reshape(B, S, Hkv, hd)
    cos, sin = rope_tables(S, hd, rope_base)
    q = apply_rope(q, cos, sin)
    kk = apply_rope(kk, cos, sin)
    q_sel = gather_rows(q, indices)
    o = sqdk_fp32(q_sel, kk, vv, indices)
    out = scatter_rows(o, indices, S).reshape(B, S, D)
    attn = out @ p["o_proj.weight"].T
    return (refl + attn).astype(F32), indices, mask, logits.astype(F32)
