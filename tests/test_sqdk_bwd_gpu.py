"""SQDK backward kernel vs the oracle's fp32 backward.

Tolerance (the forward's attention contract scaled by the gradient's size):
for each of dq, dk, dv, max |g - g_fp32| <= 2e-2 * max(1, max |g_fp32|) and
mean |g - g_fp32| <= 2e-3 * max(1, mean |g_fp32|), from bf16/f16 inputs.
The forward's log-sum-exp within 1e-5 of the oracle's.
"""

import math
import types

import numpy as np
import pytest
import torch

import oracle
from hspmn_b200 import HSPMNBlock, HSPMNConfig, ops
from hspmn_b200.kernels import sparse_query_dense_key_attention

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, S, H, Hkv, hd, K, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, K, H, hd, generator=g).to(dtype)
    k = torch.randn(B, S, Hkv, hd, generator=g).to(dtype)
    v = torch.randn(B, S, Hkv, hd, generator=g).to(dtype)
    d_o = torch.randn(B, K, H, hd, generator=g).to(dtype)
    idx = torch.stack([torch.sort(torch.randperm(S, generator=g)[:K])[0] for _ in range(B)])
    return q, k, v, d_o, idx


def _close(name, got, ref):
    got = got.float().cpu().numpy()
    err = np.abs(got - ref)
    assert np.isfinite(got).all(), name
    assert err.max() <= 2e-2 * max(1.0, float(np.abs(ref).max())), (name, float(err.max()))
    assert err.mean() <= 2e-3 * max(1.0, float(np.abs(ref).mean())), (name, float(err.mean()))


def _run(q, k, v, d_o, idx):
    qd, kd, vd, dod, idd = (t.to(DEV) for t in (q, k, v, d_o, idx))
    scale = q.shape[-1] ** -0.5
    o, lse = ops.sqdk_fwd_lse(qd, kd, vd, idd, scale)
    dq, dk, dv = ops.sqdk_bwd(qd, kd, vd, idd, o, dod, lse, scale)
    assert ops.device_errors() == 0
    return o, lse, dq, dk, dv


@pytest.mark.parametrize("B,S,H,Hkv,hd,K", [
    (1, 256, 4, 2, 64, 40), (2, 300, 8, 2, 128, 60), (1, 512, 16, 4, 128, 102), (1, 200, 6, 2, 64, 50),
    (1, 130, 2, 2, 128, 33), (2, 1024, 16, 4, 128, 205), (1, 96, 4, 4, 48, 96), (1, 640, 8, 1, 96, 17),
    # CTA order in chunks of (sequence, head) pairs: 9 pairs at 32 key blocks are chunks of
    # 4, 4 and 1; 157 key blocks give chunks of one pair
    (3, 4096, 6, 3, 64, 100), (1, 20000, 2, 2, 64, 30)])
def test_sqdk_bwd_against_oracle(B, S, H, Hkv, hd, K):
    q, k, v, d_o, idx = _inputs(B, S, H, Hkv, hd, K, seed=S + K)
    o, lse, dq, dk, dv = _run(q, k, v, d_o, idx)
    qf, kf, vf, dof = (t.float().numpy() for t in (q, k, v, d_o))
    rdq, rdk, rdv, rlse = oracle.sqdk_bwd_fp32(qf, kf, vf, idx.numpy(), dof)
    assert np.abs(lse.cpu().numpy() - rlse).max() <= 1e-5
    _close("dq", dq, rdq)
    _close("dk", dk, rdk)
    _close("dv", dv, rdv)


def test_sqdk_bwd_f16():
    q, k, v, d_o, idx = _inputs(2, 384, 8, 2, 128, 77, seed=9, dtype=torch.float16)
    _, _, dq, dk, dv = _run(q, k, v, d_o, idx)
    qf, kf, vf, dof = (t.float().numpy() for t in (q, k, v, d_o))
    rdq, rdk, rdv, _ = oracle.sqdk_bwd_fp32(qf, kf, vf, idx.numpy(), dof)
    for name, got, ref in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        _close(name, got, ref)


def test_unsorted_indices_flagged():
    """The backward needs ascending index rows; a row out of order is
    reported through the device flag word (the forward's output stays
    correct: it takes any order). Sorted rows raise nothing."""
    from hspmn_b200 import _native as N
    q, k, v, d_o, idx = _inputs(1, 512, 8, 2, 128, 96, seed=21)
    bad = idx.clone()
    bad[0, 40], bad[0, 41] = idx[0, 41], idx[0, 40]
    qd, kd, vd, dod, bd = (t.to(DEV) for t in (q, k, v, d_o, bad))
    scale = 128 ** -0.5
    ops.device_errors()  # clear
    o, lse = ops.sqdk_fwd_lse(qd, kd, vd, bd, scale)
    assert ops.device_errors() == 0
    ref_o = oracle.sqdk_fp32(q.float().numpy(), k.float().numpy(), v.float().numpy(), bad.numpy())
    assert np.abs(o.float().cpu().numpy() - ref_o).max() <= 2e-2
    ops.sqdk_bwd(qd, kd, vd, bd, o, dod, lse, scale)
    assert ops.device_errors() & N.DEVERR_UNSORTED
    _run(q, k, v, d_o, idx)  # asserts a clean flag word for the sorted rows


def test_fwd_lse_output_equals_fwd():
    q, k, v, _, idx = _inputs(2, 512, 16, 4, 128, 102, seed=4)
    qd, kd, vd, idd = (t.to(DEV) for t in (q, k, v, idx))
    o, _ = ops.sqdk_fwd_lse(qd, kd, vd, idd, 128 ** -0.5)
    assert torch.equal(o, ops.sqdk_fwd(qd, kd, vd, idd, 128 ** -0.5))


def test_autograd_and_reference_entry_point():
    q, k, v, d_o, idx = _inputs(1, 512, 8, 2, 64, 100, seed=12)
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    idd, dod = idx.to(DEV), d_o.to(DEV)
    out = sparse_query_dense_key_attention(qd, kd, vd, idd)
    gq, gk, gv = torch.autograd.grad(out, (qd, kd, vd), dod)
    with torch.no_grad():
        o, lse = ops.sqdk_fwd_lse(qd, kd, vd, idd, 64 ** -0.5)
        dq, dk, dv = ops.sqdk_bwd(qd, kd, vd, idd, o, dod, lse, 64 ** -0.5)
    assert torch.equal(out.detach(), o)
    assert torch.equal(gq, dq) and torch.equal(gk, dk) and torch.equal(gv, dv)


def test_strided_kv_views_and_unseen_keys():
    """K/V read through transposed views; keys after the last selected
    position (and the whole K=0 case) get zero gradients."""
    q, k, v, d_o, idx = _inputs(1, 400, 4, 2, 64, 20, seed=5)
    idx = torch.sort(torch.randperm(150)[:20])[0].view(1, -1)  # nothing selected past 149
    kt = k.to(DEV).transpose(1, 2).contiguous().transpose(1, 2)
    vt = v.to(DEV).transpose(1, 2).contiguous().transpose(1, 2)
    qd, dod, idd = q.to(DEV), d_o.to(DEV), idx.to(DEV)
    o, lse = ops.sqdk_fwd_lse(qd, kt, vt, idd, 0.125)
    dq, dk, dv = ops.sqdk_bwd(qd, kt, vt, idd, o, dod, lse, 0.125)
    o2, lse2 = ops.sqdk_fwd_lse(qd, k.to(DEV), v.to(DEV), idd, 0.125)
    dq2, dk2, dv2 = ops.sqdk_bwd(qd, k.to(DEV), v.to(DEV), idd, o2, dod, lse2, 0.125)
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)
    last = int(idx.max())
    assert (dk[:, last + 1:] == 0).all() and (dv[:, last + 1:] == 0).all()
    empty = torch.zeros(1, 0, dtype=torch.int64, device=DEV)
    q0 = torch.zeros(1, 0, 4, 64, dtype=torch.bfloat16, device=DEV)
    o0, lse0 = ops.sqdk_fwd_lse(q0, kt, vt, empty, 0.125)
    dq0, dk0, dv0 = ops.sqdk_bwd(q0, kt, vt, empty, o0, o0, lse0, 0.125)
    assert dq0.numel() == 0 and (dk0 == 0).all() and (dv0 == 0).all()


def test_block_training_step_matches_dense_attention():
    """A bf16 block in training mode: forward + backward through the SQDK
    kernels give the same parameter gradients as the same block whose
    contextual stream is an fp32 dense masked attention (torch autograd),
    with the same router selection (same Gumbel noise)."""
    torch.manual_seed(0)
    cfg = HSPMNConfig(dim=512, num_heads=8, num_kv_heads=2, max_seq_len=1024)
    block = HSPMNBlock(cfg).to(DEV, dtype=torch.bfloat16).train()
    x = torch.randn(2, 1024, 512, device=DEV, dtype=torch.bfloat16)

    def grads():
        block.zero_grad(set_to_none=True)
        torch.manual_seed(123)  # same Gumbel noise -> same selection
        y, aux = block(x)
        (y.float().square().mean() + aux).backward()
        return {n: p.grad.float().clone() for n, p in block.named_parameters() if p.grad is not None}

    with ops.KernelTimer() as kt:
        g_sqdk = grads()
    torch.cuda.synchronize()
    names = kt.results()
    assert names.get("sqdk_fwd", {}).get("launches", 0) >= 1 and names.get("sqdk_bwd", {}).get("launches", 0) >= 1

    def dense(self, q, k, v, router_out, B, S, D):
        H, Hkv, hd = self.num_heads, self.num_kv_heads, self.head_dim
        idx = router_out.indices
        K = idx.shape[1]
        sel = idx[:, :, None, None].expand(B, K, H, hd)
        q_sel = torch.gather(q.transpose(1, 2), 1, sel).float()
        kk = k.transpose(1, 2).float().repeat_interleave(H // Hkv, dim=2)
        vv = v.transpose(1, 2).float().repeat_interleave(H // Hkv, dim=2)
        s = torch.einsum("bkhd,bshd->bhks", q_sel, kk) / math.sqrt(hd)
        allowed = torch.arange(S, device=q.device)[None, None, None, :] <= idx[:, None, :, None]
        p = torch.softmax(s.masked_fill(~allowed, float("-inf")), -1)
        attn = torch.einsum("bhks,bshd->bkhd", p, vv).to(q.dtype)
        out = torch.zeros_like(q.transpose(1, 2)).scatter(1, sel, attn)
        return self.o_proj(out.reshape(B, S, D))

    block._attention_sqdk_train = types.MethodType(dense, block)
    g_ref = grads()
    assert set(g_sqdk) == set(g_ref)
    for n in g_ref:
        a, r = g_sqdk[n], g_ref[n]
        rel = (a - r).norm() / r.norm().clamp_min(1e-30)
        assert rel <= 3e-2, (n, float(rel))


def test_lse_and_grads_on_a_launch_without_key_splits():
    """Enough tiles (16 sequences x 820 rows, H=16, Hkv=4) that the forward
    runs unsplit, so its own epilogue writes the log-sum-exp; sequences 0
    and 15 are checked against the oracle, lse and gradients."""
    B, S, H, Hkv, hd, K = 16, 4096, 16, 4, 128, 820
    q, k, v, d_o, idx = _inputs(B, S, H, Hkv, hd, K, seed=77)
    o, lse, dq, dk, dv = _run(q, k, v, d_o, idx)
    for b in (0, B - 1):
        sl = slice(b, b + 1)
        qf, kf, vf, dof = (t[sl].float().numpy() for t in (q, k, v, d_o))
        rdq, rdk, rdv, rlse = oracle.sqdk_bwd_fp32(qf, kf, vf, idx[sl].numpy(), dof)
        assert np.abs(lse[sl].cpu().numpy() - rlse).max() <= 1e-5
        _close("dq", dq[sl], rdq)
        _close("dk", dk[sl], rdk)
        _close("dv", dv[sl], rdv)
