"""Fused write-back path: RoPE fused into the row gather (bit-exact), the
in-place residual add of the routed rows (bit-exact), and the fused block
forward against the reference-order block and the oracle (tolerance)."""

import numpy as np
import pytest
import torch

import oracle
from hspmn_b200 import HSPMNBlock, HSPMNConfig, ops
from hspmn_b200.model import RotaryEmbedding, apply_rotary_pos_emb

pytestmark = pytest.mark.gpu
DEV = "cuda"
_NAME = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def _sorted_idx(B, S, K, g):
    return torch.stack([torch.randperm(S, generator=g)[:K].sort().values for _ in range(B)])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,hd", [(16, 128), (4, 64), (4, 16), (5, 48)])  # hd=48: column groups that do not divide 32
@pytest.mark.parametrize("by_position", [True, False])
def test_rope_gather_bit_exact(dtype, H, hd, by_position):
    B, S, K = 2, 700, 140
    g = torch.Generator().manual_seed(H * hd + int(by_position))
    rope = RotaryEmbedding(hd, 1024)
    q = torch.randn(B, S, H, hd, generator=g).to(dtype)
    idx = _sorted_idx(B, S, K, g)
    cos, sin = rope(q, S)
    src = q if by_position else torch.from_numpy(oracle.gather_rows(q.float().numpy(), idx.numpy())).to(dtype)
    out = ops.rope_gather_rows(src.to(DEV), idx.to(DEV), cos.to(DEV), sin.to(DEV), by_position)
    # oracle: per-op rounding restated in numpy
    c, s_ = cos[0, 0].float().numpy(), sin[0, 0].float().numpy()
    qg = oracle.gather_rows(q.float().numpy(), idx.numpy())
    ref = np.stack([oracle.rope_rounded(qg[b], c[idx[b].numpy()][:, None, :], s_[idx[b].numpy()][:, None, :],
                                        _NAME[dtype]) for b in range(B)])
    np.testing.assert_array_equal(out.float().cpu().numpy(), ref)
    # and the reference's own tensor ops on the device, then a gather
    qt = q.to(DEV).transpose(1, 2)
    q_rot, _ = apply_rotary_pos_emb(qt, qt, cos.to(DEV), sin.to(DEV))
    ref_t = torch.gather(q_rot.transpose(1, 2), 1, idx.to(DEV)[:, :, None, None].expand(-1, -1, H, hd))
    assert torch.equal(out, ref_t)


@pytest.mark.parametrize("dtype,scale", [(torch.bfloat16, 1e-38), (torch.float16, 1e-5), (torch.bfloat16, 3e37),
                                         (torch.float16, 3e4)])
def test_rope_gather_subnormal_and_huge(dtype, scale):
    """Products and sums that land in the type's subnormal range or overflow:
    the 16-bit paths must round (and saturate) exactly as the reference's ops."""
    B, S, H, hd, K = 1, 256, 2, 64, 64
    g = torch.Generator().manual_seed(3)
    rope = RotaryEmbedding(hd, 512)
    q = (torch.randn(B, S, H, hd, generator=g) * scale).to(dtype)
    q[0, :8] = 0.0
    q[0, 8:16] = -0.0
    idx = _sorted_idx(B, S, K, g)
    cos, sin = rope(q, S)
    out = ops.rope_gather_rows(q.to(DEV), idx.to(DEV), cos.to(DEV), sin.to(DEV), True)
    qt = q.to(DEV).transpose(1, 2)
    q_rot, _ = apply_rotary_pos_emb(qt, qt, cos.to(DEV), sin.to(DEV))
    ref_t = torch.gather(q_rot.transpose(1, 2), 1, idx.to(DEV)[:, :, None, None].expand(-1, -1, H, hd))
    same = (out.view(torch.int16) == ref_t.view(torch.int16)) | (torch.isnan(out) & torch.isnan(ref_t))
    assert bool(same.all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("B,S,H,hd,pos0", [(3, 701, 4, 128, 0), (2, 257, 16, 64, 100), (1, 33, 3, 16, 7),
                                           (4, 1, 4, 128, 0), (2, 65, 5, 48, 3)])
def test_rope_rows_bit_exact(dtype, B, S, H, hd, pos0):
    """RoPE over every row (position = pos0 + row), bit-identical to the
    reference's three tensor ops on the same [B,H,S,hd] view; odd row counts
    leave a lone last row for a warp."""
    g = torch.Generator().manual_seed(B * S + hd)
    rope = RotaryEmbedding(hd, 1024)
    k = torch.randn(B, S, H, hd, generator=g).to(dtype)
    cos, sin = rope(k, pos0 + S)
    out = ops.rope_rows(k.to(DEV), cos.to(DEV), sin.to(DEV), pos0)
    kt = k.to(DEV).transpose(1, 2)
    c, s_ = cos[:, :, pos0:pos0 + S].to(DEV), sin[:, :, pos0:pos0 + S].to(DEV)
    _, k_rot = apply_rotary_pos_emb(kt, kt, c, s_)
    assert torch.equal(out, k_rot.transpose(1, 2))
    # the numpy restatement of the per-op rounding agrees
    ref = oracle.rope_rounded(k.float().numpy(), cos[0, 0, pos0:pos0 + S].float().numpy()[None, :, None, :],
                              sin[0, 0, pos0:pos0 + S].float().numpy()[None, :, None, :], _NAME[dtype])
    np.testing.assert_array_equal(out.float().cpu().numpy(), ref)


def test_rope_rows_strided_and_in_place():
    """A strided source (rows of a wider projection output) and dst == src
    through the C ABI."""
    import ctypes

    from hspmn_b200 import _native as N
    B, S, H, hd = 2, 300, 4, 128
    g = torch.Generator().manual_seed(9)
    rope = RotaryEmbedding(hd, 512)
    wide = torch.randn(B, S, 2 * H * hd, generator=g).to(torch.bfloat16).to(DEV)
    k = wide[:, :, :H * hd].view(B, S, H, hd)
    cos, sin = rope(k, S)
    cos2, sin2 = cos[0, 0].to(DEV).contiguous(), sin[0, 0].to(DEV).contiguous()
    expect = ops.rope_rows(k.contiguous(), cos2, sin2, 0)
    other = wide[:, :, H * hd:].clone()
    rc = N.lib().hspmn_rope_rows(ctypes.c_void_p(k.data_ptr()), k.stride(0), k.stride(1),
                                 ctypes.c_void_p(cos2.data_ptr()), ctypes.c_void_p(sin2.data_ptr()), hd, S, 0,
                                 ctypes.c_void_p(k.data_ptr()), k.stride(0), k.stride(1), B, S, H, hd, N.HSPMN_BF16,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(k, expect)
    assert torch.equal(wide[:, :, H * hd:], other)  # the rest of each row is left alone


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_scatter_add_rows_bit_exact(dtype):
    B, S, D, K = 3, 500, 256, 100
    g = torch.Generator().manual_seed(4)
    y = torch.randn(B, S, D, generator=g).to(dtype)
    src = torch.randn(B, K, D, generator=g).to(dtype)
    idx = _sorted_idx(B, S, K, g)
    yd = y.to(DEV)
    ops.scatter_add_rows_(yd, idx.to(DEV), src.to(DEV))
    full = torch.from_numpy(oracle.scatter_rows(src.float().numpy(), idx.numpy(), S))
    ref = oracle.round_to(y.float().numpy() + full.numpy(), _NAME[dtype])
    np.testing.assert_array_equal(yd.float().cpu().numpy(), ref)
    assert ops.device_errors() == 0


@pytest.mark.parametrize("dim,H,Hkv,S", [(2048, 16, 4, 4096), (512, 8, 2, 1000), (256, 4, 4, 512)])
def test_fused_block_matches_reference_order(dim, H, Hkv, S):
    torch.manual_seed(dim + S)
    block = HSPMNBlock(HSPMNConfig(dim=dim, num_heads=H, num_kv_heads=Hkv, max_seq_len=S))
    block = block.to(DEV, dtype=torch.bfloat16).eval()
    with torch.no_grad():
        block.router.gate.weight.normal_(0, dim ** -0.5)
    x = torch.randn(2, S, dim, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        y_fused, aux_f = block(x)
        block.sqdk_fused = False
        y_ref, aux_r = block(x)
    assert torch.equal(aux_f, aux_r)
    err = (y_fused.float() - y_ref.float()).abs()
    # only the routed rows differ (GEMM rounding of q_proj / o_proj on fewer rows)
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-4, (err.max().item(), err.mean().item())
    idx = block.router(x).indices
    unrouted = torch.ones(2, S, dtype=torch.bool, device=DEV)
    unrouted.scatter_(1, idx, False)
    assert torch.equal(y_fused[unrouted], y_ref[unrouted])


def test_fused_block_against_oracle_fp32():
    """float32 block, fused path, vs the oracle's fp32 block forward given the
    same router selection."""
    torch.manual_seed(5)
    dim, H, Hkv, S = 256, 4, 2, 384
    block = HSPMNBlock(HSPMNConfig(dim=dim, num_heads=H, num_kv_heads=Hkv, max_seq_len=S)).eval()
    with torch.no_grad():
        block.router.gate.weight.normal_(0, dim ** -0.5)
    params = {k: v.float().numpy() for k, v in block.state_dict().items()}
    block = block.to(DEV)
    x = torch.randn(2, S, dim)
    with torch.no_grad():
        y, _ = block(x.to(DEV))
        idx = block.router(x.to(DEV)).indices.cpu().numpy()
    ref, _, _, _ = oracle.block_forward(params, x.numpy(), H, Hkv, float(block.router.target_sparsity.item()),
                                        10000, float(np.finfo(np.float32).eps), indices=idx)
    err = np.abs(y.cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
