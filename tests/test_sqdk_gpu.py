"""SQDK attention kernel vs the fp32 oracle and the reference's Flex goldens.

Tolerance (the path's attention contract): max |o - o_fp32| <= 2e-2 and
mean |o - o_fp32| <= 2e-3, o computed from bf16/f16 inputs.
"""

import numpy as np
import pytest
import torch

import oracle
from hspmn_b200 import ops
from hspmn_b200.kernels import sparse_query_dense_key_attention
from tests import golden_io as G

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def check(o: torch.Tensor, ref: np.ndarray, tag=""):
    got = o.float().cpu().numpy()
    assert np.isfinite(got).all(), tag
    err = np.abs(got - ref)
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, f"{tag} max={err.max():.3e} mean={err.mean():.3e}"
    return err


def make_case(B, S, H, Hkv, hd, K, dtype, seed, sort=True, first_zero=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, H, hd, generator=g).to(dtype)
    k = torch.randn(B, S, Hkv, hd, generator=g).to(dtype)
    v = torch.randn(B, S, Hkv, hd, generator=g).to(dtype)
    idx = torch.stack([torch.randperm(S, generator=g)[:K] for _ in range(B)])
    if sort:
        idx = idx.sort(dim=1).values
    if first_zero:
        idx[:, 0] = 0
        idx = idx.sort(dim=1).values if sort else idx
    return q, k, v, idx


def run_case(q, k, v, idx):
    qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
    q_sel = oracle.gather_rows(q.float().numpy(), idx.numpy())
    ref = oracle.sqdk_fp32(q_sel, kf, vf, idx.numpy())
    q_sel_d = torch.from_numpy(q_sel).to(q.dtype).to(DEV)
    o = ops.sqdk_fwd(q_sel_d, k.to(DEV), v.to(DEV), idx.to(DEV), q.shape[-1] ** -0.5)
    assert o.dtype == q.dtype and tuple(o.shape) == tuple(q_sel.shape)
    return o, ref


@pytest.mark.parametrize("name", ["sqdk_cfg1_B2_S512_H4_hd64.npz", "sqdk_gqa_B1_S256_H8_Hkv2_hd128.npz",
                                  "sqdk_gqa3_B1_S200_H6_Hkv2_hd64.npz"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_against_reference_flex_golden(name, dtype):
    fx = G.load(name)
    q, k, v = G.sqdk_inputs(fx)
    idx = torch.from_numpy(fx["indices"])
    q_sel = torch.from_numpy(oracle.gather_rows(q, fx["indices"]))
    o = sparse_query_dense_key_attention(q_sel.to(dtype).to(DEV), torch.from_numpy(k).to(dtype).to(DEV),
                                         torch.from_numpy(v).to(dtype).to(DEV), idx.to(DEV))
    check(o, fx["out_sel"], name)
    assert ops.device_errors() == 0


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("H,Hkv", [(4, 4), (8, 2), (16, 4), (16, 1), (6, 2), (12, 4), (16, 16)])
def test_gqa_grid(hd, H, Hkv):
    q, k, v, idx = make_case(2, 333, H, Hkv, hd, 67, torch.bfloat16, seed=H * 100 + Hkv + hd)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, f"H={H} Hkv={Hkv} hd={hd}")


@pytest.mark.parametrize("B,S,K", [(1, 1, 1), (1, 63, 5), (1, 64, 64), (2, 65, 65), (1, 130, 1),
                                   (3, 1000, 200), (1, 4096, 820)])
def test_shapes_and_edges(B, S, K):
    q, k, v, idx = make_case(B, S, 16, 4, 128, K, torch.bfloat16, seed=S + K, first_zero=True)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, f"B={B} S={S} K={K}")


def test_unsorted_indices_still_correct():
    q, k, v, idx = make_case(2, 500, 8, 8, 64, 100, torch.bfloat16, seed=5, sort=False)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, "unsorted")


def test_fp16_and_fp32_entry():
    q, k, v, idx = make_case(1, 700, 8, 2, 128, 140, torch.float16, seed=6)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, "f16")
    q32, k32, v32 = q.float(), k.float(), v.float()
    o32, ref32 = run_case(q32, k32, v32, idx)
    assert o32.dtype == torch.float32
    check(o32, ref32, "f32 via bf16")


def test_strided_kv_views_of_block_layout():
    """k_t/v_t as the block passes them: transposes of [B,Hkv,S,hd] views
    over a [B,S,Hkv*hd] projection output."""
    B, S, Hkv, H, hd, K = 2, 300, 4, 16, 128, 61
    g = torch.Generator().manual_seed(11)
    kp = torch.randn(B, S, Hkv * hd, generator=g).to(torch.bfloat16)
    vp = torch.randn(B, S, Hkv * hd, generator=g).to(torch.bfloat16)
    k_t = kp.view(B, S, Hkv, hd).transpose(1, 2).to(DEV).transpose(1, 2)
    v_t = vp.view(B, S, Hkv, hd).transpose(1, 2).to(DEV).transpose(1, 2)
    q = torch.randn(B, S, H, hd, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(S, generator=g)[:K].sort().values for _ in range(B)])
    q_sel = oracle.gather_rows(q.float().numpy(), idx.numpy())
    ref = oracle.sqdk_fp32(q_sel, kp.float().view(B, S, Hkv, hd).numpy(), vp.float().view(B, S, Hkv, hd).numpy(),
                           idx.numpy())
    o = ops.sqdk_fwd(torch.from_numpy(q_sel).to(torch.bfloat16).to(DEV), k_t, v_t, idx.to(DEV), hd ** -0.5)
    check(o, ref, "strided kv")


def test_large_logit_range_rescaling():
    """Scores spanning many powers of two force the lazy O rescale."""
    q, k, v, idx = make_case(1, 2048, 4, 4, 128, 256, torch.bfloat16, seed=8)
    ramp = torch.linspace(0.1, 4.0, 2048)[None, :, None, None]
    k = (k.float() * ramp).to(torch.bfloat16)
    q = (q.float() * 3.0).to(torch.bfloat16)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, "rescale")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rescaling_on_long_key_ranges(dtype):
    """Tiles of 64-128 key blocks (the path where P V needs no commit of its
    own) with scores that grow along the keys: the running maximum jumps by
    more than the optimistic bound at many blocks, the last ones included,
    so O is rescaled mid-tile and at each tile's final block."""
    B, S, H, Hkv, hd, K = 1, 8192, 4, 4, 128, 512
    g = torch.Generator().manual_seed(21)
    q = (torch.randn(B, S, H, hd, generator=g) * 3.0).to(dtype)
    ramp = torch.linspace(0.1, 8.0 if dtype == torch.bfloat16 else 2.0, S)[None, :, None, None]
    k = (torch.randn(B, S, Hkv, hd, generator=g) * ramp).to(dtype)
    v = torch.randn(B, S, Hkv, hd, generator=g).to(dtype)
    idx = (S // 2 + torch.randperm(S // 2, generator=g)[:K]).sort().values[None]
    o, ref = run_case(q, k, v, idx)
    check(o, ref, f"long ranges {dtype}")
    assert ops.device_errors() == 0


def test_cfg5_shape_slice():
    """One sequence of the sparsity-sweep shape (S=32768, H=Hkv=16, hd=128, k=0.05)."""
    S, K = 32768, 1638
    q, k, v, idx = make_case(1, S, 16, 16, 128, K, torch.bfloat16, seed=12)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, "cfg5 slice")


def test_no_device_errors_after_suite():
    assert ops.device_errors() == 0


@pytest.mark.parametrize("hd", [8, 16, 32, 48, 96, 120])
def test_padded_head_dims(hd):
    """head_dim below the tile width (the reference's tests use dim=64 with 4
    heads, i.e. head_dim 16): zero-filled TMA columns, only hd stored."""
    q, k, v, idx = make_case(2, 200, 4, 2, hd, 50, torch.bfloat16, seed=hd)
    o, ref = run_case(q, k, v, idx)
    check(o, ref, f"hd={hd}")


@pytest.mark.parametrize("B,S,H,Hkv,hd,K", [(4, 4096, 16, 4, 128, 820), (6, 2048, 8, 8, 64, 1024),
                                            (5, 3000, 12, 4, 128, 640)])
def test_persistent_many_tiles_per_cta(B, S, H, Hkv, hd, K):
    """More 128-row tiles than the persistent grid has CTAs (2 per SM), so
    each CTA runs several tiles back to back through the same pipeline."""
    q, k, v, idx = make_case(B, S, H, Hkv, hd, K, torch.bfloat16, seed=B * S + K)
    tiles = B * Hkv * -(-K // (128 // (H // Hkv)))
    assert tiles > 2 * torch.cuda.get_device_properties(0).multi_processor_count
    o, ref = run_case(q, k, v, idx)
    check(o, ref, f"B={B} S={S} H={H} Hkv={Hkv} hd={hd} K={K}")
    assert ops.device_errors() == 0


def test_split_workspace_rule_and_parity():
    """Launches with fewer tiles than two per SM split each tile's keys over
    several CTAs (partials in a workspace, merged by a second kernel); large
    launches need no workspace. Both paths match the oracle."""
    from hspmn_b200 import _native as N
    lib = N.lib()
    assert lib.hspmn_sqdk_workspace_size(1, 820, 4096, 16, 4, 128) > 0       # 104 tiles: split
    assert lib.hspmn_sqdk_workspace_size(64, 820, 4096, 16, 4, 128) == 0     # 6656 tiles: direct
    for B in (1, 3):
        q, k, v, idx = make_case(B, 2048, 16, 4, 128, 410, torch.bfloat16, seed=40 + B)
        o, ref = run_case(q, k, v, idx)
        check(o, ref, f"B={B}")
