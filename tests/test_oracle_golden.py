"""The oracle against fixtures produced by the reference itself (CPU only).

These pin the numpy restatement before it is trusted as the oracle for the
CUDA library: router selections against the reference TopKRouter, SQDK
against the reference's FlexAttention path (GQA included) and the whole block
against the reference HSPMNBlock forward.
"""

import json

import numpy as np
import pytest

import oracle
from tests import golden_io as G


@pytest.mark.parametrize("name", ["router_f32_B2_S512.npz", "router_bf16_B2_S4096.npz"])
def test_router_matches_reference(name):
    fx = G.load(name)
    dtype = {"float32": "f32", "bfloat16": "bf16"}[fx["dtype"].item().decode()]
    B, S, D = (int(v) for v in fx["shape"])
    k = oracle.router_k(S, float(fx["target_sparsity"]))
    assert k == int(fx["k"])  # k rounding, incl. the bf16 buffer cast
    temp = float(np.clip(np.exp(fx["log_temp"][0]), 0.1, 2.0))
    temp = float(oracle.round_to(np.array([temp], np.float32), dtype)[0])
    noisy = oracle.noisy_logits(fx["logits"], temp, dtype)
    np.testing.assert_array_equal(noisy, fx["noisy"])  # bit-exact division + rounding
    idx, mask = oracle.router_topk(noisy, k, dtype)
    ref_idx, ref_mask = fx["indices"], fx["mask"]
    for b in range(B):
        keys = oracle.orderable_keys(noisy[b], dtype)
        kth = np.sort(keys)[::-1][k - 1]
        # strictly-above-threshold positions are identical; ties at the k-th
        # value are the one place the reference leaves the order open
        above = np.nonzero(keys > kth)[0]
        assert np.isin(above, ref_idx[b]).all() and np.isin(above, idx[b]).all()
        n_tie_ref = int((keys[ref_idx[b]] == kth).sum())
        n_tie_ora = int((keys[idx[b]] == kth).sum())
        assert n_tie_ref == n_tie_ora
        if (keys == kth).sum() == n_tie_ora:  # no ambiguity: identical selection
            np.testing.assert_array_equal(idx[b], ref_idx[b])
            np.testing.assert_array_equal(mask[b], ref_mask[b])
        else:  # the oracle's rule: lowest positions among the tied values
            tied = np.nonzero(keys == kth)[0]
            np.testing.assert_array_equal(np.sort(idx[b][keys[idx[b]] == kth]), tied[:n_tie_ora])
    assert (np.diff(idx, axis=1) > 0).all()


@pytest.mark.parametrize("name", [
    "sqdk_cfg1_B2_S512_H4_hd64.npz",
    "sqdk_gqa_B1_S256_H8_Hkv2_hd128.npz",
    "sqdk_gqa3_B1_S200_H6_Hkv2_hd64.npz",
])
def test_sqdk_matches_reference_flex(name):
    fx = G.load(name)
    q, k, v = G.sqdk_inputs(fx)
    idx = fx["indices"]
    q_sel = oracle.gather_rows(q, idx)
    o = oracle.sqdk_fp32(q_sel, k, v, idx)
    np.testing.assert_allclose(o, fx["out_sel"], atol=2e-5, rtol=1e-4)
    assert float(fx["unselected_absmax"]) == 0.0  # Flex leaves unselected rows zero
    out = oracle.scatter_rows(o, idx, q.shape[1])
    assert out.shape == q.shape
    unsel = np.ones(q.shape[:2], bool)
    for b in range(q.shape[0]):
        unsel[b, idx[b]] = False
    assert (out[unsel] == 0).all()


@pytest.mark.parametrize("name", ["block_d64_H4_Hkv2_S128.npz", "block_d128_H4_Hkv1_S256.npz"])
def test_block_matches_reference(name):
    fx = G.load(name)
    cfg = json.loads(fx["cfg"].item().decode())
    shapes = G.block_shapes(cfg["dim"], cfg["num_heads"], cfg["num_kv_heads"])
    cfg, x, params = G.block_inputs(fx, shapes)
    out, idx, mask, logits = oracle.block_forward(
        params, x, cfg["num_heads"], cfg["num_kv_heads"], float(fx["target_sparsity"]),
        cfg["rope_base"], eps=float(np.finfo(np.float32).eps), noisy_dtype="f32")
    np.testing.assert_allclose(logits, fx["logits"], atol=1e-5, rtol=1e-5)
    np.testing.assert_array_equal(idx, fx["indices"])
    np.testing.assert_allclose(out, fx["out"], atol=1e-4, rtol=1e-4)


def test_reference_kernel_test_passed_with_oracle():
    """make_golden.py runs the reference's own SQDK unit test with the oracle
    as the kernel and records the outcome."""
    with open(f"{G.GOLDEN}/PINNED.json") as f:
        assert json.load(f)["reference_kernel_test_passes_with_oracle"] is True


def test_rounding_helpers():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf, -0.0], np.float32)
    b = oracle.bf16_round(x)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 is a tie -> 1 + 2^-6
    assert b[1] == 1.0 and b[2] == np.float32(1.015625)
    assert b[3] == -2.5 and np.isinf(b[5])
    assert np.isnan(oracle.bf16_round(np.array([np.nan], np.float32)))[0]


def test_tie_and_nan_order():
    noisy = np.array([[0.0, 1.0, 1.0, np.nan, -0.0, 1.0, -1.0, 0.0]], np.float32)
    idx, mask = oracle.router_topk(noisy, 4, "f32")
    # NaN first, then the three 1.0s; ...
    np.testing.assert_array_equal(idx[0], [1, 2, 3, 5])
    idx, _ = oracle.router_topk(noisy, 6, "f32")
    # +0.0 ranks above -0.0 (bit order); both +0.0 ties kept in position order
    np.testing.assert_array_equal(idx[0], [0, 1, 2, 3, 5, 7])
    assert mask.sum() == 4


@pytest.mark.parametrize("name", ["block_d64_H4_Hkv2_S128.npz", "block_d128_H4_Hkv1_S256.npz"])
def test_torch_cpu_path_matches_reference(name):
    """The torch restatement of the reference's CPU path (eager Flex), which
    the bench times as the CPU baseline, reproduces the reference block's
    outputs, selection and aux loss."""
    import torch

    from oracle.torch_cpu_ref import block_forward_torch

    fx = G.load(name)
    cfg = json.loads(fx["cfg"].item().decode())
    shapes = G.block_shapes(cfg["dim"], cfg["num_heads"], cfg["num_kv_heads"])
    cfg, x, params = G.block_inputs(fx, shapes)
    sd = {k: torch.from_numpy(np.asarray(v, np.float32)) for k, v in params.items()}
    sd["router.target_sparsity"] = torch.tensor(float(fx["target_sparsity"]), dtype=torch.float32)
    out, aux, idx = block_forward_torch(sd, torch.from_numpy(x), cfg["num_heads"], cfg["num_kv_heads"],
                                        cfg["rope_base"])
    np.testing.assert_array_equal(idx.numpy(), fx["indices"])
    np.testing.assert_allclose(out.numpy(), fx["out"], atol=1e-5, rtol=1e-5)
    assert abs(float(aux) - float(fx["aux"])) <= 1e-6


def test_torch_cpu_sqdk_pattern_matches_oracle():
    """The reference's dense-masked PyTorch SQDK pattern (GQA by repeated K/V
    heads) equals the numpy oracle."""
    import torch

    from oracle.torch_cpu_ref import sqdk_dense_torch

    g = torch.Generator().manual_seed(3)
    B, S, H, Hkv, hd, K = 2, 200, 6, 2, 32, 50
    q = torch.randn(B, S, H, hd, generator=g)
    k = torch.randn(B, S, Hkv, hd, generator=g)
    v = torch.randn(B, S, Hkv, hd, generator=g)
    idx = torch.stack([torch.sort(torch.randperm(S, generator=g)[:K])[0] for _ in range(B)])
    out = sqdk_dense_torch(q, k, v, idx)
    ref = oracle.sqdk_fp32(oracle.gather_rows(q.numpy(), idx.numpy()), k.numpy(), v.numpy(), idx.numpy())
    np.testing.assert_allclose(out.numpy(), ref, atol=2e-5, rtol=1e-4)
