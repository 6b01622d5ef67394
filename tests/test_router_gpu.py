"""Router top-K kernel vs the oracle: indices and mask bit-exact."""

import numpy as np
import pytest
import torch

import oracle
from hspmn_b200 import ops
from tests import golden_io as G

pytestmark = pytest.mark.gpu
DEV = "cuda"
_NAME = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def run_and_check(logits: torch.Tensor, temp_val, k, noisy_dtype):
    temp = None if temp_val is None else torch.tensor([temp_val], dtype=logits.dtype, device=DEV)
    idx, mask = ops.router_topk(logits.to(DEV), temp, k, noisy_dtype)
    tv = 1.0 if temp is None else float(temp.float().item())
    noisy = oracle.noisy_logits(logits.float().numpy(), tv, _NAME[noisy_dtype])
    ref_idx, ref_mask = oracle.router_topk(noisy, k, _NAME[noisy_dtype])
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(mask.cpu().numpy(), ref_mask)
    # the same division PyTorch performs on the device (hspmn_v2_1.py:105)
    if temp is not None:
        torch_noisy = (logits.to(DEV) / temp).float().cpu().numpy()
        np.testing.assert_array_equal(torch_noisy, noisy)
    return idx, mask


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,S,frac", [(1, 1, 1.0), (2, 512, 0.2), (3, 4096, 0.2), (2, 4097, 0.05),
                                      (1, 777, 1.0), (4, 33, 0.5)])
def test_router_random(dtype, B, S, frac):
    g = torch.Generator().manual_seed(S * 7 + B)
    logits = torch.randn(B, S, generator=g).to(dtype)
    k = max(1, int(S * frac))
    run_and_check(logits, 0.7, k, dtype)
    run_and_check(logits, None, k, dtype)


def test_router_k_one_and_full():
    logits = torch.randn(2, 300).to(torch.bfloat16)
    idx, mask = run_and_check(logits, 1.0, 1, torch.bfloat16)
    idx, mask = run_and_check(logits, 1.0, 300, torch.bfloat16)
    assert mask.all() and (idx.cpu() == torch.arange(300)).all()


def test_router_ties_nan_signed_zero():
    base = torch.tensor([0.0, 1.0, 1.0, float("nan"), -0.0, 1.0, -1.0, 0.0, 2.0, 1.0])
    logits = base.repeat(3, 50)  # many exact ties across the row
    for k in (1, 3, 7, 40, 200, 499, 500):
        run_and_check(logits, None, k, torch.float32)
    # bf16 rounding creates ties from distinct f32 values
    fine = (torch.arange(4096, dtype=torch.float32) % 97) * 1e-3 + 1.0
    run_and_check(fine.view(1, -1).to(torch.bfloat16), 1.0, 820, torch.bfloat16)


def test_router_all_equal_selects_first_positions():
    """x = zeros gives equal logits (the reference's long-context stress input,
    benchmark_v2_1.py:84): the lowest positions are kept."""
    logits = torch.zeros(1, 8192, dtype=torch.bfloat16)
    idx, mask = run_and_check(logits, 1.0, 1640, torch.bfloat16)
    assert (idx.cpu()[0] == torch.arange(1640)).all()


@pytest.mark.parametrize("S", [65536, 262144])
def test_router_long_rows_cluster_path(S):
    """Long rows, few of them: a cluster of CTAs splits each row (262144 is
    the long-context configuration)."""
    logits = torch.randn(1, S).to(torch.bfloat16)
    run_and_check(logits, 1.0, oracle.router_k(S, 0.2001953125), torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_router_cluster_ties_across_slices(dtype):
    """Few distinct values, so the K-th largest is tied in every CTA's slice of
    the row; a row length that leaves the last slice short."""
    g = torch.Generator().manual_seed(11)
    logits = (torch.randn(2, 40001, generator=g) * 2).round() / 2
    for k in (1, 8000, 20001, 40001):
        run_and_check(logits.to(dtype), None, k, dtype)


def test_router_cluster_all_equal():
    logits = torch.zeros(1, 65536, dtype=torch.bfloat16)
    idx, _ = run_and_check(logits, 1.0, 13107, torch.bfloat16)
    assert (idx.cpu()[0] == torch.arange(13107)).all()


def test_router_long_rows_global_key_path():
    """Rows too long for the shared-memory key cache and too many for one
    cluster each: keys recomputed from the logits on every pass."""
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(20, 65536, generator=g)
    run_and_check(logits, 0.9, 13107, torch.float32)


def test_router_strided_logits():
    full = torch.randn(3, 1000)
    run_and_check(full[:, :600], 1.3, 120, torch.float32)


def test_router_golden_fixture():
    fx = G.load("router_bf16_B2_S4096.npz")
    logits = torch.from_numpy(fx["logits"]).to(torch.bfloat16)
    temp = float(np.clip(np.exp(fx["log_temp"][0]), 0.1, 2.0))
    idx, mask = run_and_check(logits, temp, int(fx["k"]), torch.bfloat16)
    # where the reference's own choice is unambiguous the selections agree
    noisy = fx["noisy"]
    for b in range(idx.shape[0]):
        keys = oracle.orderable_keys(noisy[b], "bf16")
        kth = np.sort(keys)[::-1][int(fx["k"]) - 1]
        strict = np.nonzero(keys > kth)[0]
        assert np.isin(strict, fx["indices"][b]).all() and np.isin(strict, idx[b].cpu().numpy()).all()
