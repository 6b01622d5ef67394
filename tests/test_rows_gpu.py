"""Gather and scatter kernels vs the oracle: bit-exact."""

import numpy as np
import pytest
import torch

import oracle
from hspmn_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def sorted_indices(B, S, K, g):
    return torch.stack([torch.randperm(S, generator=g)[:K].sort().values for _ in range(B)])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("B,S,K,tail", [(2, 512, 102, (4, 64)), (1, 4096, 820, (16, 128)),
                                        (3, 100, 100, (3,)), (2, 65, 1, (8, 1)), (1, 37, 9, (5, 3))])
def test_gather_scatter(dtype, B, S, K, tail):
    g = torch.Generator().manual_seed(B * 1000 + S + K)
    src = torch.randn((B, S) + tail, generator=g).to(dtype)
    idx = sorted_indices(B, S, K, g)
    out = ops.gather_rows(src.to(DEV), idx.to(DEV))
    ref = oracle.gather_rows(src.float().numpy(), idx.numpy())
    np.testing.assert_array_equal(out.cpu().float().numpy(), ref)
    o = torch.randn((B, K) + tail, generator=g).to(dtype)
    sc = ops.scatter_rows(o.to(DEV), idx.to(DEV), S)
    np.testing.assert_array_equal(sc.cpu().float().numpy(), oracle.scatter_rows(o.float().numpy(), idx.numpy(), S))
    assert ops.device_errors() == 0


def test_gather_from_strided_block_layout():
    """q.transpose(1,2) of the block's [B,H,S,hd] view: rows are dense."""
    B, S, H, hd = 2, 256, 4, 64
    q = torch.randn(B, S, H * hd, dtype=torch.bfloat16, device=DEV).view(B, S, H, hd).transpose(1, 2)
    q_t = q.transpose(1, 2)
    idx = sorted_indices(B, S, 51, torch.Generator().manual_seed(3)).to(DEV)
    out = ops.gather_rows(q_t, idx)
    ref = torch.gather(q_t, 1, idx[:, :, None, None].expand(-1, -1, H, hd))
    assert torch.equal(out, ref)


def test_gather_noncontiguous_rows_copies():
    src = torch.randn(2, 40, 6, 8, device=DEV)[:, :, ::2, :]  # rows not dense
    idx = torch.tensor([[0, 5, 39], [1, 2, 3]], device=DEV)
    out = ops.gather_rows(src, idx)
    assert torch.equal(out, torch.stack([src[b, idx[b]] for b in range(2)]))


def test_scatter_empty_selection_zero_fills():
    o = torch.empty(2, 0, 16, dtype=torch.bfloat16, device=DEV)
    idx = torch.empty(2, 0, dtype=torch.int64, device=DEV)
    out = ops.scatter_rows(o, idx, 77)
    assert out.shape == (2, 77, 16) and (out == 0).all()


def test_scatter_matches_torch_scatter():
    """The reference's zeros_like + scatter_ (hspmn_v2_1.py:195-196)."""
    B, S, H, hd, K = 3, 1000, 4, 32, 200
    g = torch.Generator().manual_seed(9)
    idx = sorted_indices(B, S, K, g).to(DEV)
    o = torch.randn(B, K, H, hd, generator=g).to(torch.bfloat16).to(DEV)
    ref = torch.zeros(B, S, H, hd, dtype=torch.bfloat16, device=DEV)
    ref.scatter_(1, idx[:, :, None, None].expand(-1, -1, H, hd), o)
    assert torch.equal(ops.scatter_rows(o, idx, S), ref)


def test_out_of_range_position_flags_error():
    src = torch.randn(1, 10, 8, device=DEV)
    idx = torch.tensor([[0, 3, 10]], device=DEV)
    ops.device_errors()  # clear
    out = ops.gather_rows(src, idx)
    assert ops.device_errors() & 1
    assert (out[0, 2] == 0).all()


def test_unsorted_scatter_flags_error():
    o = torch.randn(1, 3, 8, device=DEV)
    idx = torch.tensor([[5, 2, 7]], device=DEV)
    ops.device_errors()
    ops.scatter_rows(o, idx, 10)
    assert ops.device_errors() & 2
