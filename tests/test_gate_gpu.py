"""fp32 router gate kernel vs the oracle.

bf16 / f16 inputs: logits bit-exact against the oracle's fixed-order fp32 sum,
and within the summation error bound of the exact (float64) dot product.
f32 inputs: within that bound. Selection on the kernel's logits: bit-exact.
"""

import numpy as np
import pytest
import torch

import oracle
from hspmn_b200 import HSPMNBlock, HSPMNConfig, ops
from hspmn_b200._native import HSPMNNativeError

pytestmark = pytest.mark.gpu
DEV = "cuda"
_NAME = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def _inputs(B, S, D, dtype, seed, scale=1.0, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(B, S, D, generator=g) * scale).to(dtype)
    w = (torch.randn(1, D, generator=g) * D ** -0.5).to(dtype)
    b = (torch.randn(1, generator=g) * 0.1).to(dtype) if bias else None
    return x, w, b


def _check(x, w, b, exact=True):
    """Run the kernel on (x, w, b) (CPU tensors) and compare with the oracle."""
    dt = _NAME[x.dtype]
    bias = None if b is None else float(b.float())
    got = ops.gate_logits(x.to(DEV), w.to(DEV), None if b is None else b.to(DEV)).cpu().numpy()
    xf, wf = x.float().numpy(), w.float().numpy().reshape(-1)
    ref = oracle.gate_logits_fp32(xf, wf, bias, dt)
    if exact:
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    exact64 = xf.astype(np.float64) @ wf.astype(np.float64) + (0.0 if bias is None else bias)
    fin = np.isfinite(exact64) & np.isfinite(got)
    err = np.abs(got[fin].astype(np.float64) - exact64[fin])
    bound = oracle.gate_error_bound(xf, wf, bias)[fin]
    assert (err <= bound).all(), float((err / bound).max())
    return got


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,S,D", [(1, 1, 8), (2, 300, 2048), (3, 129, 264), (1, 64, 4096), (2, 17, 1000)])
def test_gate_16bit_bit_exact(dtype, B, S, D):
    x, w, b = _inputs(B, S, D, dtype, seed=B * 131 + S + D)
    _check(x, w, b)
    _check(x, w, None)


@pytest.mark.parametrize("B,S,D", [(1, 1, 4), (2, 300, 2048), (3, 77, 260)])
def test_gate_f32_within_bound(B, S, D):
    x, w, b = _inputs(B, S, D, torch.float32, seed=B + S * 3 + D)
    _check(x, w, b, exact=False)


def test_gate_many_rows_grid_stride():
    """More rows than resident warps: every row is still written once."""
    x, w, b = _inputs(4, 40000, 256, torch.bfloat16, seed=11)
    _check(x, w, b)


def test_gate_subnormal_huge_and_cancelling():
    D = 512
    g = torch.Generator().manual_seed(3)
    w = torch.randn(1, D, generator=g).to(torch.bfloat16)
    rows = [
        torch.full((D,), 1e-38),                                    # products far below the normal range
        torch.randn(D, generator=g) * 1e34,                         # large products; every partial sum stays finite
        torch.cat([torch.ones(D // 2), -torch.ones(D // 2)]) * 1e4,  # signs cancelling across lanes
        torch.zeros(D),
    ]
    x = torch.stack(rows).view(1, len(rows), D).to(torch.bfloat16)
    got = _check(x, w, torch.tensor([0.0], dtype=torch.bfloat16))
    assert got[0, 3] == 0.0


def test_gate_strided_view_and_row_independence():
    x, w, b = _inputs(2, 64, 1024, torch.bfloat16, seed=21)
    big = torch.zeros(2, 128, 1024, dtype=torch.bfloat16)
    big[:, ::2] = x
    strided = big.to(DEV)[:, ::2]  # x_ss = 2*D elements: used in place, no copy
    got = ops.gate_logits(strided, w.to(DEV), b.to(DEV))
    ref = ops.gate_logits(x.to(DEV).contiguous(), w.to(DEV), b.to(DEV))
    assert torch.equal(got, ref)
    # a row's logit does not depend on where the row sits or on the launch
    rolled = ops.gate_logits(torch.roll(x, 5, dims=1).to(DEV), w.to(DEV), b.to(DEV))
    assert torch.equal(torch.roll(ref, 5, dims=1), rolled)
    assert torch.equal(ops.gate_logits(x.to(DEV), w.to(DEV), b.to(DEV)), ref)


def test_gate_rejects_bad_arguments():
    x, w, b = _inputs(1, 4, 12, torch.bfloat16, seed=1)  # D=12: not a whole number of 16-byte vectors
    with pytest.raises(HSPMNNativeError):
        ops.gate_logits(x.to(DEV), w.to(DEV), b.to(DEV))
    x, w, b = _inputs(1, 4, 16, torch.bfloat16, seed=1)
    with pytest.raises(TypeError):
        ops.gate_logits(x.to(DEV), w.float().to(DEV), b.to(DEV))
    with pytest.raises(ValueError):
        ops.gate_logits(x.to(DEV), w[:, :8].to(DEV), b.to(DEV))


def test_gate_router_selection_on_fp32_logits():
    """The router kernel on the gate's f32 logits (bf16 temperature, f32
    noisy values) selects what the oracle selects on the same logits."""
    x, w, b = _inputs(3, 4096, 2048, torch.bfloat16, seed=8)
    logits = ops.gate_logits(x.to(DEV), w.to(DEV), b.to(DEV))
    temp = torch.tensor([0.8], dtype=torch.bfloat16, device=DEV)
    idx, mask = ops.router_topk(logits, temp, 820, torch.float32)
    noisy = oracle.noisy_logits(logits.cpu().numpy(), float(temp.float()), "f32")
    ref_idx, ref_mask = oracle.router_topk(noisy, 820, "f32")
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_array_equal(mask.cpu().numpy(), ref_mask)


def test_block_bf16_with_fp32_gate():
    """bf16 block with ``router.fp32_gate``: RouterOutput.logits are the
    kernel's f32 logits (bit-exact), the selection ranks them, and the block
    output equals the default path's computation for that selection."""
    torch.manual_seed(2)
    dim, H, Hkv, S = 512, 8, 2, 1024
    block = HSPMNBlock(HSPMNConfig(dim=dim, num_heads=H, num_kv_heads=Hkv, max_seq_len=S))
    with torch.no_grad():
        block.router.gate.weight.normal_(0, dim ** -0.5)
        block.router.gate.bias.fill_(0.05)
    block = block.to(DEV, dtype=torch.bfloat16).eval()
    block.router.fp32_gate = True
    x = torch.randn(2, S, dim).to(torch.bfloat16)
    with torch.no_grad():
        ro = block.router(x.to(DEV))
        y, aux = block(x.to(DEV))
    assert ro.logits.dtype == torch.float32
    ref = oracle.gate_logits_fp32(x.float().numpy(), block.router.gate.weight.detach().float().cpu().numpy().reshape(-1),
                                  float(block.router.gate.bias.float()), "bf16")
    np.testing.assert_array_equal(ro.logits.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    temp = float(torch.exp(block.router.log_temp).clamp(0.1, 2.0).float())
    k = block.router.num_selected(S)
    ref_idx, _ = oracle.router_topk(oracle.noisy_logits(ref, temp, "f32"), k, "f32")
    np.testing.assert_array_equal(ro.indices.cpu().numpy(), ref_idx)
    assert torch.isfinite(aux) and torch.isfinite(y).all()
    # the default gate on the same block picks from rounded logits; the rest
    # of the forward is the same code, so the rows selected by both agree
    block.router.fp32_gate = False
    with torch.no_grad():
        y_default, _ = block(x.to(DEV))
        ro_default = block.router(x.to(DEV))
    both = ro.mask & ro_default.mask
    assert both.sum() > 0.9 * ro.mask.sum()
    unrouted = ~(ro.mask | ro_default.mask)
    assert torch.equal(y[unrouted], y_default[unrouted])


def test_block_fp32_with_fp32_gate_against_oracle():
    """float32 block with the fp32 gate vs the oracle's fp32 block forward
    given the kernel's selection."""
    torch.manual_seed(6)
    dim, H, Hkv, S = 256, 4, 2, 384
    block = HSPMNBlock(HSPMNConfig(dim=dim, num_heads=H, num_kv_heads=Hkv, max_seq_len=S)).eval()
    with torch.no_grad():
        block.router.gate.weight.normal_(0, dim ** -0.5)
    params = {k: v.float().numpy() for k, v in block.state_dict().items()}
    block = block.to(DEV)
    block.router.fp32_gate = True
    x = torch.randn(2, S, dim)
    with torch.no_grad():
        y, _ = block(x.to(DEV))
        ro = block.router(x.to(DEV))
    idx = ro.indices.cpu().numpy()
    temp = float(torch.exp(block.router.log_temp).clamp(0.1, 2.0))
    ref_idx, _ = oracle.router_topk(oracle.noisy_logits(ro.logits.cpu().numpy(), temp, "f32"),
                                    block.router.num_selected(S), "f32")
    np.testing.assert_array_equal(idx, ref_idx)
    ref, _, _, _ = oracle.block_forward(params, x.numpy(), H, Hkv, float(block.router.target_sparsity.item()),
                                        10000, float(np.finfo(np.float32).eps), indices=idx)
    err = np.abs(y.cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
