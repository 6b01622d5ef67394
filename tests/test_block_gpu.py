"""HSPMNBlock on the B200 path: the reference's own unit tests (ported from
test_v2_1.py) plus block-level parity against the oracle and the reference
goldens."""

import json
import math

import numpy as np
import pytest
import torch
import torch.nn as nn

import oracle
from hspmn_b200 import HSPMNBlock, HSPMNConfig, TopKRouter, ops, seed_everything
from hspmn_b200.model import RouterOutput
from tests import golden_io as G

DEV = "cuda"


def _load_params(block, params):
    sd = block.state_dict()
    for name, val in params.items():
        sd[name] = torch.from_numpy(val).to(sd[name].dtype)
    block.load_state_dict(sd)


# -- ported from test_v2_1.py (reference unit tests) ------------------------

@pytest.fixture
def cfg():
    seed_everything(42)
    return HSPMNConfig(dim=64, num_heads=4, num_kv_heads=2, sparsity_k=0.5, block_size=64)


@pytest.mark.gpu
def test_router_entropy_loss(cfg):
    """test_v2_1.py:25-35."""
    router = TopKRouter(cfg.dim, target_sparsity=0.5).to(DEV)
    x = torch.randn(2, 128, cfg.dim, device=DEV)
    out = router(x)
    assert out.aux_loss > 0
    assert out.mask.shape == (2, 128)
    out.aux_loss.backward()
    assert router.gate.weight.grad is not None


@pytest.mark.gpu
def test_sparse_gradient_isolation(cfg):
    """test_v2_1.py:37-64 (training path, FlexAttention)."""
    model = HSPMNBlock(cfg).to(DEV)
    x = torch.randn(2, 128, cfg.dim, device=DEV, requires_grad=True)

    class MockRouter(nn.Module):
        def __init__(self, dim):
            super().__init__()
            self.gate = nn.Linear(dim, 1)
            self.aux_loss = torch.tensor(0.0, device=DEV, requires_grad=True)

        def forward(self, x):
            B, S, _ = x.shape
            mask = torch.zeros(B, S, dtype=torch.bool, device=x.device)
            mask[:, :S // 2] = True
            indices = torch.arange(S // 2, device=x.device).unsqueeze(0).expand(B, -1)
            return RouterOutput(mask, indices, torch.zeros(B, S, device=x.device), self.aux_loss)

    model.router = MockRouter(cfg.dim).to(DEV)
    out, _ = model(x)
    out.sum().backward()
    assert model.q_proj.weight.grad is not None
    assert not torch.isnan(model.q_proj.weight.grad).any()


def test_reflexive_stream_correctness(cfg):
    """test_v2_1.py:66-71 (stock PyTorch, runs on the CPU too)."""
    model = HSPMNBlock(cfg)
    x = torch.randn(2, 64, cfg.dim)
    out = model.reflexive(x)
    assert out.shape == x.shape and not torch.isnan(out).any()


def test_gqa_shapes():
    """test_v2_1.py:73-76."""
    model = HSPMNBlock(HSPMNConfig(dim=64, num_heads=4, num_kv_heads=1))
    assert model.num_kv_heads == 1


@pytest.mark.gpu
@pytest.mark.parametrize("train", [False, True])
def test_forward_pass_integration(cfg, train):
    """test_v2_1.py:78-83, in eval (the SQDK path) and train mode."""
    model = HSPMNBlock(cfg).to(DEV).train(train)
    x = torch.randn(1, 128, cfg.dim, device=DEV)
    out, aux = model(x)
    assert out.shape == (1, 128, cfg.dim) and torch.is_tensor(aux)
    assert torch.isfinite(out).all()


# -- block parity ----------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("name", ["block_d64_H4_Hkv2_S128.npz", "block_d128_H4_Hkv1_S256.npz"])
def test_block_matches_reference_golden(name):
    """float32 block on the B200 path vs the reference HSPMNBlock forward
    (eager Flex, CPU). The router selection must be identical; the output
    differs only by the bf16 rounding inside SQDK."""
    fx = G.load(name)
    c = json.loads(fx["cfg"].item().decode())
    cfg = HSPMNConfig(dim=c["dim"], num_heads=c["num_heads"], num_kv_heads=c["num_kv_heads"],
                      sparsity_k=c["sparsity"], max_seq_len=c["S"])
    block = HSPMNBlock(cfg)
    _, x, params = G.block_inputs(fx, {k: tuple(v.shape) for k, v in block.state_dict().items()})
    _load_params(block, params)
    block = block.to(DEV).eval()
    with torch.no_grad():
        ro = block.router(torch.from_numpy(x).to(DEV))
        out, aux = block(torch.from_numpy(x).to(DEV))
    np.testing.assert_array_equal(ro.indices.cpu().numpy(), fx["indices"])
    err = np.abs(out.cpu().numpy() - fx["out"])
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
    assert abs(aux.item() - float(fx["aux"])) <= 1e-5


@pytest.mark.gpu
def test_block_bf16_cfg2_shape_against_oracle():
    """The single-sequence benchmark block (dim=2048, H=16, Hkv=4, S=4096,
    k=0.2 -> K=820 in bf16): router bit-exact on the device logits, the
    contextual stream within tolerance of the fp32 oracle on the device q/k/v."""
    torch.manual_seed(0)
    cfg = HSPMNConfig(dim=2048, num_heads=16, max_seq_len=4096)
    block = HSPMNBlock(cfg).to(DEV, dtype=torch.bfloat16).eval()
    with torch.no_grad():
        block.router.gate.weight.normal_(0, 2048 ** -0.5)
    x = torch.randn(1, 4096, 2048, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        ro = block.router(x)
        assert ro.indices.shape == (1, 820)
        temp = torch.exp(block.router.log_temp).clamp(0.1, 2.0)
        noisy = oracle.noisy_logits(ro.logits.float().cpu().numpy(), float(temp.float()), "bf16")
        ref_idx, ref_mask = oracle.router_topk(noisy, 820, "bf16")
        np.testing.assert_array_equal(ro.indices.cpu().numpy(), ref_idx)
        np.testing.assert_array_equal(ro.mask.cpu().numpy(), ref_mask)
        # contextual stream on the device q/k/v
        B, S, D = x.shape
        xn = block.norm(x)
        q = block.q_proj(xn).view(B, S, 16, 128).transpose(1, 2)
        k = block.k_proj(xn).view(B, S, 4, 128).transpose(1, 2)
        v = block.v_proj(xn).view(B, S, 4, 128).transpose(1, 2)
        cos, sin = block.rope(q, S)
        from hspmn_b200.model import apply_rotary_pos_emb
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        q_t, k_t, v_t = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        q_sel = ops.gather_rows(q_t, ro.indices)
        o = ops.sqdk_fwd(q_sel, k_t, v_t, ro.indices, 128 ** -0.5)
        out = ops.scatter_rows(o, ro.indices, S)
    idx = ro.indices.cpu().numpy()
    qn = q_t.float().cpu().numpy()
    ref_qsel = oracle.gather_rows(qn, idx)
    np.testing.assert_array_equal(q_sel.float().cpu().numpy(), ref_qsel)
    ref_o = oracle.sqdk_fp32(ref_qsel, k_t.float().cpu().numpy(), v_t.float().cpu().numpy(), idx)
    err = np.abs(o.float().cpu().numpy() - ref_o)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
    np.testing.assert_array_equal(out.float().cpu().numpy(), oracle.scatter_rows(o.float().cpu().numpy(), idx, S))
    # the reference-order forward runs exactly that path
    with torch.no_grad():
        block.sqdk_fused = False
        y, _ = block(x)
        y_ref = block.reflexive(x) + block.o_proj(out.view(B, S, D))
    assert torch.equal(y, y_ref)


@pytest.mark.gpu
def test_fp32_block_attention_rounds_through_bf16():
    """A float32 block's eval attention runs on the bf16 tensor-core kernel
    (q, k, v rounded to bf16, fp32 accumulation, fp32 result), where the
    reference's Triton path keeps tf32 dot products. Measured here against the
    float32 oracle block (attention in fp32) on the same selection: the
    difference stays inside the attention tolerance."""
    seed_everything(5)
    D, H, Hkv, S = 512, 8, 2, 1024
    cfg = HSPMNConfig(dim=D, num_heads=H, num_kv_heads=Hkv, max_seq_len=S)
    block = HSPMNBlock(cfg)
    with torch.no_grad():
        block.router.gate.weight.normal_(0, D ** -0.5)
    params = {k: v.detach().float().numpy().copy() for k, v in block.state_dict().items()}
    block = block.to(DEV).eval()
    x = torch.randn(2, S, D, generator=torch.Generator().manual_seed(6))
    with torch.no_grad():
        out, _ = block(x.to(DEV))
        idx = block.router(x.to(DEV)).indices.cpu().numpy()
    ref, _, _, _ = oracle.block_forward(params, x.numpy(), H, Hkv, float(block.router.target_sparsity.item()),
                                        cfg.rope_base, float(np.finfo(np.float32).eps), indices=idx)
    err = np.abs(out.cpu().numpy() - ref)
    print(f"fp32 block vs fp32 oracle: max_abs={err.max():.3e} mean_abs={err.mean():.3e}")
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_reflexive_conv_layout_bit_exact(dtype):
    """The reflexive stream's depthwise convolution, run channels-last on the
    [B,S,D] memory, equals the reference's transposed Conv1d call bit for bit
    on the GPU (hspmn_v2_1.py:144), at the block's width."""
    from hspmn_b200.model import depthwise_conv_seq
    g = torch.Generator(device=DEV).manual_seed(1)
    D = 2048
    conv = nn.Conv1d(D, D, 3, padding=1, groups=D, bias=False).to(DEV, dtype)
    h = torch.randn(4, 1000, D, device=DEV, dtype=dtype, generator=g)
    with torch.no_grad():
        ref = conv(h.transpose(1, 2)).transpose(1, 2)
        out = depthwise_conv_seq(h, conv.weight, 1)
    if dtype != torch.float16:  # fp16 runs the reference's own call
        assert out.is_contiguous()
    assert torch.equal(out, ref)
