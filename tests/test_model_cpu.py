"""Host-side checks of the block module's stock-PyTorch parts."""

import pytest
import torch

from hspmn_b200.model import ReflexiveStream, depthwise_conv_seq


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,S,D,pad", [(2, 100, 64, 1), (1, 7, 256, 1), (3, 33, 96, 0), (1, 1, 32, 1)])
def test_depthwise_conv_seq_equals_reference_call(dtype, B, S, D, pad):
    """The channels-last formulation gives exactly what the reference's
    ``conv(h.transpose(1, 2)).transpose(1, 2)`` gives (hspmn_v2_1.py:144)."""
    g = torch.Generator().manual_seed(B * S + D)
    conv = torch.nn.Conv1d(D, D, 3, padding=pad, groups=D, bias=False).to(dtype)
    h = torch.randn(B, S, D, generator=g).to(dtype)
    ref = conv(h.transpose(1, 2)).transpose(1, 2)
    out = depthwise_conv_seq(h, conv.weight, pad)
    assert out.shape == ref.shape and out.is_contiguous()
    assert torch.equal(out, ref)


def test_depthwise_conv_seq_f16_keeps_reference_call():
    conv = torch.nn.Conv1d(32, 32, 3, padding=1, groups=32, bias=False).to(torch.float16)
    h = torch.randn(2, 20, 32).to(torch.float16)
    assert torch.equal(depthwise_conv_seq(h, conv.weight, 1), conv(h.transpose(1, 2)).transpose(1, 2))


def test_reflexive_stream_matches_reference_formula():
    torch.manual_seed(0)
    rs = ReflexiveStream(64)
    x = torch.randn(2, 50, 64)
    h = rs.norm(x)
    h = rs.conv(h.transpose(1, 2)).transpose(1, 2)
    ref = x + rs.down_proj(torch.nn.functional.silu(rs.gate_proj(h)) * rs.up_proj(h))
    assert torch.equal(rs(x), ref)
