"""The oracle's SQDK backward (CPU only), pinned against float64 autograd of
the dense masked attention whose forward the reference's Flex goldens pin
(the reference's Flex backward does not run on a CPU)."""

import numpy as np
import pytest
import torch

import oracle


def _autograd(q, k, v, idx, d_o):
    G = q.shape[2] // k.shape[2]
    qt, kt, vt = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
    s = torch.einsum("bkhd,bshd->bhks", qt, kt.repeat_interleave(G, dim=2)) * q.shape[3] ** -0.5
    allowed = torch.arange(k.shape[1])[None, None, None, :] <= torch.tensor(idx)[:, None, :, None]
    s = s.masked_fill(~allowed, float("-inf"))
    o = torch.einsum("bhks,bshd->bkhd", torch.softmax(s, -1), vt.repeat_interleave(G, dim=2))
    o.backward(torch.tensor(d_o, dtype=torch.float64))
    lse = torch.logsumexp(s, -1).permute(0, 2, 1).detach().numpy()
    return qt.grad.numpy(), kt.grad.numpy(), vt.grad.numpy(), lse, o.detach().numpy()


@pytest.mark.parametrize("B,S,H,Hkv,hd,K", [(2, 96, 4, 2, 16, 20), (1, 130, 6, 2, 32, 40), (1, 64, 2, 2, 8, 64)])
def test_sqdk_bwd_matches_float64_autograd(B, S, H, Hkv, hd, K):
    rng = np.random.default_rng(S + K)
    q = rng.standard_normal((B, K, H, hd)).astype(np.float32)
    k = rng.standard_normal((B, S, Hkv, hd)).astype(np.float32)
    v = rng.standard_normal((B, S, Hkv, hd)).astype(np.float32)
    d_o = rng.standard_normal((B, K, H, hd)).astype(np.float32)
    idx = np.sort(np.stack([rng.choice(S, K, replace=False) for _ in range(B)]), axis=1)
    dq, dk, dv, lse = oracle.sqdk_bwd_fp32(q, k, v, idx, d_o)
    rdq, rdk, rdv, rlse, ro = _autograd(q, k, v, idx, d_o)
    np.testing.assert_allclose(oracle.sqdk_fp32(q, k, v, idx), ro, atol=2e-5)
    for got, ref in ((dq, rdq), (dk, rdk), (dv, rdv), (lse, rlse)):
        np.testing.assert_allclose(got, ref, atol=5e-5, rtol=1e-4)
