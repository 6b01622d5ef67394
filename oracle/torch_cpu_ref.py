"""torch restatement of the reference's HSPMNBlock forward as it runs on a CPU.

TEST INFRASTRUCTURE ONLY (like the rest of ``oracle/``): used by the tests and
by ``bench.py``'s CPU baseline / reference arm, never by the product path.

On a machine without a GPU the reference module cannot take its Triton branch
(``_attention_triton``, hspmn_v2_1.py:176-198); its contextual stream then runs
``_attention_flex`` (hspmn_v2_1.py:200-216) with FlexAttention evaluated
eagerly (the compiled Flex path does not lower on a CPU). That path is what
this module restates, operation for operation, with stock torch ops on the
block's ``state_dict``:

* router: gate GEMV, ``logits / clamp(exp(log_temp), 0.1, 2)``,
  ``topk(sorted=False)`` + ascending ``sort`` + bool mask, aux loss
  (hspmn_v2_1.py:95-122, eval branch);
* reflexive stream: RMSNorm, depthwise Conv1d(k=3), SwiGLU MLP, residual
  (hspmn_v2_1.py:141-145);
* contextual stream: RMSNorm, q/k/v projections, RoPE (hspmn_v2_1.py:34-68,
  218-227), FlexAttention with the block mask ``(q_idx >= kv_idx) &
  mask[b, q_idx]`` and ``enable_gqa`` (hspmn_v2_1.py:200-216), o_proj.

Eager FlexAttention on a CPU evaluates the dense S x S score matrix, so this
path does the dense attention work whatever the sparsity.

``sqdk_dense_torch`` restates the reference's own PyTorch SQDK test pattern
(test_kernels_v2_1.py:34-65: gather -> Q K^T * scale -> masked_fill(k_pos >
q_pos) -> softmax -> P V), with K/V heads repeated for grouped queries.
"""

from __future__ import annotations

import math
from typing import Dict, Tuple

import torch
import torch.nn.functional as F


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    """hspmn_v2_1.py:34-38."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def rope_cos_sin(S: int, hd: int, base: float, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [1,1,S,hd] in ``dtype`` (hspmn_v2_1.py:45-63)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    t = torch.arange(S, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos()[None, None].to(dtype), emb.sin()[None, None].to(dtype)


def router_eval(sd: Dict[str, torch.Tensor], x: torch.Tensor, sparsity_coef: float = 0.1,
                entropy_coef: float = 0.01):
    """TopKRouter.forward in eval mode (hspmn_v2_1.py:95-122). Returns
    (mask [B,S] bool, indices [B,k] ascending, logits [B,S], aux_loss)."""
    B, S, _ = x.shape
    logits = F.linear(x, sd["router.gate.weight"], sd["router.gate.bias"]).squeeze(-1)
    temp = torch.exp(sd["router.log_temp"]).clamp(0.1, 2.0)
    noisy = logits / temp
    probs = torch.sigmoid(logits)
    ts = sd["router.target_sparsity"]
    sparsity_loss = (probs.mean() - ts).pow(2)
    ent = -(probs * (probs + 1e-10).log() + (1.0 - probs) * (1.0 - probs + 1e-10).log())
    aux = sparsity_coef * sparsity_loss + entropy_coef * ent.mean()
    k = max(1, int(S * ts.item()))
    _, indices = torch.topk(noisy, k, dim=1, sorted=False)
    indices, _ = torch.sort(indices, dim=-1)
    indices = indices.contiguous()
    mask = torch.zeros(B, S, dtype=torch.bool)
    mask.scatter_(1, indices, True)
    return mask, indices, logits, aux


def reflexive(sd: Dict[str, torch.Tensor], x: torch.Tensor) -> torch.Tensor:
    """ReflexiveStream.forward (hspmn_v2_1.py:141-145)."""
    h = F.rms_norm(x, (x.shape[-1],), sd["reflexive.norm.weight"])
    w = sd["reflexive.conv.weight"]
    h = F.conv1d(h.transpose(1, 2), w, None, padding=1, groups=w.shape[0]).transpose(1, 2)
    g = F.linear(h, sd["reflexive.gate_proj.weight"])
    u = F.linear(h, sd["reflexive.up_proj.weight"])
    return x + F.linear(F.silu(g) * u, sd["reflexive.down_proj.weight"])


def attention_flex(sd: Dict[str, torch.Tensor], x: torch.Tensor, mask: torch.Tensor, num_heads: int,
                   num_kv_heads: int, rope_base: float, block_size: int) -> torch.Tensor:
    """HSPMNBlock._attention with the FlexAttention branch, eager
    (hspmn_v2_1.py:200-234)."""
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention

    B, S, D = x.shape
    hd = D // num_heads
    xn = F.rms_norm(x, (D,), sd["norm.weight"])
    q = F.linear(xn, sd["q_proj.weight"]).view(B, S, num_heads, hd).transpose(1, 2)
    k = F.linear(xn, sd["k_proj.weight"]).view(B, S, num_kv_heads, hd).transpose(1, 2)
    v = F.linear(xn, sd["v_proj.weight"]).view(B, S, num_kv_heads, hd).transpose(1, 2)
    cos, sin = rope_cos_sin(S, hd, rope_base, q.dtype)
    q = q * cos + _rotate_half(q) * sin
    k = k * cos + _rotate_half(k) * sin

    def mask_fn(b, h, q_idx, kv_idx):
        return (q_idx >= kv_idx) & mask[b, q_idx]

    bm = create_block_mask(mask_fn, B=B, H=num_heads, Q_LEN=S, KV_LEN=S, device="cpu", BLOCK_SIZE=block_size)
    out = flex_attention(q, k, v, block_mask=bm, enable_gqa=(num_kv_heads != num_heads), scale=1.0 / math.sqrt(hd))
    return F.linear(out.transpose(1, 2).contiguous().view(B, S, D), sd["o_proj.weight"])


@torch.no_grad()
def block_forward_torch(sd: Dict[str, torch.Tensor], x: torch.Tensor, num_heads: int, num_kv_heads: int,
                        rope_base: float = 10000.0, block_size: int = 128):
    """HSPMNBlock.forward in eval mode on the CPU path (hspmn_v2_1.py:236-238).
    ``sd`` is the block's state_dict (CPU tensors of one dtype); returns
    (out [B,S,D], aux_loss, indices)."""
    mask, indices, _, aux = router_eval(sd, x)
    out = reflexive(sd, x) + attention_flex(sd, x, mask, num_heads, num_kv_heads, rope_base, block_size)
    return out, aux, indices


@torch.no_grad()
def sqdk_dense_torch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """The reference's PyTorch SQDK (test_kernels_v2_1.py:34-65) on q [B,S,H,hd],
    k, v [B,S,Hkv,hd], sorted indices [B,K]; K/V heads repeated for grouped
    queries (head h reads h // (H // Hkv), hspmn_v2_1.py:212). Returns the
    attention rows [B,K,H,hd]."""
    B, S, H, hd = q.shape
    G = H // k.shape[2]
    if G > 1:
        k = k.repeat_interleave(G, dim=2)
        v = v.repeat_interleave(G, dim=2)
    sel = indices.unsqueeze(-1).unsqueeze(-1).expand(-1, -1, H, hd)
    q_sel = torch.gather(q, 1, sel).permute(0, 2, 1, 3)
    scores = torch.matmul(q_sel, k.permute(0, 2, 3, 1)) * (1.0 / hd ** 0.5)
    allowed = torch.arange(S).reshape(1, 1, 1, S) <= indices.unsqueeze(1).unsqueeze(-1)
    scores = scores.masked_fill(~allowed, float("-inf"))
    return torch.matmul(F.softmax(scores, dim=-1), v.permute(0, 2, 1, 3)).permute(0, 2, 1, 3)
