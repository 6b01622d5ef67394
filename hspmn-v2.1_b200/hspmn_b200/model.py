"""HSPMNBlock and its parts, API-compatible with hspmn_v2_1.py.

Parameter names, buffers, init and forward semantics follow the reference
(hspmn_v2_1.py:26-238) so ``state_dict``s load across. In eval mode the
contextual stream runs the B200 path: router selection (``ops.router_topk``),
gather, SQDK attention (``ops.sqdk_fwd``) and the write-back, all sm_100a CUDA
kernels. By default (``sqdk_fused``) the write-back skips the zero-filled
scatter: q_proj, RoPE and o_proj run only on the routed rows and the result
is added into the residual in place (``ops.scatter_add_rows_``); with
``sqdk_fused = False`` the reference's order (gather -> SQDK -> zero-filling
``ops.scatter_rows`` -> o_proj on all rows) is used. The
surrounding projections, norms, RoPE and the reflexive stream are stock
PyTorch, as in the reference. In training mode the contextual stream of a
bf16/f16 block on CUDA runs the same attention with its backward on the
sm_100a kernels (``ops.sqdk_attention``: gather -> SQDK -> scatter, autograd
through both kernels); with ``sqdk_train = False``, or for float32 blocks, it
keeps the reference's FlexAttention formulation (hspmn_v2_1.py:200-216).
"""

from __future__ import annotations

import math
from typing import NamedTuple, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .utils import HSPMNConfig

__all__ = ["HSPMNBlock", "TopKRouter", "HSPMNConfig", "RouterOutput", "RotaryEmbedding",
           "apply_rotary_pos_emb", "rotate_half", "ReflexiveStream", "depthwise_conv_seq"]


class RouterOutput(NamedTuple):
    """Output of TopKRouter (hspmn_v2_1.py:26-31)."""

    mask: torch.Tensor
    indices: torch.Tensor
    logits: torch.Tensor
    aux_loss: torch.Tensor


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """hspmn_v2_1.py:34-38."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


class RotaryEmbedding(nn.Module):
    """RoPE cos/sin cache [1,1,L,hd], grown on demand (hspmn_v2_1.py:40-63)."""

    def __init__(self, dim: int, max_len: int = 131072, base: int = 10000):
        super().__init__()
        self.dim = dim
        self.base = base
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._build_cache(max_len)

    def _build_cache(self, seq_len: int):
        t = torch.arange(seq_len, dtype=torch.float32, device=self.inv_freq.device)
        freqs = torch.outer(t, self.inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.register_buffer("cached_cos", emb.cos()[None, None, :, :], persistent=False)
        self.register_buffer("cached_sin", emb.sin()[None, None, :, :], persistent=False)

    def forward(self, x: torch.Tensor, seq_len: int):
        if seq_len > self.cached_cos.shape[2]:
            self._build_cache(seq_len)
        cos = self.cached_cos[:, :, :seq_len, :]
        sin = self.cached_sin[:, :, :seq_len, :]
        return cos.to(dtype=x.dtype), sin.to(dtype=x.dtype)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                         sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """hspmn_v2_1.py:66-68."""
    return (q * cos) + (rotate_half(q) * sin), (k * cos) + (rotate_half(k) * sin)


_compiled_flex_attention = None


def get_compiled_flex_attention():
    """Compiled FlexAttention for the training path (hspmn_v2_1.py:71-78)."""
    global _compiled_flex_attention
    if _compiled_flex_attention is None:
        from torch.nn.attention.flex_attention import flex_attention
        _compiled_flex_attention = torch.compile(flex_attention, dynamic=True)
    return _compiled_flex_attention


class TopKRouter(nn.Module):
    """Top-K token router (hspmn_v2_1.py:81-122).

    The gate GEMV, temperature and auxiliary loss are PyTorch exactly as in
    the reference; the top-K selection, index sort and mask are one CUDA
    kernel (``ops.router_topk``). Among equal noisy logits the lower position
    is selected first (the reference's ``torch.topk`` leaves that order
    unspecified).

    ``fp32_gate`` (off by default): in eval mode the gate GEMV runs as one CUDA
    kernel (``ops.gate_logits``) that keeps the logits in float32 instead of
    rounding them to the module dtype; the selection then ranks fp32 values,
    and ``RouterOutput.logits`` and the auxiliary loss are float32. Training
    always uses the ``nn.Linear`` gate (its weights need gradients)."""

    def __init__(self, dim: int, target_sparsity: float = 0.2, sparsity_coef: float = 0.1,
                 entropy_coef: float = 0.01):
        super().__init__()
        self.gate = nn.Linear(dim, 1, bias=True)
        self.register_buffer("target_sparsity", torch.tensor(target_sparsity))
        self.sparsity_coef = sparsity_coef
        self.entropy_coef = entropy_coef
        self.log_temp = nn.Parameter(torch.zeros(1))
        nn.init.xavier_uniform_(self.gate.weight, gain=0.02)
        nn.init.zeros_(self.gate.bias)
        self.fp32_gate = False
        self._k_cache_key = None
        self._k_cache_val = 0.0

    def _sparsity_value(self) -> float:
        """``target_sparsity.item()`` (hspmn_v2_1.py:112), read from the device
        only when the buffer changed (its version counter, storage or dtype),
        so a steady-state forward does not synchronise."""
        ts = self.target_sparsity
        key = (ts._version, ts.data_ptr(), ts.dtype, ts.device)
        if key != self._k_cache_key:
            self._k_cache_val = ts.item()
            self._k_cache_key = key
        return self._k_cache_val

    def num_selected(self, S: int) -> int:
        """``k = max(1, int(S * target_sparsity))`` with the buffer in the module
        dtype (0.2 in bf16 is 0.2001953125: S=4096 selects 820)."""
        return max(1, int(S * self._sparsity_value()))

    def gate_logits(self, x: torch.Tensor) -> torch.Tensor:
        """``self.gate(x).squeeze(-1)`` (hspmn_v2_1.py:96), or the fp32 gate
        kernel when ``fp32_gate`` is set and the module is in eval mode."""
        if self.fp32_gate and not self.training:
            return ops.gate_logits(x, self.gate.weight, self.gate.bias)
        return self.gate(x).squeeze(-1)

    def forward(self, x: torch.Tensor) -> RouterOutput:
        B, S, _ = x.shape
        logits = self.gate_logits(x)
        temp = torch.exp(self.log_temp).clamp(0.1, 2.0)
        k = self.num_selected(S)
        if self.training:
            U = torch.rand_like(logits)
            gumbel_noise = -torch.log(-torch.log(U + 1e-10) + 1e-10)
            noisy = (logits + gumbel_noise) / temp
            indices, mask = ops.router_topk(noisy.detach(), None, k, noisy.dtype)
        else:
            noisy_dtype = torch.result_type(logits, temp)
            indices, mask = ops.router_topk(logits.detach(), temp.detach(), k, noisy_dtype)

        probs = torch.sigmoid(logits)
        sparsity_loss = (probs.mean() - self.target_sparsity).pow(2)
        dist_entropy = -(probs * (probs + 1e-10).log() + (1.0 - probs) * (1.0 - probs + 1e-10).log())
        aux_loss = (self.sparsity_coef * sparsity_loss) + (self.entropy_coef * dist_entropy.mean())
        return RouterOutput(mask, indices, logits, aux_loss)


def depthwise_conv_seq(h: torch.Tensor, weight: torch.Tensor, padding: int = 1) -> torch.Tensor:
    """``conv(h.transpose(1, 2)).transpose(1, 2)`` of ReflexiveStream.forward
    (hspmn_v2_1.py:144) for ``h`` [B,S,D] and the depthwise Conv1d weight
    [D,1,k]: the same convolution, computed as a 2-D depthwise convolution
    of the [B,D,1,S] view of ``h``, whose memory is channels-last when ``h``
    is contiguous. PyTorch then runs its channels-last depthwise kernel on
    the memory as it lies and returns a contiguous [B,S,D] result, instead of
    copying ``h`` into [B,D,S] order, running the generic depthwise kernel
    and copying the transposed result again for the next GEMM. For bf16 and
    fp32 the results are bit-identical to the reference's call; fp16 keeps
    that call, since the channels-last kernel rounds a few fp16 outputs
    differently (by one unit in the last place)."""
    D = h.shape[2]
    if h.dtype == torch.float16:
        return F.conv1d(h.transpose(1, 2), weight, None, padding=padding, groups=D).transpose(1, 2)
    y = F.conv2d(h.contiguous().permute(0, 2, 1).unsqueeze(2), weight.unsqueeze(2), None, padding=(0, padding),
                 groups=D)
    return y.squeeze(2).permute(0, 2, 1)


class ReflexiveStream(nn.Module):
    """RMSNorm -> depthwise Conv1d(k=3) -> SwiGLU MLP, residual
    (hspmn_v2_1.py:125-145). Stock PyTorch; the convolution is called in the
    layout the [B,S,D] stream already has (``depthwise_conv_seq``)."""

    def __init__(self, dim: int, mlp_ratio: int = 4):
        super().__init__()
        hidden = dim * mlp_ratio
        self.conv = nn.Conv1d(dim, dim, kernel_size=3, padding=1, groups=dim, bias=False)
        self.norm = nn.RMSNorm(dim)
        self.gate_proj = nn.Linear(dim, hidden, bias=False)
        self.up_proj = nn.Linear(dim, hidden, bias=False)
        self.down_proj = nn.Linear(hidden, dim, bias=False)
        self._init_weights()

    def _init_weights(self):
        for w in [self.gate_proj, self.up_proj, self.down_proj]:
            nn.init.xavier_uniform_(w.weight, gain=0.02)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        res = x
        x = self.norm(x)
        x = depthwise_conv_seq(x, self.conv.weight, self.conv.padding[0])
        return res + self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class HSPMNBlock(nn.Module):
    """Reflexive stream + router-selected contextual stream
    (hspmn_v2_1.py:148-238). ``forward(x) -> (out, aux_loss)``."""

    def __init__(self, config: HSPMNConfig):
        super().__init__()
        self.config = config
        self.dim = config.dim
        self.head_dim = config.head_dim
        self.num_heads = config.num_heads
        self.num_kv_heads = config.num_kv_heads
        self.kv_dim = self.num_kv_heads * self.head_dim

        self.router = TopKRouter(config.dim, config.sparsity_k, config.router_sparsity_coef,
                                 config.router_entropy_coef)
        self.norm = nn.RMSNorm(config.dim)
        self.q_proj = nn.Linear(config.dim, config.dim, bias=False)
        self.k_proj = nn.Linear(config.dim, self.kv_dim, bias=False)
        self.v_proj = nn.Linear(config.dim, self.kv_dim, bias=False)
        self.o_proj = nn.Linear(config.dim, config.dim, bias=False)
        self.rope = RotaryEmbedding(self.head_dim, config.max_seq_len, config.rope_base)
        self.reflexive = ReflexiveStream(config.dim, config.mlp_ratio)
        # eval: run q_proj / RoPE / o_proj only on the routed rows (True), or
        # follow the reference's operation order on all rows (False)
        self.sqdk_fused = True
        # training: SQDK forward + backward kernels for bf16/f16 on CUDA (True),
        # or the reference's FlexAttention formulation (False)
        self.sqdk_train = True
        self._init_weights()

    def _init_weights(self):
        scale = 1.0 / math.sqrt(self.dim)
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.o_proj):
            nn.init.xavier_uniform_(lin.weight, gain=scale)

    # -- contextual stream, inference: the sm_100a path --------------------
    def _attention_sqdk(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        router_out: RouterOutput, B: int, S: int, D: int) -> torch.Tensor:
        """gather -> SQDK -> scatter -> o_proj (hspmn_v2_1.py:176-198), with
        grouped K/V heads read in place (no expansion)."""
        q_t = q.transpose(1, 2)  # [B,S,H,hd]
        k_t = k.transpose(1, 2)  # [B,S,Hkv,hd]
        v_t = v.transpose(1, 2)
        idx = router_out.indices
        q_sel = ops.gather_rows(q_t, idx)
        attn = ops.sqdk_fwd(q_sel, k_t, v_t, idx, 1.0 / math.sqrt(self.head_dim))
        out = ops.scatter_rows(attn, idx, S)
        return self.o_proj(out.view(B, S, D))

    def _attention_sqdk_fused(self, x_norm: torch.Tensor, idx: torch.Tensor, B: int, S: int,
                              D: int) -> torch.Tensor:
        """The same contextual stream with the work outside SQDK cut to the
        selected rows: q_proj on the gathered rows only, RoPE fused into their
        gather (bit-identical rows), K/V projections + RoPE on all rows as in
        the reference, and o_proj on the K attention rows only. Returns the
        [B,K,D] rows of ``o_proj(scatter(attn))`` (every other row is zero);
        the caller adds them into the residual at ``idx``."""
        H, Hkv, hd = self.num_heads, self.num_kv_heads, self.head_dim
        K = idx.shape[1]
        x_sel = ops.gather_rows(x_norm, idx)
        q_sel = self.q_proj(x_sel).view(B, K, H, hd)
        cos, sin = self.rope(x_norm, S)
        q_sel = ops.rope_gather_rows(q_sel, idx, cos, sin, False)
        # K RoPE on every position in one pass (same rounding as the reference's
        # three tensor ops, hspmn_v2_1.py:66-68)
        k = ops.rope_rows(self.k_proj(x_norm).view(B, S, Hkv, hd), cos, sin, 0)
        v = self.v_proj(x_norm).view(B, S, Hkv, hd)
        attn = ops.sqdk_fwd(q_sel, k, v, idx, 1.0 / math.sqrt(hd))
        return self.o_proj(attn.reshape(B, K, D))

    def _fused_ok(self, x: torch.Tensor) -> bool:
        vec = 16 // x.element_size()
        return self.sqdk_fused and self.head_dim % (2 * vec) == 0

    # -- contextual stream, training: SQDK forward + backward -------------
    def _sqdk_train_ok(self, q: torch.Tensor, router_out: RouterOutput) -> bool:
        return (self.sqdk_train and router_out.indices is not None and q.is_cuda
                and q.dtype in (torch.bfloat16, torch.float16) and self.head_dim % 8 == 0
                and self.head_dim <= 128 and self.num_heads // self.num_kv_heads <= 64)

    def _attention_sqdk_train(self, q, k, v, router_out: RouterOutput, B: int, S: int, D: int) -> torch.Tensor:
        """The contextual stream with gradients (the training branch of
        hspmn_v2_1.py:229-234): the selected query rows are gathered, attend
        through ``ops.sqdk_attention`` (forward and backward kernels) and are
        scattered into zero rows before o_proj, which is what the FlexAttention
        mask (q_idx >= kv_idx) & mask[b, q_idx] computes."""
        H, hd = self.num_heads, self.head_dim
        idx = router_out.indices
        K = idx.shape[1]
        q_t, k_t, v_t = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        sel = idx[:, :, None, None].expand(B, K, H, hd)
        q_sel = torch.gather(q_t, 1, sel)
        attn = ops.sqdk_attention(q_sel, k_t, v_t, idx, 1.0 / math.sqrt(hd))
        out = torch.zeros_like(q_t).scatter(1, sel, attn)
        return self.o_proj(out.reshape(B, S, D))

    # -- contextual stream, training: reference FlexAttention formulation --
    def _attention_flex(self, q, k, v, router_out: RouterOutput, B: int, S: int, D: int) -> torch.Tensor:
        from torch.nn.attention.flex_attention import create_block_mask
        sel = router_out.mask

        def block_mask_fn(b, h, q_idx, kv_idx):
            return (q_idx >= kv_idx) & sel[b, q_idx]

        block_mask = create_block_mask(block_mask_fn, B=B, H=self.num_heads, Q_LEN=S, KV_LEN=S,
                                       device=q.device, BLOCK_SIZE=self.config.block_size)
        out = get_compiled_flex_attention()(
            q, k, v, block_mask=block_mask, enable_gqa=(self.num_kv_heads != self.num_heads),
            scale=1.0 / math.sqrt(self.head_dim))
        return self.o_proj(out.transpose(1, 2).contiguous().view(B, S, D))

    def _attention(self, x: torch.Tensor, router_out: RouterOutput) -> torch.Tensor:
        B, S, D = x.shape
        x_norm = self.norm(x)
        q = self.q_proj(x_norm).view(B, S, self.num_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x_norm).view(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x_norm).view(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)
        cos, sin = self.rope(q, S)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        if router_out.indices is not None and not self.training:
            return self._attention_sqdk(q, k, v, router_out, B, S, D)
        if self._sqdk_train_ok(q, router_out):
            return self._attention_sqdk_train(q, k, v, router_out, B, S, D)
        return self._attention_flex(q, k, v, router_out, B, S, D)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        router_out = self.router(x)
        if not self.training and router_out.indices is not None and self._fused_ok(x):
            B, S, D = x.shape
            o_sel = self._attention_sqdk_fused(self.norm(x), router_out.indices, B, S, D)
            y = self.reflexive(x).contiguous()
            ops.scatter_add_rows_(y, router_out.indices, o_sel)
            return y, router_out.aux_loss
        return self.reflexive(x) + self._attention(x, router_out), router_out.aux_loss
