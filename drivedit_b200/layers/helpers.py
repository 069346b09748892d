"""Small building blocks from the reference's ``layers/nn_helpers.py``: activations,
the gate/up-fused MLP, a scaled-dot-product attention module, the residual-add + norm
helper, rotate-half rotary embedding and sinusoidal absolute positions
(reference :13-36, :142-356).

On CUDA, :class:`FusedMLP` runs its two projections on this framework's tcgen05 GEMM
(one GEMM for gate and up together, as in the reference) and
:class:`ScaledDotProductAttention` runs the sm_100a flash-attention forward kernel for
inference calls (no gradient needed, d_head 64, no explicit mask); training calls and
other shapes use the PyTorch formula, which is also the CPU path.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def silu(x: torch.Tensor) -> torch.Tensor:
    """``x * sigmoid(x)``."""
    return F.silu(x)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """GELU with the tanh approximation (Hendrycks & Gimpel)."""
    return F.gelu(x, approximate="tanh")


class FusedMLP(nn.Module):
    """``down(act(gate) * up)`` with gate and up produced by one ``[2 d_ff, d]``
    projection (its rows: gate then up). Parameter names follow the reference
    (``gate_up_proj``, ``down_proj``)."""

    def __init__(self, d_model: int, d_ff: int, activation: str = "silu", bias: bool = False):
        super().__init__()
        if activation not in ("silu", "gelu"):
            raise ValueError(f"Unsupported activation: {activation}")
        self.d_model, self.d_ff, self.activation_name = d_model, d_ff, activation
        self.gate_up_proj = nn.Linear(d_model, 2 * d_ff, bias=bias)
        self.down_proj = nn.Linear(d_ff, d_model, bias=bias)
        nn.init.normal_(self.gate_up_proj.weight, std=0.02)
        nn.init.normal_(self.down_proj.weight, std=0.02 / math.sqrt(24))
        for lin in (self.gate_up_proj, self.down_proj):
            if lin.bias is not None:
                nn.init.zeros_(lin.bias)

    def activation(self, x: torch.Tensor) -> torch.Tensor:
        return F.silu(x) if self.activation_name == "silu" else F.gelu(x)

    def _proj(self, x: torch.Tensor, lin: nn.Linear) -> torch.Tensor:
        if x.is_cuda and x.shape[-1] % 64 == 0 and lin.out_features % 64 == 0:
            from ..ops.linear import linear

            flat = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
            b = lin.bias.float() if lin.bias is not None else None
            y = linear(flat, lin.weight.to(torch.bfloat16), b, lin.weight, lin.bias)
            return y.view(*x.shape[:-1], -1)
        return lin(x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate, up = self._proj(x, self.gate_up_proj).chunk(2, dim=-1)
        return self._proj((self.activation(gate) * up).contiguous(), self.down_proj)


class ScaledDotProductAttention(nn.Module):
    """``softmax(q k^T / sqrt(d) [masked]) v`` on ``[B, H, T, D]`` tensors. A mask holds 0
    where attention is blocked. ``use_flash`` without a mask means causal attention
    (the reference's convention)."""

    def __init__(self, dropout: float = 0.0, use_flash: bool = False):
        super().__init__()
        self.dropout, self.use_flash = dropout, use_flash

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        causal = self.use_flash and mask is None
        p_drop = self.dropout if self.training else 0.0
        needs_grad = torch.is_grad_enabled() and (q.requires_grad or k.requires_grad
                                                  or v.requires_grad)
        if (q.is_cuda and mask is None and p_drop == 0.0 and q.shape[-1] == 64
                and not needs_grad and k.shape == v.shape):
            from ..ops.attention_kernels import flash_attention

            bf = lambda t: t.transpose(1, 2).to(torch.bfloat16).contiguous()
            # causal: query i sees keys 0..i (top-left aligned, as in the formula below)
            o, _ = flash_attention(bf(q), bf(k), bf(v), "token" if causal else "none")
            return o.transpose(1, 2).to(q.dtype)
        scores = (q @ k.transpose(-2, -1)) / math.sqrt(q.shape[-1])
        if mask is not None:
            scores = scores.masked_fill(mask == 0, float("-inf"))
        elif causal:
            T, S = scores.shape[-2:]
            keep = torch.ones(T, S, dtype=torch.bool, device=q.device).tril()
            scores = scores.masked_fill(~keep, float("-inf"))
        w = scores.softmax(dim=-1)
        if p_drop > 0.0:
            w = F.dropout(w, p=p_drop)
        return w @ v


def fused_add_norm(x: torch.Tensor, residual: torch.Tensor,
                   norm: nn.Module) -> Tuple[torch.Tensor, torch.Tensor]:
    """``residual + x`` and its normalisation: returns ``(norm(sum), sum)``."""
    total = residual + x
    return norm(total), total


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rotary_pos_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                         position_ids: Optional[torch.Tensor] = None
                         ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotate-half rotary embedding on ``[B, H, T, D]`` q/k. ``cos``/``sin`` are
    ``[T, D]`` or ``[B, T, D]`` (or their ``D/2`` halves, repeated to full width);
    ``position_ids [B, T]`` gathers their rows."""
    if position_ids is not None:
        cos, sin = cos[position_ids], sin[position_ids]
    if cos.shape[-1] * 2 == q.shape[-1]:
        cos, sin = torch.cat([cos, cos], -1), torch.cat([sin, sin], -1)
    if cos.dim() == 2:
        cos, sin = cos[None, None], sin[None, None]
    elif cos.dim() == 3:
        cos, sin = cos[:, None], sin[:, None]
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


class PositionalEncoding(nn.Module):
    """Sinusoidal absolute positions added to ``[B, T, D]`` (Vaswani et al.): even
    channels ``sin(p w_i)``, odd channels ``cos(p w_i)``, ``w_i = 10000^(-2i/D)``."""

    def __init__(self, d_model: int, max_len: int = 5000):
        super().__init__()
        w = torch.exp(torch.arange(0, d_model, 2, dtype=torch.float64) * (-math.log(1e4) / d_model))
        ang = torch.arange(max_len, dtype=torch.float64)[:, None] * w[None, :]
        pe = torch.stack([ang.sin(), ang.cos()], -1).reshape(max_len, -1)[:, :d_model]
        self.register_buffer("pe", pe.float()[None])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.pe[:, :x.shape[1]].to(x.dtype)
