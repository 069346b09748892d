"""Transformer blocks with the reference's public API (``blocks/dit_block.py``,
``blocks/flow_matching.py``).

* :class:`DiTBlock` (dit_block.py:21-140): pre-norm attention + MLP with RMSNorm or AdaLN,
  returns ``(x, kv_cache)``. Unlike the reference, ``start_pos`` is honoured (RoPE
  positions continue across cached steps) and a causal block masks its new tokens even
  when a cache is passed.
* :class:`DiTBlockWithCrossAttention` (:143-246): the reference computes a second
  *self*-attention and never projects ``context``; here the cross-attention attends to the
  projected context.
* :class:`MemoryEfficientDiTBlock` (:249-307): activation checkpointing wrapper.
* :class:`MoEDiTBlock` (``layers/moe.py:427-547``): the same block with the MoE FFN.
* :class:`FlowMatchingBlock` / :class:`FlowPredictor` (flow_matching.py:94-218): 6-way
  AdaLN-Zero modulation from the time embedding, zero-initialised output.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from ..layers.attention import (BidirectionalMultiHeadAttention, CausalMultiHeadAttention,
                                CrossAttention, MultiHeadAttention)
from ..layers.mlp import MLP, create_mlp
from ..layers.norms import AdaLN, RMSNorm
from ..layers.rope import RoPELayer


class DiTBlock(nn.Module):
    def __init__(self, d_model: int, n_heads: int, d_ff: Optional[int] = None,
                 mlp_type: str = "swiglu", dropout: float = 0.0, causal: bool = True,
                 use_rope: bool = True, max_seq_len: int = 2048, cond_dim: Optional[int] = None,
                 bias: bool = False, tokens_per_frame: Optional[int] = None):
        super().__init__()
        self.d_model, self.n_heads, self.causal, self.cond_dim = d_model, n_heads, causal, cond_dim
        self.rope_layer = RoPELayer(d_model // n_heads, max_seq_len) if use_rope else None
        cls = CausalMultiHeadAttention if causal else BidirectionalMultiHeadAttention
        self.attn = cls(d_model, n_heads, dropout=dropout, bias=bias, rope_layer=self.rope_layer,
                        tokens_per_frame=tokens_per_frame)
        self.mlp = create_mlp(d_model, mlp_type, d_ff, dropout, bias)
        if cond_dim is not None:
            self.norm_attn = AdaLN(d_model, cond_dim)
            self.norm_mlp = AdaLN(d_model, cond_dim)
        else:
            self.norm_attn = RMSNorm(d_model)
            self.norm_mlp = RMSNorm(d_model)

    def _norm(self, norm, x, cond):
        return norm(x, cond) if (self.cond_dim is not None and cond is not None) else (
            norm.norm(x) if isinstance(norm, AdaLN) else norm(x))

    def forward(self, x: torch.Tensor, kv_cache=None, pos=None, cond: Optional[torch.Tensor] = None,
                causal_mask: Optional[torch.Tensor] = None, start_pos: Optional[int] = None):
        h = self._norm(self.norm_attn, x, cond)
        if causal_mask is not None:
            a, new_cache = MultiHeadAttention.forward(self.attn, h, kv_cache, causal_mask, start_pos)
        else:
            a, new_cache = self.attn(h, kv_cache=kv_cache, start_pos=start_pos)
        x = x + a
        x = x + self.mlp(self._norm(self.norm_mlp, x, cond))
        return x, new_cache


class DiTBlockWithCrossAttention(DiTBlock):
    def __init__(self, d_model: int, n_heads: int, context_dim: Optional[int] = None, **kw):
        super().__init__(d_model, n_heads, **kw)
        self.norm_cross = RMSNorm(d_model)
        self.cross_attn = CrossAttention(d_model, n_heads, context_dim)

    def forward(self, x, context: Optional[torch.Tensor] = None, kv_cache=None, pos=None,
                cond=None, causal_mask=None, start_pos=None, context_mask=None):
        h = self._norm(self.norm_attn, x, cond)
        a, new_cache = self.attn(h, kv_cache=kv_cache, start_pos=start_pos)
        x = x + a
        if context is not None:
            x = x + self.cross_attn(self.norm_cross(x), context, context_mask)
        x = x + self.mlp(self._norm(self.norm_mlp, x, cond))
        return x, new_cache


class MemoryEfficientDiTBlock(DiTBlock):
    """Recomputes the block in the backward pass (activation checkpointing)."""

    def forward(self, x, kv_cache=None, pos=None, cond=None, causal_mask=None, start_pos=None):
        if self.training and kv_cache is None and x.requires_grad:
            fn = lambda x_, c_: DiTBlock.forward(self, x_, None, None, c_, causal_mask, start_pos)[0]
            return checkpoint(fn, x, cond, use_reentrant=False), None
        return super().forward(x, kv_cache, pos, cond, causal_mask, start_pos)


class MoEDiTBlock(DiTBlock):
    """DiT block whose FFN is the DeepSeek-style MoE (reference ``layers/moe.py:427-547``):
    returns ``(x, kv_cache)`` like :class:`DiTBlock`; the last load-balance loss and
    (when asked for) routing metrics stay on the block."""

    def __init__(self, d_model: int, n_heads: int, num_experts: int = 8, top_k: int = 2,
                 expert_dim: Optional[int] = None, num_shared_experts: int = 0, dropout: float = 0.0,
                 causal: bool = True, use_rope: bool = True, max_seq_len: int = 2048,
                 cond_dim: Optional[int] = None, bias: bool = False, jitter_noise: float = 0.0,
                 bias_update_speed: float = 0.001, aux_loss_weight: float = 0.0,
                 tokens_per_frame: Optional[int] = None):
        from ..layers.moe import MoEFFN

        super().__init__(d_model, n_heads, d_ff=None, dropout=dropout, causal=causal, use_rope=use_rope,
                         max_seq_len=max_seq_len, cond_dim=cond_dim, bias=bias,
                         tokens_per_frame=tokens_per_frame)
        del self.mlp
        self.moe_ffn = MoEFFN(d_model, num_experts, top_k, expert_dim, num_shared_experts, dropout,
                              jitter_noise=jitter_noise, bias_update_speed=bias_update_speed,
                              aux_loss_weight=aux_loss_weight)
        self._last_moe_metrics = None
        self._last_aux_loss = None

    def forward(self, x, kv_cache=None, pos=None, cond=None, causal_mask=None, start_pos=None,
                return_moe_metrics: bool = False):
        h = self._norm(self.norm_attn, x, cond)
        if causal_mask is not None:
            a, new_cache = MultiHeadAttention.forward(self.attn, h, kv_cache, causal_mask, start_pos)
        else:
            a, new_cache = self.attn(h, kv_cache=kv_cache, start_pos=start_pos)
        x = x + a
        out = self.moe_ffn(self._norm(self.norm_mlp, x, cond), return_metrics=return_moe_metrics)
        self._last_aux_loss = out.aux_loss
        if return_moe_metrics:
            self._last_moe_metrics = out.metrics
        return x + out.output, new_cache

    def get_aux_loss(self):
        return self._last_aux_loss

    def get_moe_metrics(self):
        return self._last_moe_metrics

    def get_load_balance_stats(self):
        return self.moe_ffn.get_load_balance_stats()


def create_moe_dit_block(d_model: int, n_heads: int, num_experts: int = 8, top_k: int = 2,
                         **kw) -> MoEDiTBlock:
    return MoEDiTBlock(d_model, n_heads, num_experts=num_experts, top_k=top_k, **kw)


def create_dit_block(block_type: str = "standard", **kw) -> nn.Module:
    return {"standard": DiTBlock, "cross_attention": DiTBlockWithCrossAttention,
            "memory_efficient": MemoryEfficientDiTBlock, "moe": MoEDiTBlock}[block_type](**kw)


# ----------------------------------------------------------------------------- flow matching
class FlowTimestepEmbedding(nn.Module):
    """256 Fourier features of ``t`` (in [0, 1], scaled by ``time_scale``) -> MLP."""

    def __init__(self, dim: int, fourier_features: int = 256, time_scale: float = 1.0):
        super().__init__()
        self.fourier_features, self.time_scale = fourier_features, time_scale
        self.linear1 = nn.Linear(fourier_features, dim)
        self.linear2 = nn.Linear(dim, dim)

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        half = self.fourier_features // 2
        freq = torch.exp(-torch.log(torch.tensor(10000.0)) * torch.arange(half, device=t.device)
                         / (half - 1))
        ang = t.float()[:, None] * self.time_scale * freq[None]
        return self.linear2(F.silu(self.linear1(torch.cat([ang.sin(), ang.cos()], -1))))


class FlowMatchingBlock(nn.Module):
    """Bidirectional block with AdaLN-Zero (shift, scale, gate) x 2 from the time embedding."""

    def __init__(self, d_model: int, n_heads: int, d_ff: Optional[int] = None, dropout: float = 0.0):
        super().__init__()
        self.norm1 = RMSNorm(d_model)
        self.attn = BidirectionalMultiHeadAttention(d_model, n_heads, dropout=dropout)
        self.norm2 = RMSNorm(d_model)
        self.mlp = MLP(d_model, d_ff or 4 * d_model, "gelu", dropout)
        self.modulation = nn.Sequential(nn.SiLU(), nn.Linear(d_model, 6 * d_model))
        nn.init.zeros_(self.modulation[1].weight)
        nn.init.zeros_(self.modulation[1].bias)

    def forward(self, x: torch.Tensor, t_emb: torch.Tensor) -> torch.Tensor:
        sh1, sc1, g1, sh2, sc2, g2 = self.modulation(t_emb)[:, None].chunk(6, -1)
        x = x + g1 * self.attn(self.norm1(x) * (1 + sc1) + sh1)[0]
        return x + g2 * self.mlp(self.norm2(x) * (1 + sc2) + sh2)


class FlowPredictor(nn.Module):
    """Velocity network ``v(z_t, t[, context])`` over token sequences ``[B, T, latent_dim]``."""

    def __init__(self, latent_dim: int, d_model: int = 512, n_layers: int = 6, n_heads: int = 8,
                 d_ff: Optional[int] = None, context_dim: Optional[int] = None):
        super().__init__()
        self.time_embed = FlowTimestepEmbedding(d_model)
        self.input_proj = nn.Linear(latent_dim, d_model)
        self.context_proj = nn.Linear(context_dim, d_model) if context_dim else None
        self.blocks = nn.ModuleList([FlowMatchingBlock(d_model, n_heads, d_ff) for _ in range(n_layers)])
        self.norm = RMSNorm(d_model)
        self.output_proj = nn.Linear(d_model, latent_dim)
        nn.init.zeros_(self.output_proj.weight)
        nn.init.zeros_(self.output_proj.bias)

    def forward(self, z_t: torch.Tensor, t: torch.Tensor, context: Optional[torch.Tensor] = None):
        if t.dim() == 0:
            t = t.expand(z_t.shape[0])
        te = self.time_embed(t)
        x = self.input_proj(z_t)
        if context is not None and self.context_proj is not None:
            x = x + self.context_proj(context).mean(1, keepdim=True)
        for blk in self.blocks:
            x = blk(x, te)
        return self.output_proj(self.norm(x))
