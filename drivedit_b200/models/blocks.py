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
* :class:`FlowMatchingConfig`, :class:`FlowMatchingBlock`, :class:`FlowPredictor`
  (flow_matching.py:35-218): the reference's module names and call signatures, so its
  weights and configs load; the predictor can also map a token width other than ``dim``.
"""
from __future__ import annotations

from dataclasses import dataclass
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
        self.mlp = create_mlp(d_model, mlp_type=mlp_type, d_ff=d_ff, dropout=dropout, bias=bias)
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
    """:class:`DiTBlock` plus attention from the tokens to a projected ``context``
    between the self-attention and the MLP, normalised by ``norm_cross`` (AdaLN when
    ``cond_dim`` is set). The reference's constructor and call (blocks/dit_block.py:
    143-246); its forward returns ``(x, kv_cache, cross_kv_cache)``, where the cross cache
    holds the context's projected keys and values, so a streaming caller projects a
    fixed context once."""

    def __init__(self, d_model: int, n_heads: int, d_ff: Optional[int] = None,
                 mlp_type: str = "swiglu", dropout: float = 0.0, causal: bool = True,
                 use_rope: bool = True, max_seq_len: int = 2048, cond_dim: Optional[int] = None,
                 bias: bool = False, context_dim: Optional[int] = None,
                 tokens_per_frame: Optional[int] = None):
        super().__init__(d_model, n_heads, d_ff, mlp_type, dropout, causal, use_rope, max_seq_len,
                         cond_dim, bias, tokens_per_frame)
        self.norm_cross = AdaLN(d_model, cond_dim) if cond_dim is not None else RMSNorm(d_model)
        self.cross_attn = CrossAttention(d_model, n_heads, context_dim, bias=bias)

    def forward(self, x, context: Optional[torch.Tensor] = None, kv_cache=None,
                cross_kv_cache: Optional[Dict[str, torch.Tensor]] = None, pos=None, cond=None,
                causal_mask=None, start_pos=None, context_mask=None):
        h = self._norm(self.norm_attn, x, cond)
        if causal_mask is not None:
            a, new_cache = MultiHeadAttention.forward(self.attn, h, kv_cache, causal_mask, start_pos)
        else:
            a, new_cache = self.attn(h, kv_cache=kv_cache, start_pos=start_pos)
        x = x + a
        new_cross = cross_kv_cache
        if context is not None or cross_kv_cache is not None:
            if new_cross is None:
                new_cross = self.cross_attn.project_context(context)
            x = x + self.cross_attn.attend(self._norm(self.norm_cross, x, cond), new_cross, context_mask)
        x = x + self.mlp(self._norm(self.norm_mlp, x, cond))
        return x, new_cache, new_cross


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


def create_dit_block(d_model: int, n_heads: int, block_type: str = "standard", **kwargs) -> nn.Module:
    """``standard``, ``cross_attn`` (also ``cross_attention``), ``memory_efficient`` or
    ``moe`` (blocks/dit_block.py:310-335)."""
    kinds = {"standard": DiTBlock, "cross_attn": DiTBlockWithCrossAttention,
             "cross_attention": DiTBlockWithCrossAttention,
             "memory_efficient": MemoryEfficientDiTBlock, "moe": MoEDiTBlock}
    if block_type not in kinds:
        raise ValueError(f"Unsupported block type: {block_type}")
    return kinds[block_type](d_model, n_heads, **kwargs)


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


@dataclass
class FlowMatchingConfig:
    """Settings of the flow-matching predictor, sampler and trainer (the reference's
    schema, blocks/flow_matching.py:35-59, kept field for field so its configs load).
    ``latent_dim`` and ``context_dim`` are additions: the token width when it differs
    from ``dim`` (an input and an output projection then map between them), and the
    width of a context that is projected to ``dim`` instead of added as it is."""
    dim: int = 512
    num_layers: int = 6
    num_heads: int = 8
    mlp_ratio: int = 4
    num_steps: int = 4
    sigma_min: float = 1e-4
    sigma_max: float = 80.0
    use_cfg: bool = True
    cfg_scale: float = 7.5
    teacher_steps: int = 4
    student_steps: int = 1
    distillation_weight: float = 1.0
    time_embed_dim: int = 128
    fourier_features: int = 256
    latent_dim: Optional[int] = None
    context_dim: Optional[int] = None


class FlowMatchingBlock(nn.Module):
    """Bidirectional transformer block modulated by the time embedding: ``time_mlp`` maps
    it to (scale, shift, gate) for the attention and for the MLP, in that order, and each
    branch computes ``x + gate * f(norm(x) * (1 + scale) + shift)``
    (blocks/flow_matching.py:94-146; same module names, so its weights load)."""

    def __init__(self, dim: int, num_heads: int, mlp_ratio: int = 4):
        super().__init__()
        self.dim, self.num_heads = dim, num_heads
        self.norm1 = RMSNorm(dim)
        self.norm2 = RMSNorm(dim)
        self.time_mlp = nn.Sequential(nn.SiLU(), nn.Linear(dim, 6 * dim))
        self.attention = MultiHeadAttention(dim, num_heads)
        self.mlp = MLP(dim, dim * mlp_ratio)

    def forward(self, x: torch.Tensor, time_emb: torch.Tensor,
                mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        mods = self.time_mlp(time_emb)[:, None]
        sc1, sh1, g1, sc2, sh2, g2 = mods.chunk(6, dim=-1)
        a, _ = self.attention(torch.addcmul(sh1, self.norm1(x), 1 + sc1), mask=mask)
        x = torch.addcmul(x, g1, a)
        return torch.addcmul(x, g2, self.mlp(torch.addcmul(sh2, self.norm2(x), 1 + sc2)))


class FlowPredictor(nn.Module):
    """Velocity network ``v(z_t, t)`` over token sequences: time embedding, input
    projection, :class:`FlowMatchingBlock` stack, RMSNorm + zero-initialised output
    projection (blocks/flow_matching.py:149-218; same module names). A context
    ``[B, C, D]`` enters as its token mean added to every token."""

    def __init__(self, config: FlowMatchingConfig):
        super().__init__()
        self.config = config
        d, ld = config.dim, config.latent_dim or config.dim
        self.time_embed = FlowTimestepEmbedding(d, config.fourier_features, time_scale=1.0)
        self.input_proj = nn.Linear(ld, d)
        self.context_proj = nn.Linear(config.context_dim, d) if config.context_dim else None
        self.blocks = nn.ModuleList([FlowMatchingBlock(d, config.num_heads, config.mlp_ratio)
                                     for _ in range(config.num_layers)])
        self.output_proj = nn.Sequential(RMSNorm(d), nn.Linear(d, ld))
        nn.init.zeros_(self.output_proj[1].weight)
        nn.init.zeros_(self.output_proj[1].bias)

    def forward(self, z: torch.Tensor, t: torch.Tensor, mask: Optional[torch.Tensor] = None,
                context: Optional[torch.Tensor] = None) -> torch.Tensor:
        if t.dim() == 0:
            t = t.expand(z.shape[0])
        te = self.time_embed(t)
        h = self.input_proj(z)
        if context is not None:
            c = self.context_proj(context) if self.context_proj is not None else context
            h = h + c.mean(dim=1, keepdim=True)
        for blk in self.blocks:
            h = blk(h, te, mask)
        return self.output_proj(h)
