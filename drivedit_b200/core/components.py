"""Earlier-generation building blocks (the reference's ``core/components.py``): a
materialised 3-D RoPE, multi-head attention with KV cache and cross-attention,
pre-LayerNorm transformer block, causal video transformer, a SAM2-style object-memory
tracker, adaptive LayerNorm and a time-conditioned flow predictor.

Kept for users of that API; the world models use :mod:`drivedit_b200.layers`. One fix: the
reference's attention assumes a square ``sqrt(T) x sqrt(T)`` spatial grid when it builds
RoPE positions (``:165``), which is wrong for every non-square or multi-frame sequence;
here the grid ``(frames, height, width)`` is an argument (default: one row of ``T``
tokens), and positions continue after a KV cache.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class RoPE3D(nn.Module):
    """Tables ``sin, cos [T, H, W, dim]``: the first third of the rotary channels rotates
    with the frame index, the second with the row, the rest with the column."""

    def __init__(self, dim: int, max_seq_len: int = 512, temperature: float = 10000.0):
        super().__init__()
        self.dim, self.max_seq_len, self.temperature = dim, max_seq_len, temperature
        self.register_buffer("inv_freq", 1.0 / temperature ** (torch.arange(0, dim, 2).float() / dim),
                             persistent=False)

    def forward(self, seq_len: int, height: int, width: int) -> Tuple[torch.Tensor, torch.Tensor]:
        dev = self.inv_freq.device
        ang = [torch.outer(torch.arange(n, device=dev, dtype=torch.float32), self.inv_freq)
               for n in (seq_len, height, width)]
        third = self.dim // 3
        half = self.inv_freq.numel()
        full = [torch.cat([a, a], -1)[..., :self.dim] if 2 * half >= self.dim else a for a in ang]
        t, h, w = full
        emb = torch.empty(seq_len, height, width, self.dim, device=dev)
        emb[..., :third] = t[:, None, None, :third]
        emb[..., third:2 * third] = h[None, :, None, third:2 * third]
        emb[..., 2 * third:] = w[None, None, :, 2 * third:]
        return emb.sin(), emb.cos()

    @staticmethod
    def apply_rope(q: torch.Tensor, k: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor):
        def rot(x):
            a, b = x.chunk(2, -1)
            return torch.cat([-b, a], -1)

        return q * cos + rot(q) * sin, k * cos + rot(k) * sin


class MultiHeadAttention(nn.Module):
    def __init__(self, dim: int, num_heads: int = 8, causal: bool = False, dropout: float = 0.1,
                 use_rope: bool = True):
        super().__init__()
        assert dim % num_heads == 0
        self.dim, self.num_heads, self.head_dim = dim, num_heads, dim // num_heads
        self.causal, self.use_rope, self.dropout = causal, use_rope, dropout
        self.qkv = nn.Linear(dim, 3 * dim, bias=False)
        self.proj = nn.Linear(dim, dim)
        if use_rope:
            self.rope = RoPE3D(self.head_dim)

    def forward(self, x: torch.Tensor, kv: Optional[torch.Tensor] = None,
                past_kv: Optional[Dict[str, torch.Tensor]] = None, use_cache: bool = False,
                attn_mask: Optional[torch.Tensor] = None, grid: Optional[Tuple[int, int, int]] = None):
        B, T, D = x.shape
        H, hd = self.num_heads, self.head_dim
        if kv is not None:
            q = F.linear(x, self.qkv.weight[:D])
            k, v = F.linear(kv, self.qkv.weight[D:]).chunk(2, -1)
        else:
            q, k, v = self.qkv(x).chunk(3, -1)
        q = q.view(B, T, H, hd).transpose(1, 2)
        k = k.reshape(B, -1, H, hd).transpose(1, 2)
        v = v.reshape(B, -1, H, hd).transpose(1, 2)
        past = 0
        if self.use_rope and kv is None:
            past = 0 if past_kv is None else past_kv["k"].shape[2]
            g = grid or (1, 1, past + T)
            sin, cos = self.rope(*g)
            sin = sin.reshape(-1, hd)[past:past + T]
            cos = cos.reshape(-1, hd)[past:past + T]
            q, k = self.rope.apply_rope(q, k, sin, cos)
        if past_kv is not None:
            k = torch.cat([past_kv["k"], k], 2)
            v = torch.cat([past_kv["v"], v], 2)
        mask = None
        if self.causal:
            S = k.shape[2]
            mask = torch.arange(S, device=x.device)[None] <= (torch.arange(T, device=x.device)[:, None] + S - T)
        if attn_mask is not None:
            am = attn_mask if attn_mask.dtype != torch.bool else torch.zeros_like(attn_mask, dtype=q.dtype).masked_fill(~attn_mask, float("-inf"))
            mask = am if mask is None else am.masked_fill(~mask, float("-inf"))
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask,
                                           dropout_p=self.dropout if self.training else 0.0)
        out = self.proj(o.transpose(1, 2).reshape(B, T, D))
        return out, ({"k": k.detach(), "v": v.detach()} if use_cache else None)


class TransformerBlock(nn.Module):
    def __init__(self, dim: int, num_heads: int = 8, mlp_ratio: int = 4, causal: bool = False,
                 cross_attention: bool = False, dropout: float = 0.1, use_rope: bool = True):
        super().__init__()
        self.cross_attention = cross_attention
        self.norm1 = nn.LayerNorm(dim)
        self.self_attn = MultiHeadAttention(dim, num_heads, causal, dropout, use_rope)
        if cross_attention:
            self.norm_cross = nn.LayerNorm(dim)
            self.cross_attn = MultiHeadAttention(dim, num_heads, False, dropout, use_rope=False)
        self.norm2 = nn.LayerNorm(dim)
        self.mlp = nn.Sequential(nn.Linear(dim, dim * mlp_ratio), nn.GELU(), nn.Dropout(dropout),
                                 nn.Linear(dim * mlp_ratio, dim), nn.Dropout(dropout))

    def forward(self, x, context=None, past_kv=None, use_cache: bool = False, attn_mask=None, grid=None):
        a, cache = self.self_attn(self.norm1(x), past_kv=past_kv, use_cache=use_cache, attn_mask=attn_mask,
                                  grid=grid)
        x = x + a
        if self.cross_attention and context is not None:
            x = x + self.cross_attn(self.norm_cross(x), kv=context)[0]
        return x + self.mlp(self.norm2(x)), cache


class CausalVideoTransformer(nn.Module):
    """Stack of causal blocks; the second half cross-attends to ``context`` by default."""

    def __init__(self, dim: int = 512, num_layers: int = 12, num_heads: int = 8, mlp_ratio: int = 4,
                 max_seq_len: int = 512, cross_attention_layers: Optional[List[int]] = None, dropout: float = 0.1):
        super().__init__()
        self.dim, self.num_layers, self.max_seq_len = dim, num_layers, max_seq_len
        xl = set(range(num_layers // 2, num_layers) if cross_attention_layers is None else cross_attention_layers)
        self.layers = nn.ModuleList([TransformerBlock(dim, num_heads, mlp_ratio, True, i in xl, dropout, True)
                                     for i in range(num_layers)])
        self.norm = nn.LayerNorm(dim)

    def forward(self, x, context=None, past_kvs=None, use_cache: bool = False):
        past_kvs = past_kvs or [None] * self.num_layers
        new = [] if use_cache else None
        for layer, pk in zip(self.layers, past_kvs):
            x, c = layer(x, context=context, past_kv=pk, use_cache=use_cache)
            if use_cache:
                new.append(c)
        return self.norm(x), new


class SAM2InspiredTracker(nn.Module):
    """Per-frame object features (conv encoder) written into learned object-memory slots
    by attention (memory slots query the observed features)."""

    def __init__(self, dim: int = 256, max_objects: int = 32):
        super().__init__()
        self.dim, self.max_objects = dim, max_objects
        self.object_encoder = nn.Sequential(
            nn.Conv2d(3, 64, 3, padding=1), nn.ReLU(), nn.Conv2d(64, 128, 3, stride=2, padding=1), nn.ReLU(),
            nn.Conv2d(128, 256, 3, stride=2, padding=1), nn.ReLU(), nn.AdaptiveAvgPool2d((8, 8)), nn.Flatten(),
            nn.Linear(256 * 64, dim))
        self.object_memory = nn.Parameter(torch.randn(max_objects, dim) * 0.02)
        self.memory_attention = MultiHeadAttention(dim, num_heads=8 if dim % 8 == 0 else 1, use_rope=False,
                                                   dropout=0.0)
        self.object_states: Dict[int, torch.Tensor] = {}

    def encode_objects(self, frames: torch.Tensor) -> torch.Tensor:
        B, T = frames.shape[:2]
        return self.object_encoder(frames.flatten(0, 1)).view(B, T, self.dim)

    def update_memory(self, object_features: torch.Tensor, frame_idx: int = 0) -> torch.Tensor:
        B = object_features.shape[0]
        mem = self.object_memory.unsqueeze(0).expand(B, -1, -1)
        out, _ = self.memory_attention(mem, kv=object_features.reshape(B, -1, self.dim))
        self.object_states[frame_idx] = out.detach()
        return out

    def get_memory_tokens(self, batch_size: int) -> torch.Tensor:
        return self.object_memory.unsqueeze(0).expand(batch_size, -1, -1)


class AdaptiveLayerNorm(nn.Module):
    """``LayerNorm(x) * scale(c) + shift(c)``, initialised to the identity."""

    def __init__(self, dim: int, condition_dim: int):
        super().__init__()
        self.norm = nn.LayerNorm(dim, elementwise_affine=False)
        self.scale = nn.Linear(condition_dim, dim)
        self.shift = nn.Linear(condition_dim, dim)
        nn.init.zeros_(self.scale.weight)
        nn.init.ones_(self.scale.bias)
        nn.init.zeros_(self.shift.weight)
        nn.init.zeros_(self.shift.bias)

    def forward(self, x: torch.Tensor, condition: torch.Tensor) -> torch.Tensor:
        s, b = self.scale(condition), self.shift(condition)
        if x.dim() == 3 and s.dim() == 2:
            s, b = s.unsqueeze(1), b.unsqueeze(1)
        return self.norm(x) * s + b


class FlowMatchingPredictor(nn.Module):
    """Velocity MLP over ``[z, embed(t)]`` with Euler sampling."""

    def __init__(self, dim: int, num_steps: int = 4):
        super().__init__()
        self.dim, self.num_steps = dim, num_steps
        self.time_embed = nn.Sequential(nn.Linear(1, dim), nn.SiLU(), nn.Linear(dim, dim))
        self.flow_net = nn.Sequential(nn.Linear(2 * dim, 2 * dim), nn.SiLU(), nn.Linear(2 * dim, dim), nn.Tanh())

    def forward(self, z: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        te = self.time_embed(t.to(z.dtype).reshape(*t.shape, 1))
        while te.dim() < z.dim():
            te = te.unsqueeze(-2)
        return self.flow_net(torch.cat([z, te.expand_as(z)], -1))

    @torch.no_grad()
    def sample(self, z_init: torch.Tensor, num_steps: Optional[int] = None) -> torch.Tensor:
        n = num_steps or self.num_steps
        z = z_init.clone()
        for i in range(n):
            z = z + self.forward(z, torch.full((z.shape[0],), i / n, device=z.device)) / n
        return z


def create_attention_mask(seq_len: int, causal: bool = True, device=None) -> torch.Tensor:
    """Additive mask ``[seq_len, seq_len]`` (core/components.py:496-502): 0 where a query
    may attend, ``-inf`` above the diagonal when ``causal``; all zeros otherwise."""
    if not causal:
        return torch.zeros(seq_len, seq_len, device=device)
    return torch.full((seq_len, seq_len), float("-inf"), device=device).triu(1)


from ..utils.model_utils import count_parameters  # noqa: E402,F401  (the reference exports it here too)
