"""Causal DiT student and bidirectional DiT teacher with the reference's public API.

``DiTStudent`` (reference models/dit_student.py:215-507) — token embedding (latent
projection, 4-d control projection, modality embedding, sinusoidal position), causal
``DiTBlock`` stack with per-layer KV caches, RMSNorm, ``lm_head`` to latent space, an
optional attention ``MemoryBank`` (:109-212), ``generate`` (continuous "sampling" =
prediction + temperature-scaled noise, :394-475) and ``compute_loss`` (MSE, :477-507).
Fixes: cached steps pass ``start_pos`` so RoPE positions continue (reference
:362-366 restarts them at 0), and the causal mask covers new tokens with a cache.

``DiTTeacher`` (reference models/dit_teacher.py:123-484; its constructor raises TypeError
in the reference, :195) — bidirectional blocks conditioned on the flow time through AdaLN,
flow-matching ``add_noise``/``compute_loss``/``sample`` (Euler) and ``distill_to_student``.

State-dict keys follow the reference (``token_embed.*``, ``blocks.N.attn.qkv.weight``,
``blocks.N.mlp.w1.weight``, ``norm.weight``, ``lm_head.weight``, ``memory_bank.*``).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..layers.norms import RMSNorm
from ..training.flow_matching import interpolate
from .blocks import DiTBlock, FlowTimestepEmbedding


class PositionalEncoding(nn.Module):
    """Sinusoidal absolute position encoding added to ``[B, T, D]`` (buffer name ``pe``)."""

    def __init__(self, d_model: int, max_len: int = 2048):
        super().__init__()
        pos = torch.arange(max_len, dtype=torch.float32)[:, None]
        div = torch.exp(torch.arange(0, d_model, 2, dtype=torch.float32) * (-math.log(10000.0) / d_model))
        pe = torch.zeros(max_len, d_model)
        pe[:, 0::2] = torch.sin(pos * div)
        pe[:, 1::2] = torch.cos(pos * div)
        self.register_buffer("pe", pe[None])

    def forward(self, x: torch.Tensor, start: int = 0) -> torch.Tensor:
        return x + self.pe[:, start:start + x.shape[1]].to(x.dtype)


class TokenEmbedding(nn.Module):
    def __init__(self, latent_dim: int, d_model: int, vocab_size: Optional[int] = None,
                 max_seq_len: int = 2048, control_dim: int = 4):
        super().__init__()
        self.latent_proj = nn.Linear(latent_dim, d_model)
        self.token_embed = nn.Embedding(vocab_size, d_model) if vocab_size else None
        self.control_proj = nn.Linear(control_dim, d_model)
        self.modality_embed = nn.Embedding(4, d_model)  # rgb, depth, memory, control
        self.pos_embed = PositionalEncoding(d_model, max_seq_len)

    def forward(self, latent_tokens=None, discrete_tokens=None, control_signals=None,
                modality_ids=None, add_pos_embed: bool = True, start_pos: int = 0):
        parts = []
        if latent_tokens is not None:
            parts.append(self.latent_proj(latent_tokens))
        if discrete_tokens is not None:
            parts.append(self.token_embed(discrete_tokens))
        if control_signals is not None:
            parts.append(self.control_proj(control_signals))
        x = parts[0] if len(parts) == 1 else torch.cat(parts, 1)
        if modality_ids is not None:
            x = x + self.modality_embed(modality_ids)
        return self.pos_embed(x, start_pos) if add_pos_embed else x


class MemoryBank(nn.Module):
    """Importance-pruned token memory with attention retrieval (reference :109-212)."""

    def __init__(self, d_model: int, max_memory_size: int = 1024, num_heads: int = 8,
                 memory_decay: float = 0.99):
        super().__init__()
        self.max_memory_size, self.memory_decay = max_memory_size, memory_decay
        self.memory_attn = nn.MultiheadAttention(d_model, num_heads, batch_first=True)
        self.memory_proj = nn.Linear(d_model, d_model)
        self.gate = nn.Linear(2 * d_model, d_model)
        self.register_buffer("memory", torch.zeros(1, 0, d_model), persistent=False)
        self.register_buffer("memory_scores", torch.zeros(1, 0), persistent=False)

    def reset(self):
        d = self.memory.shape[-1]
        self.memory = self.memory.new_zeros(1, 0, d)
        self.memory_scores = self.memory_scores.new_zeros(1, 0)

    @torch.no_grad()
    def update(self, new_tokens: torch.Tensor, importance_scores: Optional[torch.Tensor] = None):
        B, T, D = new_tokens.shape
        if importance_scores is None:
            importance_scores = new_tokens.new_ones(B, T)
        mem, sc = self.memory, self.memory_scores * self.memory_decay
        if mem.shape[0] != B:
            mem = mem.expand(B, -1, -1) if mem.shape[1] else new_tokens.new_zeros(B, 0, D)
            sc = sc.expand(B, -1) if sc.shape[1] else new_tokens.new_zeros(B, 0)
        mem = torch.cat([mem, new_tokens.detach()], 1)
        sc = torch.cat([sc, importance_scores.detach().to(sc.dtype)], 1)
        if mem.shape[1] > self.max_memory_size:
            idx = torch.topk(sc, self.max_memory_size, dim=1).indices.sort(1).values
            mem = torch.gather(mem, 1, idx[..., None].expand(-1, -1, D))
            sc = torch.gather(sc, 1, idx)
        self.memory, self.memory_scores = mem, sc

    def retrieve(self, query: torch.Tensor, top_k: int = 64) -> Optional[torch.Tensor]:
        if self.memory.shape[1] == 0:
            return None
        mem = self.memory
        if mem.shape[0] != query.shape[0]:
            mem = mem[:1].expand(query.shape[0], -1, -1)
        k = min(top_k, mem.shape[1])
        sel = torch.topk(self.memory_scores[:1].expand(query.shape[0], -1), k, dim=1).indices
        mem = torch.gather(mem, 1, sel[..., None].expand(-1, -1, mem.shape[-1]))
        out, _ = self.memory_attn(mem, query, query)
        g = torch.sigmoid(self.gate(torch.cat([out, mem], -1)))
        return self.memory_proj(g * out + (1 - g) * mem)


class DiTStudent(nn.Module):
    def __init__(self, latent_dim: int = 8, d_model: int = 1024, n_layers: int = 24,
                 n_heads: int = 16, d_ff: Optional[int] = None, mlp_type: str = "swiglu",
                 dropout: float = 0.0, max_seq_len: int = 2048, vocab_size: Optional[int] = None,
                 use_rope: bool = True, use_memory: bool = True, memory_size: int = 1024,
                 bias: bool = False, tokens_per_frame: Optional[int] = None):
        super().__init__()
        self.latent_dim, self.d_model, self.n_layers, self.n_heads = latent_dim, d_model, n_layers, n_heads
        self.max_seq_len = max_seq_len
        self.token_embed = TokenEmbedding(latent_dim, d_model, vocab_size, max_seq_len)
        self.blocks = nn.ModuleList([
            DiTBlock(d_model, n_heads, d_ff, mlp_type, dropout, causal=True, use_rope=use_rope,
                     max_seq_len=max_seq_len, bias=bias, tokens_per_frame=tokens_per_frame)
            for _ in range(n_layers)])
        self.norm = RMSNorm(d_model)
        self.lm_head = nn.Linear(d_model, latent_dim, bias=False)
        self.memory_bank = MemoryBank(d_model, memory_size, n_heads) if use_memory else None
        for m in self.modules():
            if isinstance(m, nn.Linear) and m not in (self.blocks,):
                if not any(m is b.attn.qkv or m is b.attn.proj for b in self.blocks):
                    nn.init.normal_(m.weight, std=0.02)
                    if m.bias is not None:
                        nn.init.zeros_(m.bias)

    def forward(self, tokens: torch.Tensor, kv_cache: Optional[List] = None, use_cache: bool = False,
                causal_mask: Optional[torch.Tensor] = None, memory_context: Optional[torch.Tensor] = None,
                return_hidden: bool = False, start_pos: Optional[int] = None):
        past = 0
        if kv_cache is not None and kv_cache[0] is not None:
            past = kv_cache[0]["k"].shape[1]
        pos = past if start_pos is None else start_pos
        x = (self.token_embed(discrete_tokens=tokens, start_pos=pos) if tokens.dim() == 2
             else self.token_embed(latent_tokens=tokens, start_pos=pos))
        mem_len = 0
        if memory_context is not None:
            mem_len = memory_context.shape[1]
            x = torch.cat([memory_context, x], 1)
        if use_cache and kv_cache is None:
            kv_cache = [None] * self.n_layers
        new_cache, hidden = [], []
        for i, blk in enumerate(self.blocks):
            layer_cache = kv_cache[i] if kv_cache is not None else None
            if use_cache and layer_cache is None:
                layer_cache = {}
            x, c = blk(x, kv_cache=layer_cache, causal_mask=causal_mask, start_pos=pos)
            if use_cache:
                new_cache.append(c)
            if return_hidden:
                hidden.append(x)
        x = self.norm(x)[:, mem_len:]
        out = self.lm_head(x)
        res = (out, hidden) if return_hidden else out
        return res, (new_cache if use_cache else None)

    @torch.no_grad()
    def generate(self, context: torch.Tensor, max_new_tokens: int = 100, temperature: float = 1.0,
                 top_k: Optional[int] = None, top_p: Optional[float] = None,
                 use_memory: bool = True, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        seq = context
        cache = None
        if use_memory and self.memory_bank is not None:
            self.memory_bank.update(self.token_embed(latent_tokens=context))
        cur = context
        for _ in range(max_new_tokens):
            out, cache = self.forward(cur, kv_cache=cache, use_cache=True)
            nxt = out[:, -1:]
            if temperature > 0:
                nxt = nxt + temperature * torch.randn(nxt.shape, device=nxt.device, dtype=nxt.dtype,
                                                      generator=generator)
            seq = torch.cat([seq, nxt], 1)
            cur = nxt
        return seq

    def compute_loss(self, input_tokens, target_tokens, mask: Optional[torch.Tensor] = None):
        pred, _ = self.forward(input_tokens)
        err = (pred.float() - target_tokens.float()).pow(2)
        if mask is not None:
            err = err * mask[..., None]
            return err.sum() / (mask.sum() * err.shape[-1]).clamp(min=1)
        return err.mean()


class DiTTeacher(nn.Module):
    """Bidirectional flow-matching teacher: ``forward(z_t, t)`` predicts the velocity."""

    def __init__(self, latent_dim: int = 8, d_model: int = 1024, n_layers: int = 24,
                 n_heads: int = 16, d_ff: Optional[int] = None, mlp_type: str = "swiglu",
                 dropout: float = 0.0, max_seq_len: int = 2048, time_embed_dim: int = 256,
                 use_rope: bool = True, bias: bool = False, num_diffusion_steps: int = 1000,
                 num_steps: int = 4, time_scale: float = 1000.0):
        """The reference's constructor arguments (models/dit_teacher.py:126-140);
        ``time_embed_dim`` is the number of Fourier features of the time embedding,
        ``num_diffusion_steps`` the scale of integer timesteps (``t / steps`` in [0, 1])."""
        super().__init__()
        self.latent_dim, self.num_steps = latent_dim, num_steps
        self.num_diffusion_steps = num_diffusion_steps
        self.input_proj = nn.Linear(latent_dim, d_model)
        self.pos_embed = PositionalEncoding(d_model, max_seq_len)
        self.time_embed = FlowTimestepEmbedding(d_model, time_embed_dim, time_scale=time_scale)
        self.blocks = nn.ModuleList([
            DiTBlock(d_model, n_heads, d_ff, mlp_type, dropout, causal=False, use_rope=use_rope,
                     max_seq_len=max_seq_len, cond_dim=d_model, bias=bias) for _ in range(n_layers)])
        self.norm = RMSNorm(d_model)
        self.out_proj = nn.Linear(d_model, latent_dim)
        nn.init.zeros_(self.out_proj.weight)
        nn.init.zeros_(self.out_proj.bias)

    def forward(self, z_t: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        if t.dim() == 0:
            t = t.expand(z_t.shape[0])
        if not t.is_floating_point():  # integer diffusion timesteps
            t = t.float() / self.num_diffusion_steps
        cond = F.silu(self.time_embed(t))
        x = self.pos_embed(self.input_proj(z_t))
        for blk in self.blocks:
            x, _ = blk(x, cond=cond)
        return self.out_proj(self.norm(x))

    def add_noise(self, x1: torch.Tensor, t: torch.Tensor, noise: Optional[torch.Tensor] = None):
        noise = torch.randn_like(x1) if noise is None else noise
        return interpolate(noise, x1, t), noise

    def compute_loss(self, x1: torch.Tensor, t: Optional[torch.Tensor] = None) -> torch.Tensor:
        t = torch.rand(x1.shape[0], device=x1.device) if t is None else t
        z_t, x0 = self.add_noise(x1, t)
        return F.mse_loss(self.forward(z_t, t).float(), (x1 - x0).float())

    @torch.no_grad()
    def sample(self, shape, num_steps: Optional[int] = None, device=None,
               generator: Optional[torch.Generator] = None) -> torch.Tensor:
        n = num_steps or self.num_steps
        x = torch.randn(shape, device=device, generator=generator)
        ts = torch.linspace(0, 1, n + 1, device=device)
        for i in range(n):
            x = x + (ts[i + 1] - ts[i]) * self.forward(x, ts[i].expand(shape[0]))
        return x

    def distill_to_student(self, student: nn.Module, z_t: torch.Tensor, t: torch.Tensor,
                           dt: float = 0.25) -> torch.Tensor:
        """One-step distillation target: the teacher's Euler step from ``t`` to ``t + dt``;
        returns the student's MSE to the implied velocity."""
        with torch.no_grad():
            v_t = self.forward(z_t, t)
            z_next = z_t + dt * v_t
            target = (z_next - z_t) / dt
        pred = student(z_t, t) if not isinstance(student, DiTStudent) else student(z_t)[0]
        return F.mse_loss(pred.float(), target.float())
