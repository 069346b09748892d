"""Action-conditioned latent-video flow-matching DiT (the flagship world model).

Built from the reference's pieces, with the semantics decisions spelled out:
  * tokens: latent frames ``[B, F, C, H, W]`` cut into ``p x p`` patches
    (``C*p*p``-dim), projected by ``patch_embed``; ``unpatchify`` inverts it. (The
    reference's ``WorldModel`` patches RGB at 16x16, models/world_model.py:113-134;
    ``DiTStudent`` projects whole latent vectors, models/dit_student.py:42.)
  * conditioning: per-frame ``c = silu(t_embed(t) + action_embed(a_f))`` where
    ``t_embed`` is the reference's ``TimestepEmbedding`` (blocks/flow_matching.py:62-91,
    256 Fourier features -> MLP; ``t`` is scaled by ``time_scale`` first) and the
    action MLP maps each frame's action vector.
  * blocks: the reference's ``DiTBlock`` (blocks/dit_block.py:21-140): pre-norm
    AdaLN(RMSNorm) -> attention -> residual, AdaLN -> SwiGLU -> residual; the AdaLN
    scale/shift come per frame from ``c`` (one ``ada`` projection per block), optional
    adaLN-Zero gates (blocks/flow_matching.py:131-144).
  * attention: 3-D RoPE with an explicit (16, 24, 24) channel split for d_head = 64,
    frame-causal masking (every token of frame f sees frames <= f) or token-causal /
    bidirectional, dense softmax or SLA (:mod:`drivedit_b200.layers.sla`).
  * FFN: dense SwiGLU (gate/value rows interleaved by 32 for the fused epilogue) or the
    DeepSeek MoE (:mod:`drivedit_b200.layers.moe`).
  * head: AdaLN final norm + zero-initialised linear to patch space.

On CUDA the blocks run through the fused sm_100a path (:mod:`drivedit_b200.ops.block`);
on CPU the same math runs in PyTorch (the numerical oracle and the CPU baseline).
"""
from __future__ import annotations

import math
import re
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from ..layers.attention import attention_reference, frame_causal_mask
from ..layers.mlp import split_gu
from ..layers.moe import MoEFFN
from ..layers.rope import RoPE3D, apply_rope
from ..layers.sla import SLAConfig, sla_topk_reference


def patchify(x: torch.Tensor, p: int) -> torch.Tensor:
    """``[B, F, C, H, W]`` -> ``[B, F*(H/p)*(W/p), C*p*p]`` (channel-major patch vectors)."""
    B, Fr, C, H, W = x.shape
    x = x.reshape(B, Fr, C, H // p, p, W // p, p)
    x = x.permute(0, 1, 3, 5, 2, 4, 6)
    return x.reshape(B, Fr * (H // p) * (W // p), C * p * p)


def unpatchify(t: torch.Tensor, frames: int, C: int, H: int, W: int, p: int) -> torch.Tensor:
    B = t.shape[0]
    t = t.reshape(B, frames, H // p, W // p, C, p, p)
    t = t.permute(0, 1, 4, 2, 5, 3, 6)
    return t.reshape(B, frames, C, H, W)


class TimestepEmbedding(nn.Module):
    """Sinusoidal features of ``t * time_scale`` -> Linear -> SiLU -> Linear
    (reference names ``linear1`` / ``linear2``)."""

    def __init__(self, dim: int, fourier_features: int = 256, time_scale: float = 1000.0):
        super().__init__()
        self.fourier_features = fourier_features
        self.time_scale = time_scale
        self.linear1 = nn.Linear(fourier_features, dim)
        self.linear2 = nn.Linear(dim, dim)

    def features(self, t: torch.Tensor) -> torch.Tensor:
        half = self.fourier_features // 2
        freq = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32)
                         / (half - 1))
        ang = t.float()[..., None] * self.time_scale * freq
        return torch.cat([ang.sin(), ang.cos()], -1)

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        return self.linear2(F.silu(self.linear1(self.features(t))))


class ActionEmbedding(nn.Module):
    def __init__(self, action_dim: int, dim: int):
        super().__init__()
        self.linear1 = nn.Linear(action_dim, dim)
        self.linear2 = nn.Linear(dim, dim)

    def forward(self, a: torch.Tensor) -> torch.Tensor:
        return self.linear2(F.silu(self.linear1(a)))


class _Lin(nn.Module):
    """Bias-free weight holder with the reference's ``<name>.weight`` key."""

    def __init__(self, out_f: int, in_f: int, std: float = 0.02):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(out_f, in_f) * std)


class _Norm(nn.Module):
    def __init__(self, d: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))


class WorldDiTBlock(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_idx: int):
        super().__init__()
        d, F_ = cfg.d_model, cfg.mlp_hidden
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.n_mod = 6 if cfg.adaln_zero else 4
        self.norm1 = _Norm(d)
        self.norm2 = _Norm(d)
        self.attn = nn.Module()
        self.attn.qkv = _Lin(3 * d, d, 0.02)
        self.attn.proj = _Lin(d, d, 0.02 / math.sqrt(2 * cfg.n_layers))
        if cfg.attention == "sla":
            self.attn.proj_lin = _Lin(d, d, 0.0)
        if cfg.moe is None:
            self.mlp = nn.Module()
            # gate/value rows interleaved by 32 (see layers/mlp.py: pack_swiglu)
            self.mlp.w13 = _Lin(2 * F_, d, 0.02)
            self.mlp.w3 = _Lin(d, F_, 0.02 / math.sqrt(2 * cfg.n_layers))
            self.moe = None
        else:
            m = cfg.moe
            self.moe = MoEFFN(d, m.num_experts, m.top_k, m.expert_dim, m.num_shared,
                              bias_update_speed=m.bias_update_speed,
                              aux_loss_weight=m.aux_loss_weight)
        # per-frame modulation: (scale1, shift1, scale2, shift2[, gate1, gate2])
        self.ada = nn.Linear(d, self.n_mod * d)
        nn.init.zeros_(self.ada.weight)
        nn.init.zeros_(self.ada.bias)

    # ---------------------------------------------------------------- torch path
    def forward_torch(self, x: torch.Tensor, mod: torch.Tensor, rope_tab: torch.Tensor,
                      frames: int) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        """``x [B, T, d]``, ``mod [B, F, n_mod*d]``; returns (x, aux_loss)."""
        cfg = self.cfg
        B, T, d = x.shape
        H, Dh = cfg.n_heads, cfg.d_head
        tpf = T // frames
        m = mod.repeat_interleave(tpf, dim=1)
        chunks = m.chunk(self.n_mod, -1)
        s1, b1, s2, b2 = chunks[:4]
        dt = x.dtype

        def norm(v, w):
            vf = v.float()
            return (vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + cfg.norm_eps)).to(dt) * w.to(dt)

        h = norm(x, self.norm1.weight) * (1 + s1) + b1
        qkv = (h @ self.attn.qkv.weight.to(dt).t()).view(B, T, 3, H, Dh)
        q, k, v = qkv.unbind(2)
        q, k = apply_rope(q, rope_tab), apply_rope(k, rope_tab)
        if cfg.attention == "sla":
            scfg = SLAConfig(block_size=cfg.sla.block_size, topk_frac=cfg.sla.topk_frac,
                             always_diag=cfg.sla.always_diag,
                             tokens_per_frame=tpf if cfg.causal == "frame" else None,
                             causal=cfg.causal == "token")
            o_s, o_l, _ = sla_topk_reference(q, k, v, scfg)
            a = o_s.to(dt).reshape(B, T, d) @ self.attn.proj.weight.to(dt).t() + \
                o_l.to(dt).reshape(B, T, d) @ self.attn.proj_lin.weight.to(dt).t()
        else:
            if cfg.causal == "frame":
                mask = frame_causal_mask(T, tpf, device=x.device)
            elif cfg.causal == "token":
                mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=x.device))[None, None]
            else:
                mask = None
            if x.dtype == torch.float32:
                o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                   v.transpose(1, 2), attn_mask=mask).transpose(1, 2)
            else:
                o = attention_reference(q, k, v, mask).to(dt)
            a = o.reshape(B, T, d) @ self.attn.proj.weight.to(dt).t()
        if self.n_mod == 6:
            a = a * chunks[4]
        x = x + a
        h2 = norm(x, self.norm2.weight) * (1 + s2) + b2
        aux = None
        if self.moe is None:
            gu = h2 @ self.mlp.w13.weight.to(dt).t()
            g, u = split_gu(gu)
            f = (F.silu(g) * u) @ self.mlp.w3.weight.to(dt).t()
        else:
            out = self.moe(h2)
            f, aux = out.output, out.aux_loss
        if self.n_mod == 6:
            f = f * chunks[5]
        return x + f, aux


class WorldDiT(nn.Module):
    """Flow-matching latent-video DiT: predicts the velocity ``x1 - x0`` of ``x_t``."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        d = cfg.d_model
        self.patch_embed = nn.Linear(cfg.patch_dim, d)
        self.t_embed = TimestepEmbedding(d, 256, cfg.time_scale)
        self.a_embed = ActionEmbedding(cfg.action_dim, d)
        self.blocks = nn.ModuleList([WorldDiTBlock(cfg, i) for i in range(cfg.n_layers)])
        self.final_norm = _Norm(d)
        self.final_ada = nn.Linear(d, 2 * d)
        nn.init.zeros_(self.final_ada.weight)
        nn.init.zeros_(self.final_ada.bias)
        self.out_proj = nn.Linear(d, cfg.patch_dim)
        nn.init.zeros_(self.out_proj.weight)
        nn.init.zeros_(self.out_proj.bias)
        self.rope = RoPE3D(cfg.d_head, cfg.grid_h, cfg.grid_w, cfg.max_frames, cfg.rope_base,
                           cfg.rope_temporal_factor, cfg.rope_split)
        self.repa_head = None
        if cfg.repa is not None:
            # REPA projection of the layer-`cfg.repa.layer` hidden states onto the frozen
            # teacher's feature space; trained with the model (same optimizer / shards)
            from ..training.repa import ProjectionMLP

            rp = cfg.repa
            hid = rp.proj_hidden or (d + rp.teacher_dim) // 2
            self.repa_head = ProjectionMLP(d, hid, rp.teacher_dim)
        self.fused = None  # set by enable_fused() on CUDA

    # ---------------------------------------------------------------- helpers
    def condition(self, t: torch.Tensor, actions: torch.Tensor,
                  extra: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Per-frame conditioning ``[B, F, d]`` from ``t [B]`` or ``[B, F]`` and actions;
        ``extra`` (``[B, d]`` or ``[B, F, d]``, e.g. control / future-anchor embeddings)
        is added before the activation."""
        te = self.t_embed(t)
        if te.dim() == 2:
            te = te[:, None]
        h = te + self.a_embed(actions.float())
        if extra is not None:
            h = h + (extra[:, None] if extra.dim() == 2 else extra).float()
        return F.silu(h)

    def no_decay_names(self) -> List[str]:
        return [n for n, p in self.named_parameters()
                if p.dim() < 2 or n.endswith(".bias") or "norm" in n.split(".")[-2]]

    MOD_PARAM = re.compile(r"^(blocks\.\d+\.ada|final_ada)\.(weight|bias)$")

    def flat_layout(self, named):
        """Parameter order for flat buffers: every block's AdaLN modulation projection
        and the final one, weights and biases each as one contiguous run (block order,
        then final), so the fused path computes all modulations with one GEMM."""
        named = list(named)
        mods = [(n, p) for n, p in named if self.MOD_PARAM.match(n)]
        rest = [(n, p) for n, p in named if not self.MOD_PARAM.match(n)]
        key = lambda np_: (np_[0].endswith(".bias"), np_[0].startswith("final"),
                           int(np_[0].split(".")[1]) if np_[0].startswith("blocks") else 0)
        return rest + sorted(mods, key=key)

    # ---------------------------------------------------------------- forward
    def forward(self, x_t: torch.Tensor, t: torch.Tensor, actions: torch.Tensor,
                frame_offset: int = 0, return_aux: bool = False, return_features: Optional[int] = None,
                extra_cond: Optional[torch.Tensor] = None):
        """``x_t [B, F, C, H, W]``, ``t [B]`` / ``[B, F]``, ``actions [B, F, A]``,
        optional ``extra_cond`` added to the per-frame conditioning."""
        cfg = self.cfg
        B, Fr, C, H, W = x_t.shape
        if self.fused is not None and x_t.is_cuda:
            return self.fused.forward(self, x_t, t, actions, frame_offset, return_aux,
                                      return_features, extra_cond)
        dt = x_t.dtype
        tok = patchify(x_t, cfg.patch)
        x = self.patch_embed(tok.to(self.patch_embed.weight.dtype)).to(dt)
        c = self.condition(t, actions, extra_cond)           # [B, F, d] fp32
        tab = self.rope.table(Fr, frame_offset).to(x.device)
        aux_total = x.new_zeros((), dtype=torch.float32)
        feats = None
        for i, blk in enumerate(self.blocks):
            mod = blk.ada(c).to(dt)
            x, aux = blk.forward_torch(x, mod, tab, Fr)
            if aux is not None:
                aux_total = aux_total + aux
            if return_features is not None and i + 1 == return_features:
                feats = x
        fm = self.final_ada(c).to(dt).repeat_interleave(x.shape[1] // Fr, 1)
        sc, sh = fm.chunk(2, -1)
        xf = x.float()
        hn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.norm_eps)).to(dt) * \
            self.final_norm.weight.to(dt)
        out = self.out_proj((hn * (1 + sc) + sh).to(self.out_proj.weight.dtype))
        v = unpatchify(out.to(dt), Fr, C, H, W, cfg.patch)
        if return_features is not None:
            return v, aux_total, feats
        return (v, aux_total) if return_aux else v

    def enable_expert_parallel(self, ep) -> List[str]:
        """Shard every MoE layer's routed experts over the EP group ``ep``
        (:class:`~drivedit_b200.parallel.expert.ExpertParallel`); returns the names of the
        now rank-local parameters. Call before any flat parameter group is built."""
        for blk in self.blocks:
            if blk.moe is not None:
                blk.moe.shard_experts(ep)
        return self.expert_parameter_names()

    def expert_parameter_names(self) -> List[str]:
        return [n for i, blk in enumerate(self.blocks) if blk.moe is not None
                for n in blk.moe.expert_parameter_names(f"blocks.{i}.moe.")]

    def enable_fused(self, **kw):
        from ..ops.block import FusedWorldDiT

        self.fused = FusedWorldDiT(self, **kw)
        return self.fused


# ----------------------------------------------------------------------------- KV-cached
class LayerKVCache:
    """Per-layer key/value window for streaming generation.

    ``k``/``v`` are ``[B, capacity, d]`` buffers holding consecutive tokens; ``start`` is
    the buffer row of the first token inside the attention window, ``end`` one past the
    last written token and ``pos0`` the absolute token position of buffer row 0. When a
    new chunk would not fit, the last ``window`` tokens are moved to the front (amortised:
    once every ``window / chunk`` chunks)."""

    def __init__(self, B: int, capacity: int, d: int, window: int, device, dtype):
        self.k = torch.zeros(B, capacity, d, device=device, dtype=dtype)
        self.v = torch.zeros(B, capacity, d, device=device, dtype=dtype)
        self.capacity, self.window = capacity, window
        self.start = self.end = 0
        self.pos0 = 0

    def reserve(self, n: int) -> int:
        """Make room for ``n`` new tokens after the window; returns their buffer row."""
        keep_from = max(self.start, self.end - self.window)
        if self.end + n > self.capacity:
            keep = self.end - keep_from
            self.k[:, :keep] = self.k[:, keep_from:self.end].clone()
            self.v[:, :keep] = self.v[:, keep_from:self.end].clone()
            self.pos0 += keep_from
            self.end = keep
            keep_from = 0
        self.start = keep_from
        return self.end

    def commit(self, n: int):
        self.end += n


class KVCacheSet:
    """One :class:`LayerKVCache` per block; ``frames`` counts committed frames."""

    def __init__(self, model: "WorldDiT", B: int, window_frames: int, chunk_frames: int,
                 device, dtype):
        cfg = model.cfg
        tpf = cfg.tokens_per_frame
        cap = (2 * window_frames + chunk_frames) * tpf
        self.layers = [LayerKVCache(B, cap, cfg.d_model, window_frames * tpf, device, dtype)
                       for _ in model.blocks]
        self.frames = 0
        self.tpf = tpf

    def reserve(self, n_tokens: int) -> int:
        rows = [c.reserve(n_tokens) for c in self.layers]
        return rows[0]

    def commit(self, n_frames: int):
        for c in self.layers:
            c.commit(n_frames * self.tpf)
        self.frames += n_frames


def _block_cached_torch(blk: WorldDiTBlock, x, mod, tab_q, cache: LayerKVCache, row, frames):
    """One block over a chunk ``x [B, T, d]`` attending to the cache window + itself;
    writes the chunk's K/V into the cache rows ``[row, row + T)``."""
    cfg = blk.cfg
    B, T, d = x.shape
    H, Dh = cfg.n_heads, cfg.d_head
    dt = x.dtype
    tpf = T // frames
    m = mod.repeat_interleave(tpf, dim=1)
    s1, b1, s2, b2 = m.chunk(blk.n_mod, -1)[:4]

    def norm(v, w):
        vf = v.float()
        return (vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + cfg.norm_eps)).to(dt) * w.to(dt)

    h = norm(x, blk.norm1.weight) * (1 + s1) + b1
    qkv = (h @ blk.attn.qkv.weight.to(dt).t()).view(B, T, 3, H, Dh)
    q, k, v = qkv.unbind(2)
    q, k = apply_rope(q, tab_q), apply_rope(k, tab_q)
    cache.k[:, row:row + T] = k.reshape(B, T, d)
    cache.v[:, row:row + T] = v.reshape(B, T, d)
    kk = cache.k[:, cache.start:row + T].view(B, -1, H, Dh)
    vv = cache.v[:, cache.start:row + T].view(B, -1, H, Dh)
    S = kk.shape[1]
    mask = frame_causal_mask(T, tpf, S, x.device)
    o = attention_reference(q, kk, vv, mask).to(dt)
    x = x + o.reshape(B, T, d) @ blk.attn.proj.weight.to(dt).t()
    h2 = norm(x, blk.norm2.weight) * (1 + s2) + b2
    gu = h2 @ blk.mlp.w13.weight.to(dt).t()
    g, u = split_gu(gu)
    return x + (F.silu(g) * u) @ blk.mlp.w3.weight.to(dt).t()


@torch.no_grad()
def forward_cached(model: "WorldDiT", x_t: torch.Tensor, t: torch.Tensor, actions: torch.Tensor,
                   cache: KVCacheSet, commit: bool = False,
                   extra_cond: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Velocity for a chunk of frames ``x_t [B, Fc, C, H, W]`` at absolute frame
    ``cache.frames``, attending to the cached window. With ``commit`` the chunk's K/V stay
    in the cache (call this on the clean chunk after sampling it)."""
    if model.fused is not None and x_t.is_cuda:
        return model.fused.forward_cached(model, x_t, t, actions, cache, commit, extra_cond)
    cfg = model.cfg
    B, Fc, C, H, W = x_t.shape
    dt = x_t.dtype
    tok = patchify(x_t, cfg.patch)
    x = model.patch_embed(tok.to(model.patch_embed.weight.dtype)).to(dt)
    c = model.condition(t, actions, extra_cond)
    T = x.shape[1]
    tab = model.rope.table(Fc, cache.frames).to(x.device)
    row = cache.reserve(T)
    for blk, lc in zip(model.blocks, cache.layers):
        mod = blk.ada(c).to(dt)
        x = _block_cached_torch(blk, x, mod, tab, lc, row, Fc)
    if commit:
        cache.commit(Fc)
    fm = model.final_ada(c).to(dt).repeat_interleave(T // Fc, 1)
    sc, sh = fm.chunk(2, -1)
    xf = x.float()
    hn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.norm_eps)).to(dt) * \
        model.final_norm.weight.to(dt)
    out = model.out_proj((hn * (1 + sc) + sh).to(model.out_proj.weight.dtype))
    return unpatchify(out.to(dt), Fc, C, H, W, cfg.patch)
