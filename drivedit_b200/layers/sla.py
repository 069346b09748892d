"""Sparse-Linear Attention (SLA): block routing, block-sparse softmax, linear branch.

Two routing/combination semantics are provided:

``mode="topk"`` (default; what the world-model presets and the CUDA kernels use)
    Tokens are cut into ``block_size`` blocks. Block representatives are the mean q and
    k of each block; block scores are ``q̄ · k̄ / sqrt(D)``. Per (batch, head, query
    block), among the key blocks the mask allows (frame-causal at block granularity),
    the ``ceil(topk_frac * n_key_blocks)`` best-scoring ones are *selected* (the
    diagonal block always is). Selected blocks get exact softmax attention, normalised
    jointly over all selected keys. Every other allowed block goes to the linear branch
    ``phi(q) S / (phi(q) . z)`` with ``phi = elu + 1``, ``S = sum phi(k)^T v``,
    ``z = sum phi(k)`` over those blocks. The module returns
    ``proj(o_sparse) + proj_lin(o_linear)`` with ``proj_lin`` zero-initialised, the
    combination of the SLA paper (Zhang et al. 2025, "SLA: Beyond Sparsity in Diffusion
    Transformers via Fine-Tunable Sparse-Linear Attention").

``mode="reference"``
    The reference's semantics (``layers/sla.py:61-357``): importance = softmax-variance
    x score range, global min-max normalised; critical >= 0.5 -> per-block softmax,
    negligible <= 0.01 -> dropped, marginal -> per-block linear attention; output =
    sum of block outputs / sum of block weights (``layers/sla.py:244``). Kept for
    parity with reference checkpoints and tests; it runs in PyTorch only.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import attention_reference


@dataclass
class SLAConfig:
    """The reference's fields in its order (layers/sla.py:23-32; ``flash_attention`` and
    ``linear_feature_dim`` are accepted, the exact branch always runs on this framework's
    attention kernels and the feature map is elu + 1), then this framework's: the
    routing ``mode`` (``topk``: a fixed share of key blocks per query block, or
    ``reference``: the threshold classification), its share and diagonal rule, the
    frame size of frame-causal routing and the linear branch's epsilon."""
    block_size: int = 64
    critical_threshold: float = 0.5  # reference mode
    negligible_threshold: float = 0.01
    causal: bool = False             # token-causal (reference mode) / block-causal
    flash_attention: bool = True
    use_elu_feature: bool = True
    linear_feature_dim: int = 64
    temperature: float = 1.0
    mode: str = "topk"               # "topk" | "reference"
    topk_frac: float = 0.125
    always_diag: bool = True
    tokens_per_frame: Optional[int] = None  # frame-causal when set (topk mode)
    eps: float = 1e-6


def phi(x: torch.Tensor) -> torch.Tensor:
    return F.elu(x) + 1.0


def block_valid_mask(nq: int, nk: int, block: int, tokens_per_frame: Optional[int],
                     causal: bool, device=None, q_offset_blocks: int = 0) -> torch.Tensor:
    """``[nq, nk]`` bool: key block j may be seen by query block i."""
    qi = torch.arange(q_offset_blocks, q_offset_blocks + nq, device=device)[:, None]
    kj = torch.arange(nk, device=device)[None, :]
    if tokens_per_frame:
        bpf = max(tokens_per_frame // block, 1)
        return (kj // bpf) <= (qi // bpf)
    if causal:
        return kj <= qi
    return torch.ones(nq, nk, dtype=torch.bool, device=device)


def n_selected(nk: int, frac: float) -> int:
    return max(1, math.ceil(frac * nk))


def sla_route(q: torch.Tensor, k: torch.Tensor, cfg: SLAConfig,
              q_offset_blocks: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k block routing. ``q [B,T,H,D]``, ``k [B,S,H,D]`` (T, S multiples of the block).

    Returns ``sel [B,H,nq,nk]`` (bool) and ``valid [nq,nk]`` (bool)."""
    B, T, H, D = q.shape
    S = k.shape[1]
    bs = cfg.block_size
    nq, nk = T // bs, S // bs
    qm = q.float().view(B, nq, bs, H, D).mean(2)
    km = k.float().view(B, nk, bs, H, D).mean(2)
    score = torch.einsum("bqhd,bkhd->bhqk", qm, km) / math.sqrt(D)
    valid = block_valid_mask(nq, nk, bs, cfg.tokens_per_frame, cfg.causal, q.device,
                             q_offset_blocks)
    score = score.masked_fill(~valid, float("-inf"))
    kk = min(n_selected(nk, cfg.topk_frac), nk)
    if cfg.always_diag:
        diag = torch.arange(q_offset_blocks, q_offset_blocks + nq, device=q.device).clamp(max=nk - 1)
        score = score.clone()
        score[:, :, torch.arange(nq, device=q.device), diag] = float("inf")
    top = score.topk(kk, dim=-1).indices
    sel = torch.zeros_like(score, dtype=torch.bool).scatter_(-1, top, True)
    return sel & valid, valid


def expand_block_mask(m: torch.Tensor, bs: int) -> torch.Tensor:
    """``[..., nq, nk]`` block mask -> ``[..., nq*bs, nk*bs]`` token mask."""
    return m.repeat_interleave(bs, -2).repeat_interleave(bs, -1)


def sla_sparse_reference(q, k, v, sel: torch.Tensor, block: int, scale=None,
                         return_lse=False):
    """Exact softmax over the keys of the selected blocks (fp32 oracle)."""
    mask = expand_block_mask(sel, block)
    return attention_reference(q, k, v, mask, scale, return_lse)


def sla_linear_reference(q, k, v, lin: torch.Tensor, block: int, eps: float = 1e-6,
                         temperature: float = 1.0):
    """Linear branch over the blocks in ``lin [B,H,nq,nk]`` (fp32 oracle).

    ``o_i = phi(q_i) S_i / (phi(q_i) . z_i + eps)`` with ``S_i = sum_j lin_ij phi(K_j)^T V_j``.
    """
    B, T, H, D = q.shape
    S = k.shape[1]
    nq, nk = T // block, S // block
    fq = phi(q.float() / temperature).view(B, nq, block, H, D)
    fk = phi(k.float() / temperature).view(B, nk, block, H, D)
    vv = v.float().view(B, nk, block, H, D)
    kv = torch.einsum("bjshd,bjshe->bhjde", fk, vv)          # [B,H,nk,D,D]
    z = fk.sum(2).permute(0, 2, 1, 3)                          # [B,H,nk,D]
    w = lin.float()
    st = torch.einsum("bhij,bhjde->bhide", w, kv)             # [B,H,nq,D,D]
    zt = torch.einsum("bhij,bhjd->bhid", w, z)                 # [B,H,nq,D]
    num = torch.einsum("bishd,bhide->bishe", fq, st)
    den = torch.einsum("bishd,bhid->bish", fq, zt)
    o = num / (den[..., None] + eps)
    return o.reshape(B, T, H, D)


def sla_topk_reference(q, k, v, cfg: SLAConfig, q_offset_blocks: int = 0):
    """(o_sparse, o_linear, sel) for the top-k mode, all fp32."""
    sel, valid = sla_route(q, k, cfg, q_offset_blocks)
    o_s = sla_sparse_reference(q, k, v, sel, cfg.block_size)
    lin = valid[None, None] & ~sel
    o_l = sla_linear_reference(q, k, v, lin, cfg.block_size, cfg.eps, cfg.temperature)
    return o_s, o_l, sel


# ----------------------------------------------------------------- reference semantics
def classify_blocks_reference(q, k, cfg: SLAConfig):
    """The reference's block classification (layers/sla.py:61-137)."""
    B, T, H, D = q.shape
    S = k.shape[1]
    bs = cfg.block_size
    nq, nk = -(-T // bs), -(-S // bs)
    qp = F.pad(q, (0, 0, 0, 0, 0, nq * bs - T)).float()
    kp = F.pad(k, (0, 0, 0, 0, 0, nk * bs - S)).float()
    qm = qp.view(B, nq, bs, H, D).mean(2)
    km = kp.view(B, nk, bs, H, D).mean(2)
    sc = torch.einsum("bqhd,bkhd->bhqk", qm, km) / math.sqrt(D)
    tri = torch.tril(torch.ones(nq, nk, dtype=torch.bool, device=q.device))
    if cfg.causal:
        sc = sc.masked_fill(~tri, -1e9)
    var = F.softmax(sc, -1).var(-1, keepdim=True)
    imp = var.expand_as(sc) * (sc.max(-1, keepdim=True).values - sc.min()).clamp(min=1e-6)
    imp = (imp - imp.min()) / (imp.max() - imp.min() + 1e-6)
    crit = imp >= cfg.critical_threshold
    negl = imp <= cfg.negligible_threshold
    marg = ~crit & ~negl
    if cfg.causal:
        crit, marg, negl = crit & tri, marg & tri, negl | ~tri
    return crit, marg, negl


def classify_blocks(q, k, config: SLAConfig, mask: Optional[torch.Tensor] = None):
    """The reference's name and signature for :func:`classify_blocks_reference`
    (its ``mask`` argument is accepted and, as there, unused)."""
    return classify_blocks_reference(q, k, config)


@dataclass
class SLAStats:
    """Block counts of one classification (layers/sla.py:36-43): ``critical_ratio`` =
    critical / total, ``compute_savings`` = 1 - (critical + marginal / block_size) /
    total, the share of exact-softmax work a classification avoids when a marginal block
    costs 1/block_size of a critical one (linear attention against quadratic)."""
    critical_blocks: int
    marginal_blocks: int
    negligible_blocks: int
    total_blocks: int
    critical_ratio: float
    compute_savings: float

    @classmethod
    def from_masks(cls, critical: torch.Tensor, marginal: torch.Tensor, negligible: torch.Tensor,
                   block_size: int = 64) -> "SLAStats":
        c, m, n = int(critical.sum()), int(marginal.sum()), int(negligible.sum())
        tot = max(c + m + n, 1)
        return cls(c, m, n, c + m + n, c / tot, 1.0 - (c + m / block_size) / tot)


def sla_reference(q, k, v, cfg: SLAConfig) -> torch.Tensor:
    """The reference's SLA output (layers/sla.py:140-247), vectorised over block pairs."""
    B, T, H, D = q.shape
    S = k.shape[1]
    bs = cfg.block_size
    if T <= bs or S <= bs:
        mask = torch.tril(torch.ones(T, S, dtype=torch.bool, device=q.device)) if cfg.causal else None
        return attention_reference(q, k, v, mask, 1.0 / (math.sqrt(D) * cfg.temperature)).to(q.dtype)
    crit, marg, _ = classify_blocks_reference(q, k, cfg)
    nq, nk = crit.shape[-2:]
    qp = F.pad(q, (0, 0, 0, 0, 0, nq * bs - T)).float().view(B, nq, bs, H, D)
    kp = F.pad(k, (0, 0, 0, 0, 0, nk * bs - S)).float().view(B, nk, bs, H, D)
    vp = F.pad(v, (0, 0, 0, 0, 0, nk * bs - S)).float().view(B, nk, bs, H, D)
    scale = 1.0 / (math.sqrt(D) * cfg.temperature)
    out = torch.zeros(B, nq, bs, H, D, device=q.device)
    wsum = torch.zeros(B, nq, bs, H, 1, device=q.device)
    tri_tok = torch.tril(torch.ones(bs, bs, dtype=torch.bool, device=q.device))
    fk_all = phi(kp / cfg.temperature)
    for i in range(nq):
        s = torch.einsum("bthd,bjshd->bhjts", qp[:, i], kp) * scale     # [B,H,nk,bs,bs]
        if cfg.causal:
            blk = torch.arange(nk, device=q.device)
            s = s.masked_fill((blk > i)[None, None, :, None, None], -1e9)
            s[:, :, i] = s[:, :, i].masked_fill(~tri_tok, -1e9)
        p = F.softmax(s, -1)
        oc = torch.einsum("bhjts,bjshd->bjthd", p, vp)                  # [B,nk,bs,H,D]
        wc = p.sum(-1).permute(0, 2, 3, 1)[..., None]                   # [B,nk,bs,H,1]
        fq = phi(qp[:, i] / cfg.temperature)                            # [B,bs,H,D]
        kv = torch.einsum("bjshd,bjshe->bjhde", fk_all, vp)
        num = torch.einsum("bthd,bjhde->bjthe", fq, kv)
        den = torch.einsum("bthd,bjhd->bjth", fq, fk_all.sum(2)) + 1e-6
        ol = num / den[..., None]
        wl = den[..., None]
        c = crit[:, :, i].permute(0, 2, 1)[:, :, None, :, None].float()  # [B,nk,1,H,1]
        m = marg[:, :, i].permute(0, 2, 1)[:, :, None, :, None].float()
        out[:, i] = (oc * c + ol * m).sum(1)
        wsum[:, i] = (wc * c + wl * m).sum(1)
    out = out / (wsum + 1e-6)
    return out.view(B, nq * bs, H, D)[:, :T].to(q.dtype)


class SparseLinearAttention(nn.Module):
    """Drop-in self-attention module with SLA (reference state-dict names ``qkv``/``proj``
    plus ``proj_lin`` for the linear branch in top-k mode)."""

    def __init__(self, d_model: int, n_heads: int, config: Optional[SLAConfig] = None,
                 dropout: float = 0.0, bias: bool = False, rope_layer=None):
        super().__init__()
        self.d_model, self.n_heads = d_model, n_heads
        self.d_head = d_model // n_heads
        self.config = config or SLAConfig()
        self.rope_layer = rope_layer
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=bias)
        self.proj = nn.Linear(d_model, d_model, bias=bias)
        self.proj_lin = nn.Linear(d_model, d_model, bias=False)
        nn.init.normal_(self.qkv.weight, std=0.02)
        nn.init.normal_(self.proj.weight, std=0.02 / math.sqrt(2 * 12))
        nn.init.zeros_(self.proj_lin.weight)

    def forward(self, x, kv_cache=None, mask=None, start_pos: int = 0):
        B, T, D = x.shape
        q, k, v = self.qkv(x).view(B, T, 3, self.n_heads, self.d_head).unbind(2)
        if self.rope_layer is not None:
            q, k = self.rope_layer(q, start_pos), self.rope_layer(k, start_pos)
        new_cache = None
        if isinstance(kv_cache, dict):
            if kv_cache.get("k") is not None:
                k = torch.cat([kv_cache["k"], k], 1)
                v = torch.cat([kv_cache["v"], v], 1)
            new_cache = {"k": k.detach(), "v": v.detach()}
        cfg = self.config
        if cfg.mode == "reference":
            o = sla_reference(q, k, v, cfg)
            return self.proj(o.reshape(B, T, D)), new_cache
        bs = cfg.block_size
        if T % bs or k.shape[1] % bs:
            raise ValueError("top-k SLA needs sequence lengths that are multiples of the block")
        o_s, o_l, _ = sla_topk_reference(q, k, v, cfg,
                                         q_offset_blocks=(k.shape[1] - T) // bs)
        out = self.proj(o_s.to(x.dtype).reshape(B, T, D)) + self.proj_lin(
            o_l.to(x.dtype).reshape(B, T, D))
        return out, new_cache


class CausalSparseLinearAttention(SparseLinearAttention):
    def __init__(self, d_model, n_heads, config: Optional[SLAConfig] = None, **kw):
        config = config or SLAConfig()
        config.causal = True
        super().__init__(d_model, n_heads, config, **kw)


def create_sla_layer(d_model: int, n_heads: int, causal: bool = False, block_size: int = 64,
                     **kw) -> SparseLinearAttention:
    cfg = SLAConfig(block_size=block_size, causal=causal)
    cls = CausalSparseLinearAttention if causal else SparseLinearAttention
    return cls(d_model, n_heads, cfg, **kw)
