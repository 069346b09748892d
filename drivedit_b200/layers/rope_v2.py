"""RoPE v2 class surface: configuration, frequency cache and the multi-mode RoPE layer.

Parity with the reference's ``layers/rope_v2.py``: ``RoPEConfig`` (:29-88),
``rope_apply_qk`` (:151-174), ``compute_rope_3d_freqs`` (:405-501),
``apply_rope_3d_efficient`` (:504-571), ``interpolate_rope_freqs`` (:578-620),
``compute_resolution_aware_rope_freqs`` (:623-682), ``RoPEFrequencyCache`` (:689-865),
``RoPELayerV2`` with ``forward`` / ``forward_qk`` / ``forward_3d`` / ``forward_flash`` /
``forward_chunked`` (:872-1249) and the compat helpers ``precompute_rope_freqs``,
``precompute_rope_3d_freqs``, ``rope`` (:1292-1332).

Everything here is built on the angle functions of :mod:`.rope` (float64 angles, one
code path for plain / NTK / dynamic-NTK / YaRN frequencies). Differences from the
reference, by design:

* 3-D factorisation takes an explicit (t, h, w) channel split. With ``dim % 6 == 0``
  the split is equal thirds (the reference's rule); any other even ``dim`` (d_head = 64,
  which every latent world-model preset uses) gets :func:`.rope.default_split`.
* Packed sequences (``forward_flash`` with ``cu_seqlens``) compute every token's
  position with one vectorised expression instead of a per-sequence Python loop.
* The fused GEMM path of this framework does not use this module: it rotates q/k in the
  QKV GEMM epilogue with the in-place pair layout (:class:`.rope.RoPE3D` tables). These
  classes serve reference-compatible model code and user code.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Literal, Optional, Sequence, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .rope import (compute_dynamic_ntk_rope_freqs, compute_ntk_rope_freqs, compute_rope_freqs,
                   default_split, inv_freqs, rope_apply, yarn_inv_freqs)

SinCos = Tuple[torch.Tensor, torch.Tensor]


@dataclass
class RoPEConfig:
    """Field names and defaults follow the reference config so saved configs load."""
    dim: int = 64
    max_seq_len: int = 2048
    base: float = 10000.0
    # NTK-aware scaling
    ntk_alpha: float = 1.0
    dynamic_ntk: bool = False
    ntk_factor: float = 1.0
    original_max_seq_len: int = 2048
    # YaRN
    yarn_enabled: bool = False
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0
    yarn_mscale: float = 1.0
    yarn_mscale_all_dim: float = 0.0
    # 3-D factorisation
    spatial_dims: Optional[Tuple[int, int]] = None
    temporal_base_factor: float = 1.0
    # variable resolution
    interpolate_factor: float = 1.0
    # storage
    use_half_precision: bool = True
    cache_common_lengths: Tuple[int, ...] = (64, 128, 256, 512, 1024, 2048)


# --------------------------------------------------------------------------- functions
def rope_apply_qk(q: torch.Tensor, k: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor,
                  interleaved: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """The same rotation applied to q and k."""
    return rope_apply(q, sin, cos, interleaved), rope_apply(k, sin, cos, interleaved)


def axis_split(dim: int) -> Tuple[int, int, int]:
    """(t, h, w) channel counts: equal thirds when ``dim % 6 == 0``, else the default
    split for this framework's head sizes."""
    if dim % 6 == 0:
        return dim // 3, dim // 3, dim // 3
    return default_split(dim)


def _axis_freqs(n: int, channels: int, base: float, device, dtype, scale: float = 1.0) -> SinCos:
    ang = torch.outer(torch.arange(n, dtype=torch.float64, device=device) * scale,
                      inv_freqs(channels, base, device))
    return ang.sin().to(dtype), ang.cos().to(dtype)


def compute_rope_3d_freqs(dim: int, max_time: int, max_height: int, max_width: int,
                          base: float = 10000.0, temporal_base_factor: float = 1.0,
                          device=None, dtype: torch.dtype = torch.float32,
                          efficient_mode: bool = True,
                          split: Optional[Sequence[int]] = None
                          ) -> Union[SinCos, Tuple[SinCos, SinCos, SinCos]]:
    """Factorised (time, height, width) frequencies. ``efficient_mode``: the three 1-D
    tables ``((sin_t, cos_t), (sin_h, cos_h), (sin_w, cos_w))``, each ``[n_axis,
    channels_axis / 2]``; otherwise the full grid ``(sin, cos)`` of shape
    ``[max_time, max_height, max_width, dim / 2]``. The time axis uses the base
    ``base * temporal_base_factor``."""
    st, sh, sw = split if split is not None else axis_split(dim)
    if st + sh + sw != dim or min(st, sh, sw) % 2:
        raise ValueError(f"3-D RoPE split {(st, sh, sw)} must be even and sum to {dim}")
    ft = _axis_freqs(max_time, st, base * temporal_base_factor, device, dtype)
    fh = _axis_freqs(max_height, sh, base, device, dtype)
    fw = _axis_freqs(max_width, sw, base, device, dtype)
    if efficient_mode:
        return ft, fh, fw
    shape = (max_time, max_height, max_width)
    sin = torch.cat([ft[0][:, None, None, :].expand(*shape, -1),
                     fh[0][None, :, None, :].expand(*shape, -1),
                     fw[0][None, None, :, :].expand(*shape, -1)], -1)
    cos = torch.cat([ft[1][:, None, None, :].expand(*shape, -1),
                     fh[1][None, :, None, :].expand(*shape, -1),
                     fw[1][None, None, :, :].expand(*shape, -1)], -1)
    return sin, cos


def apply_rope_3d_efficient(x: torch.Tensor, freqs_t: SinCos, freqs_h: SinCos, freqs_w: SinCos,
                            t_indices: Optional[torch.Tensor] = None,
                            h_indices: Optional[torch.Tensor] = None,
                            w_indices: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotate the (t, h, w) channel groups of ``x [..., seq, heads, dim]`` with their
    own 1-D tables, gathered at per-token indices (default: the table rows in order).
    Each group's width is twice its table's last dimension."""
    groups = []
    c0 = 0
    for (sin, cos), idx in ((freqs_t, t_indices), (freqs_h, h_indices), (freqs_w, w_indices)):
        width = 2 * sin.shape[-1]
        if idx is not None:
            sin, cos = sin[idx], cos[idx]
        # broadcast over the heads axis (and any batch axes the indices lack)
        sin, cos = sin.unsqueeze(-2), cos.unsqueeze(-2)
        groups.append(rope_apply(x[..., c0:c0 + width], sin.to(x.dtype), cos.to(x.dtype)))
        c0 += width
    if c0 != x.shape[-1]:
        raise ValueError(f"tables cover {c0} channels, x has {x.shape[-1]}")
    return torch.cat(groups, dim=-1)


def interpolate_rope_freqs(sin: torch.Tensor, cos: torch.Tensor, target_len: int,
                           mode: Literal["linear", "nearest", "area"] = "linear") -> SinCos:
    """Resample ``[n, pairs]`` tables to ``target_len`` positions (variable-resolution
    inference): ``linear`` with the end points kept, ``nearest``, or ``area`` (mean over
    each target cell)."""
    n = sin.shape[0]
    if n == target_len:
        return sin, cos
    if mode == "area":
        pool = lambda t: F.adaptive_avg_pool1d(t.t()[None].float(), target_len)[0].t().to(t.dtype)
        return pool(sin), pool(cos)
    pos = torch.linspace(0, n - 1, target_len, device=sin.device, dtype=torch.float64)
    if mode == "nearest":
        idx = pos.round().long()
        return sin[idx], cos[idx]
    if mode != "linear":
        raise ValueError(f"unknown interpolation mode {mode!r}")
    lo = pos.floor().long().clamp(max=n - 1)
    hi = (lo + 1).clamp(max=n - 1)
    w = (pos - lo).to(sin.dtype)[:, None]
    return torch.lerp(sin[lo], sin[hi], w), torch.lerp(cos[lo], cos[hi], w)


def compute_resolution_aware_rope_freqs(dim: int, height: int, width: int, original_height: int,
                                        original_width: int, base: float = 10000.0,
                                        device=None, dtype: torch.dtype = torch.float32) -> SinCos:
    """2-D (row, column) tables ``[height * width, dim / 2]`` for a grid whose size
    differs from the training grid: positions are scaled by training / current size, so
    the grid spans the same angle range at any resolution. Half the channels follow the
    row, half the column."""
    if dim % 4:
        raise ValueError("resolution-aware RoPE needs dim divisible by 4")
    half = dim // 2
    sh, ch = _axis_freqs(height, half, base, device, torch.float64, original_height / height)
    sw, cw = _axis_freqs(width, half, base, device, torch.float64, original_width / width)
    grid = lambda a, b: torch.cat([a[:, None, :].expand(height, width, -1),
                                   b[None, :, :].expand(height, width, -1)], -1)
    # angle addition is not needed: the row and column pairs are separate channels
    sin = grid(sh, sw).reshape(height * width, half)
    cos = grid(ch, cw).reshape(height * width, half)
    return sin.to(dtype), cos.to(dtype)


def _freqs_for(config: RoPEConfig, seq_len: int, device=None) -> Tuple[torch.Tensor, torch.Tensor, float]:
    """(sin, cos, attention scale) for ``seq_len`` positions under the config's
    extension method (YaRN > dynamic NTK > static NTK > plain)."""
    if config.yarn_enabled:
        inv, temp = yarn_inv_freqs(config.dim, seq_len, config.original_max_seq_len, config.base,
                                   config.yarn_beta_fast, config.yarn_beta_slow, device)
        ang = torch.outer(torch.arange(seq_len, dtype=torch.float64, device=device), inv)
        return ang.sin().float(), ang.cos().float(), temp * config.yarn_mscale
    if config.dynamic_ntk:
        s, c = compute_dynamic_ntk_rope_freqs(config.dim, seq_len, config.original_max_seq_len,
                                              config.base, config.ntk_factor, device)
        return s, c, 1.0
    if config.ntk_alpha != 1.0:
        s, c = compute_ntk_rope_freqs(config.dim, seq_len, config.base, config.ntk_alpha, device)
        return s, c, 1.0
    s, c = compute_rope_freqs(config.dim, seq_len, config.base, device)
    return s, c, 1.0


# --------------------------------------------------------------------------- cache
class RoPEFrequencyCache:
    """Lazily filled tables keyed by length: ``get(n)`` returns a cached table, a slice
    of a longer cached one, or computes and stores it. The configured common lengths
    are computed up front. Tables are computed in float64/float32 and stored in
    ``dtype`` (fp16 when ``use_half_precision``)."""

    def __init__(self, config: RoPEConfig, device=None, dtype: Optional[torch.dtype] = None):
        self.config = config
        self.device = device
        self.dtype = dtype or (torch.float16 if config.use_half_precision else torch.float32)
        self.compute_dtype = torch.float32
        self._cache: Dict[int, SinCos] = {}
        self._3d_cache: Dict[tuple, object] = {}
        for n in config.cache_common_lengths:
            if n <= config.max_seq_len:
                self._store(n)

    def _store(self, n: int) -> SinCos:
        s, c, _ = _freqs_for(self.config, n, self.device)
        self._cache[n] = (s.to(self.dtype), c.to(self.dtype))
        return self._cache[n]

    def get(self, seq_len: int) -> SinCos:
        hit = self._cache.get(seq_len)
        if hit is not None:
            return hit
        longer = [n for n in self._cache if n >= seq_len]
        # dynamic NTK tables depend on the length itself: never slice them
        if longer and not self.config.dynamic_ntk and not self.config.yarn_enabled:
            s, c = self._cache[min(longer)]
            return s[:seq_len], c[:seq_len]
        return self._store(seq_len)

    def get_3d(self, max_time: int, max_height: int, max_width: int, efficient_mode: bool = True):
        key = (max_time, max_height, max_width, efficient_mode)
        if key not in self._3d_cache:
            res = compute_rope_3d_freqs(self.config.dim, max_time, max_height, max_width,
                                        self.config.base, self.config.temporal_base_factor,
                                        self.device, self.compute_dtype, efficient_mode)
            if efficient_mode:
                res = tuple((s.to(self.dtype), c.to(self.dtype)) for s, c in res)
            else:
                res = (res[0].to(self.dtype), res[1].to(self.dtype))
            self._3d_cache[key] = res
        return self._3d_cache[key]

    def to(self, device) -> "RoPEFrequencyCache":
        self.device = device
        self._cache = {n: (s.to(device), c.to(device)) for n, (s, c) in self._cache.items()}
        self._3d_cache = {}
        return self

    def clear(self) -> None:
        self._cache.clear()
        self._3d_cache.clear()


# --------------------------------------------------------------------------- layer
class RoPELayerV2(nn.Module):
    """Multi-mode RoPE on ``[B, T, H, D]`` (reference output layout: each pair's rotated
    halves written concatenated). Modes: 1-D with plain / NTK / dynamic-NTK / YaRN
    frequencies (``forward``, ``forward_qk``), factorised 3-D for video tokens
    (``forward_3d``), packed variable-length batches (``forward_flash`` with
    ``cu_seqlens``) and chunked application for long sequences (``forward_chunked``)."""

    def __init__(self, config: RoPEConfig):
        super().__init__()
        self.config = config
        self.cache: Optional[RoPEFrequencyCache] = None
        sin, cos, self._yarn_attention_scale = _freqs_for(config, config.max_seq_len)
        dt = torch.float16 if config.use_half_precision else torch.float32
        self.register_buffer("sin", sin.to(dt), persistent=False)
        self.register_buffer("cos", cos.to(dt), persistent=False)
        self._3d_freqs = None

    def get_attention_scale(self) -> float:
        """Multiplier of the attention logits under YaRN (1.0 otherwise)."""
        return self._yarn_attention_scale

    def _tables(self, end: int, seq_len: Optional[int], device, dtype) -> SinCos:
        n = seq_len or end
        if self.config.dynamic_ntk and n > self.config.original_max_seq_len:
            s, c, _ = _freqs_for(self.config, max(n, end), device)
        elif end > self.sin.shape[0]:
            s, c, _ = _freqs_for(self.config, end, device)
        else:
            s, c = self.sin, self.cos
        return s.to(device=device, dtype=dtype), c.to(device=device, dtype=dtype)

    def forward(self, x: torch.Tensor, start_pos: int = 0,
                seq_len: Optional[int] = None) -> torch.Tensor:
        T = x.shape[1]
        s, c = self._tables(start_pos + T, seq_len, x.device, x.dtype)
        return rope_apply(x, s[start_pos:start_pos + T, None, :], c[start_pos:start_pos + T, None, :])

    def forward_qk(self, q: torch.Tensor, k: torch.Tensor,
                   start_pos: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        T = q.shape[1]
        s, c = self._tables(start_pos + T, None, q.device, q.dtype)
        s, c = s[start_pos:start_pos + T, None, :], c[start_pos:start_pos + T, None, :]
        return rope_apply_qk(q, k, s, c)

    def forward_3d(self, x: torch.Tensor, time: int, height: int, width: int,
                   t_offset: int = 0, h_offset: int = 0, w_offset: int = 0) -> torch.Tensor:
        """``x [B, time*height*width, heads, dim]`` in (t, h, w) row-major token order."""
        if x.shape[1] != time * height * width:
            raise ValueError(f"sequence length {x.shape[1]} != {time}*{height}*{width}")
        need = (time + t_offset, height + h_offset, width + w_offset)
        f = self._3d_freqs
        if f is None or any(t[0].shape[0] < n for t, n in zip(f, need)) or f[0][0].device != x.device:
            sd = self.config.spatial_dims or (0, 0)
            self._3d_freqs = f = compute_rope_3d_freqs(
                self.config.dim, max(need[0], 1), max(need[1], sd[0]), max(need[2], sd[1]),
                self.config.base, self.config.temporal_base_factor, x.device, torch.float32)
        dev = x.device
        t_idx = torch.arange(t_offset, t_offset + time, device=dev)
        h_idx = torch.arange(h_offset, h_offset + height, device=dev)
        w_idx = torch.arange(w_offset, w_offset + width, device=dev)
        ti = t_idx[:, None, None].expand(time, height, width).reshape(-1)
        hi = h_idx[None, :, None].expand(time, height, width).reshape(-1)
        wi = w_idx[None, None, :].expand(time, height, width).reshape(-1)
        return apply_rope_3d_efficient(x, f[0], f[1], f[2], ti, hi, wi)

    def forward_flash(self, q: torch.Tensor, k: torch.Tensor, start_pos: int = 0,
                      cu_seqlens: Optional[torch.Tensor] = None,
                      max_seqlen: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Packed ``[total, heads, dim]`` tokens (``cu_seqlens [batch + 1]`` offsets, each
        sequence starting at ``start_pos``), or padded ``[B, T, H, D]`` / ``[T, H, D]``."""
        if cu_seqlens is None:
            if q.dim() == 3:
                qr, kr = self.forward_qk(q[None], k[None], start_pos)
                return qr[0], kr[0]
            return self.forward_qk(q, k, start_pos)
        total = q.shape[0]
        cu = cu_seqlens.to(device=q.device, dtype=torch.long)
        lengths = cu[1:] - cu[:-1]
        seq_start = torch.repeat_interleave(cu[:-1], lengths, output_size=total)
        pos = torch.arange(total, device=q.device) - seq_start + start_pos
        longest = int(max_seqlen) if max_seqlen is not None else int(lengths.max().item())
        s, c = self._tables(start_pos + longest, None, q.device, q.dtype)
        s, c = s[pos][:, None, :], c[pos][:, None, :]
        return rope_apply(q, s, c), rope_apply(k, s, c)

    def forward_chunked(self, x: torch.Tensor, chunk_size: int = 512,
                        start_pos: int = 0) -> torch.Tensor:
        """Rotation in chunks of ``chunk_size`` tokens (bounded temporaries)."""
        T = x.shape[1]
        if T <= chunk_size:
            return self.forward(x, start_pos)
        return torch.cat([self.forward(x[:, i:i + chunk_size], start_pos + i)
                          for i in range(0, T, chunk_size)], dim=1)

    def extra_repr(self) -> str:
        c = self.config
        parts = [f"dim={c.dim}", f"max_seq_len={c.max_seq_len}"]
        if c.ntk_alpha != 1.0:
            parts.append(f"ntk_alpha={c.ntk_alpha}")
        if c.dynamic_ntk:
            parts.append("dynamic_ntk=True")
        if c.yarn_enabled:
            parts.append("yarn=True")
        if c.spatial_dims:
            parts.append(f"spatial_dims={c.spatial_dims}")
        return ", ".join(parts)


# --------------------------------------------------------------------------- compat helpers
def precompute_rope_freqs(dim: int, max_seq_len: int, base: float = 10000.0, device=None) -> SinCos:
    return compute_rope_freqs(dim, max_seq_len, base, device)


def precompute_rope_3d_freqs(dim: int, max_time: int, max_height: int, max_width: int,
                             base: float = 10000.0, device=None) -> SinCos:
    return compute_rope_3d_freqs(dim, max_time, max_height, max_width, base, device=device,
                                 efficient_mode=False)


def rope(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor) -> torch.Tensor:
    return rope_apply(x, sin, cos, interleaved=True)


def yarn_attention_scale(seq_len: int, original_max_len: int, mscale: float = 1.0) -> float:
    """YaRN's logit temperature ``(0.1 ln s + 1) * mscale`` for the length ratio ``s``."""
    s = seq_len / original_max_len
    return (0.1 * math.log(s) + 1.0) * mscale if s > 1 else mscale
