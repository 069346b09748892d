"""Rotary position embeddings: 1-D, NTK / dynamic-NTK / YaRN extensions, factorised 3-D.

Capabilities mirror the reference's ``layers/rope_v2.py`` (basic freqs :181-220,
NTK :223-271, dynamic NTK :274-308, YaRN :311-398, 3-D factorised :405-501,
``RoPELayer`` compat :1256-1285, ``rope_apply`` :95-148).

Conventions used by this framework (and by the fused GEMM epilogue):
  * a table is ``[P, dim/2, 2]`` fp32 holding (cos, sin) of the angle of each rotation
    pair at each position ``P``;
  * pair ``i`` rotates channels ``(2i, 2i+1)`` in place ("interleaved in, interleaved
    out"). The reference's ``rope_apply`` reads interleaved pairs but writes the two
    rotated halves concatenated; :func:`rope_apply` reproduces that layout for
    reference-compatibility, and :func:`apply_rope` is the in-place convention.
  * 3-D RoPE splits the head dim over (t, h, w) axes. The reference requires
    ``dim % 6 == 0`` (rope_v2.py:456), which rules out d_head = 64; here the split is
    explicit and defaults to (16, 24, 24) channels for d_head = 64 (8/12/12 pairs),
    i.e. any split with even parts works.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn


def inv_freqs(dim: int, base: float = 10000.0, device=None) -> torch.Tensor:
    """``base ** (-2i/dim)`` for the ``dim/2`` rotation pairs of a ``dim``-channel axis."""
    assert dim % 2 == 0, f"rotary dim must be even, got {dim}"
    return 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64, device=device) / dim))


def rope_angles_1d(dim: int, positions: torch.Tensor, base: float = 10000.0) -> torch.Tensor:
    """Angles ``[len(positions), dim/2]`` (float64 for accuracy, cast by the caller)."""
    return torch.outer(positions.to(torch.float64), inv_freqs(dim, base, positions.device))


def compute_rope_freqs(dim: int, max_seq_len: int, base: float = 10000.0, device=None,
                       dtype: torch.dtype = torch.float32):
    """(sin, cos) ``[max_seq_len, dim/2]`` — the reference's return order; angles in
    float64, tables in ``dtype``."""
    ang = rope_angles_1d(dim, torch.arange(max_seq_len, device=device), base)
    return ang.sin().to(dtype), ang.cos().to(dtype)


def ntk_base(base: float, dim: int, alpha: float) -> float:
    """NTK-aware base stretch ``base * alpha^(dim/(dim-2))`` (Code Llama style)."""
    return base * alpha ** (dim / (dim - 2)) if alpha != 1.0 else base


def compute_ntk_rope_freqs(dim, max_seq_len, base=10000.0, alpha=1.0, device=None,
                           dtype: torch.dtype = torch.float32):
    return compute_rope_freqs(dim, max_seq_len, ntk_base(base, dim, alpha), device, dtype)


def compute_dynamic_ntk_rope_freqs(dim, seq_len, original_max_len, base=10000.0,
                                   ntk_factor=1.0, device=None, dtype: torch.dtype = torch.float32):
    """Standard RoPE up to the training length; past it, alpha grows with the ratio."""
    if seq_len <= original_max_len:
        return compute_rope_freqs(dim, seq_len, base, device, dtype)
    alpha = ntk_factor * seq_len / original_max_len - (ntk_factor - 1)
    return compute_ntk_rope_freqs(dim, seq_len, base, alpha, device, dtype)


def yarn_inv_freqs(dim, max_seq_len, original_max_len, base=10000.0, beta_fast=32.0,
                   beta_slow=1.0, device=None) -> Tuple[torch.Tensor, float]:
    """YaRN (Peng et al. 2023, arXiv:2309.00071): frequencies whose wavelength fits many
    times in the training window keep their value, those longer than it are
    interpolated by the length ratio, with a linear ramp between ``beta_fast`` and
    ``beta_slow`` rotations. Returns the frequencies and the attention temperature
    ``0.1 ln(s) + 1``."""
    inv = inv_freqs(dim, base, device)
    s = max_seq_len / original_max_len
    if s <= 1.0:
        return inv, 1.0
    rotations = original_max_len * inv / (2 * math.pi)  # turns inside the training window
    ramp = ((rotations - beta_slow) / (beta_fast - beta_slow)).clamp(0, 1)
    mixed = inv / s * (1 - ramp) + inv * ramp
    return mixed, 0.1 * math.log(s) + 1.0


def compute_yarn_rope_freqs(dim, max_seq_len, original_max_len, base=10000.0,
                            beta_fast=32.0, beta_slow=1.0, mscale: float = 0.0, device=None,
                            dtype: torch.dtype = torch.float32):
    """(sin, cos, attention scale); ``mscale > 0`` overrides the automatic scale
    ``0.1 ln(s) + 1``."""
    inv, auto = yarn_inv_freqs(dim, max_seq_len, original_max_len, base, beta_fast,
                               beta_slow, device)
    ang = torch.outer(torch.arange(max_seq_len, dtype=torch.float64, device=device), inv)
    return ang.sin().to(dtype), ang.cos().to(dtype), (mscale if mscale > 0 else auto)


def interpolate_positions(seq_len: int, train_len: int, device=None) -> torch.Tensor:
    """Position interpolation: squeeze ``seq_len`` positions into ``[0, train_len)``."""
    scale = min(1.0, train_len / max(seq_len, 1))
    return torch.arange(seq_len, dtype=torch.float64, device=device) * scale


DEFAULT_SPLIT_64 = (16, 24, 24)


def default_split(head_dim: int) -> Tuple[int, int, int]:
    """Channel split over (t, h, w): 1/4 time, 3/8 height, 3/8 width, all even."""
    if head_dim == 64:
        return DEFAULT_SPLIT_64
    t = (head_dim // 4) & ~1
    h = ((head_dim - t) // 2) & ~1
    w = head_dim - t - h
    return t, h, w


def rope_angles_3d(
    head_dim: int,
    frames: int,
    height: int,
    width: int,
    base: float = 10000.0,
    temporal_base_factor: float = 1.0,
    split: Optional[Sequence[int]] = None,
    frame_offset: int = 0,
    device=None,
) -> torch.Tensor:
    """Angles ``[frames*height*width, head_dim/2]`` for tokens in (t, h, w) row-major
    order. Pairs ``[0, st/2)`` follow the frame index, the next ``sh/2`` the row, the
    last ``sw/2`` the column. The temporal base is ``base * temporal_base_factor``
    (reference rope_v2.py:463)."""
    st, sh, sw = split if split is not None else default_split(head_dim)
    assert st + sh + sw == head_dim and st % 2 == 0 and sh % 2 == 0 and sw % 2 == 0
    t = torch.arange(frame_offset, frame_offset + frames, dtype=torch.float64, device=device)
    h = torch.arange(height, dtype=torch.float64, device=device)
    w = torch.arange(width, dtype=torch.float64, device=device)
    at = torch.outer(t, inv_freqs(st, base * temporal_base_factor, device))  # [F, st/2]
    ah = torch.outer(h, inv_freqs(sh, base, device))
    aw = torch.outer(w, inv_freqs(sw, base, device))
    F_, H_, W_ = frames, height, width
    at = at[:, None, None, :].expand(F_, H_, W_, -1)
    ah = ah[None, :, None, :].expand(F_, H_, W_, -1)
    aw = aw[None, None, :, :].expand(F_, H_, W_, -1)
    return torch.cat([at, ah, aw], -1).reshape(F_ * H_ * W_, head_dim // 2)


def rope_table(angles: torch.Tensor) -> torch.Tensor:
    """``[P, pairs]`` angles -> contiguous fp32 ``[P, pairs, 2]`` (cos, sin) table."""
    return torch.stack([angles.cos(), angles.sin()], -1).float().contiguous()


def apply_rope(x: torch.Tensor, table: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """Rotate channel pairs ``(2i, 2i+1)`` of ``x [..., T, H, D]`` with ``table
    [T, D/2, 2]``; ``inverse`` rotates by the negative angle (the backward pass)."""
    T, H, D = x.shape[-3:]
    xf = x.float().reshape(*x.shape[:-1], D // 2, 2)
    c = table[:T, None, :, 0]
    s = table[:T, None, :, 1]
    if inverse:
        s = -s
    x0, x1 = xf[..., 0], xf[..., 1]
    out = torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], -1)
    return out.reshape(x.shape).to(x.dtype)


def rope_apply(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor,
               interleaved: bool = True) -> torch.Tensor:
    """Reference-layout rotation (rope_v2.py:95-148): reads pairs interleaved (or as
    halves) and writes ``cat(x1*cos - x2*sin, x1*sin + x2*cos)``."""
    if interleaved:
        x1, x2 = x[..., 0::2], x[..., 1::2]
    else:
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


class RoPELayer(nn.Module):
    """Reference-compatible 1-D RoPE layer: ``forward(x [B,T,H,D], start_pos)`` rotates
    with the reference's output layout; positions start at ``start_pos``."""

    def __init__(self, dim: int, max_seq_len: int = 2048, base: float = 10000.0):
        super().__init__()
        self.dim, self.max_seq_len, self.base = dim, max_seq_len, base
        sin, cos = compute_rope_freqs(dim, max_seq_len, base)
        self.register_buffer("sin_cached", sin, persistent=False)
        self.register_buffer("cos_cached", cos, persistent=False)

    def forward(self, x: torch.Tensor, start_pos: int = 0) -> torch.Tensor:
        T = x.shape[1]
        if start_pos + T > self.sin_cached.shape[0]:
            sin, cos = compute_rope_freqs(self.dim, start_pos + T, self.base, x.device)
        else:
            sin, cos = self.sin_cached, self.cos_cached
        sin = sin[start_pos:start_pos + T].to(x.device, x.dtype)[None, :, None, :]
        cos = cos[start_pos:start_pos + T].to(x.device, x.dtype)[None, :, None, :]
        return rope_apply(x, sin, cos, interleaved=True)


class RoPE3D(nn.Module):
    """Factorised (t, h, w) RoPE for a latent-video token grid, in-place pair layout.

    ``table(frames, frame_offset)`` returns the ``[frames*H*W, D/2, 2]`` table that both
    the PyTorch path and the fused QKV-GEMM epilogue consume."""

    def __init__(self, head_dim: int, height: int, width: int, max_frames: int = 256,
                 base: float = 10000.0, temporal_base_factor: float = 1.0,
                 split: Optional[Sequence[int]] = None):
        super().__init__()
        self.head_dim, self.height, self.width = head_dim, height, width
        self.base, self.temporal_base_factor = base, temporal_base_factor
        self.split = tuple(split) if split is not None else default_split(head_dim)
        self.max_frames = max_frames
        ang = rope_angles_3d(head_dim, max_frames, height, width, base,
                             temporal_base_factor, self.split)
        self.register_buffer("tab", rope_table(ang), persistent=False)

    @property
    def tokens_per_frame(self) -> int:
        return self.height * self.width

    def table(self, frames: int, frame_offset: int = 0) -> torch.Tensor:
        if frame_offset + frames > self.max_frames:
            ang = rope_angles_3d(self.head_dim, frames, self.height, self.width, self.base,
                                 self.temporal_base_factor, self.split, frame_offset,
                                 self.tab.device)
            return rope_table(ang)
        n = self.tokens_per_frame
        return self.tab[frame_offset * n:(frame_offset + frames) * n]

    def forward(self, x: torch.Tensor, frame_offset: int = 0) -> torch.Tensor:
        frames = x.shape[-3] // self.tokens_per_frame
        return apply_rope(x, self.table(frames, frame_offset))
