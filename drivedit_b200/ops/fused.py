"""Wrappers of the memory-bound fused kernels (``csrc/fused``): AdaLN-RMSNorm fwd/bwd,
flat AdamW, casts, squared norm, rotary rotation."""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ._ext import ext


def adaln_rmsnorm(x: torch.Tensor, w: torch.Tensor, mod: torch.Tensor, scale_off: int,
                  shift_off: int, rows_per_group: int, eps: float = 1e-6
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """``h = rmsnorm(x) * w * (1 + mod[g, scale_off:+D]) + mod[g, shift_off:+D]`` with
    ``g = row // rows_per_group``; returns ``(h bf16, rstd fp32)``."""
    return tuple(ext().adaln_fwd(x, w, mod, scale_off, shift_off, rows_per_group, eps))


def adaln_rmsnorm_bwd(dh, x, rstd, w, mod, scale_off, shift_off, rows_per_group,
                      dmod: torch.Tensor, dw: Optional[torch.Tensor] = None,
                      dres: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Returns ``dx (+ dres)``; accumulates into ``dw`` and ``dmod`` (fp32)."""
    return ext().adaln_bwd(dh, x, rstd, w, mod, scale_off, shift_off, rows_per_group, dres,
                           dw, dmod)


def adamw_flat(master, grad, m, v, compute, clip, *, lr, b1, b2, eps, wd, bc1, bc2,
               grad_scale=1.0, decay_end=None):
    ext().adamw_flat(master, grad, m, v, compute, clip, lr, b1, b2, eps, wd, bc1, bc2,
                     grad_scale, master.numel() if decay_end is None else decay_end)


def cast_bf16(src: torch.Tensor, dst: Optional[torch.Tensor] = None) -> torch.Tensor:
    dst = torch.empty(src.shape, device=src.device, dtype=torch.bfloat16) if dst is None else dst
    ext().cast_bf16(src, dst)
    return dst


def sq_norm(x: torch.Tensor) -> torch.Tensor:
    return ext().sq_norm(x)


def rope_rotate_(x: torch.Tensor, rot_cols: int, tab: torch.Tensor, head_dim: int = 64,
                 rows_per_seq: int = 1 << 30, pos_offset: int = 0, inverse: bool = False):
    ext().rope_rotate(x, rot_cols, tab, head_dim, rows_per_seq, pos_offset, inverse)
    return x
