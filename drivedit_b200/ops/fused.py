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


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).to(torch.bfloat16).contiguous()
        w = None if weight is None else weight.detach().float().contiguous()
        b = None if bias is None else bias.detach().float().contiguous()
        y, mean, rstd = ext().layernorm_fwd(x2, w, b, eps)
        ctx.save_for_backward(x2, mean, rstd)
        ctx.w, ctx.params = w, (weight, bias)
        ctx.shp = shp
        return y.view(shp)

    @staticmethod
    def backward(ctx, dy):
        x2, mean, rstd = ctx.saved_tensors
        weight, bias = ctx.params
        D = x2.shape[1]
        dw = torch.zeros(D, device=x2.device) if weight is not None and weight.requires_grad else None
        db = torch.zeros(D, device=x2.device) if bias is not None and bias.requires_grad else None
        dx = ext().layernorm_bwd(dy.reshape(-1, D).to(torch.bfloat16).contiguous(), x2, mean, rstd,
                                 ctx.w, dw, db)
        return (dx.view(ctx.shp), None if dw is None else dw.to(weight.dtype),
                None if db is None else db.to(bias.dtype), None)


def layer_norm(x: torch.Tensor, weight: Optional[torch.Tensor] = None,
               bias: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm over the last dim on ``csrc/fused/layernorm.cu`` (bf16 out, fp32 stats),
    differentiable in ``x``, ``weight`` and ``bias``; ``D`` a multiple of 256."""
    return _LayerNormFn.apply(x, weight, bias, eps)
