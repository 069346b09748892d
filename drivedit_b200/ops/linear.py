"""``y = x W^T (+ b)`` on the tcgen05 GEMM with a hand-written backward.

Forward and both backward products (``dx = dy W`` reading ``W`` transposed in place,
``dW += dy^T x`` reading both operands transposed, fp32 split-K accumulation straight
into the parameter's flat gradient view) run on ``csrc/gemm/gemm.cu``; no cuBLAS.
"""
from __future__ import annotations

from typing import Optional

import torch

from .gemm import gemm


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_bf16, bias, w_param, b_param):
        y = gemm(x, w_bf16, bias=bias)
        ctx.save_for_backward(x, w_bf16)
        ctx.w_param, ctx.b_param = w_param, b_param
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = gemm(dy, w, b_t=True) if ctx.needs_input_grad[0] else None
        wp, bp = ctx.w_param, ctx.b_param
        if wp is not None:
            if wp.grad is None:
                wp.grad = torch.zeros_like(wp)
            gemm(dy, x, wp.grad, epi="f32_acc", a_t=True, b_t=True)
        if bp is not None:
            if bp.grad is None:
                bp.grad = torch.zeros_like(bp)
            bp.grad.add_(dy.float().sum(0))
        return dx, None, None, None, None


def linear(x: torch.Tensor, w_bf16: torch.Tensor, bias: Optional[torch.Tensor] = None,
           w_param: Optional[torch.nn.Parameter] = None,
           b_param: Optional[torch.nn.Parameter] = None) -> torch.Tensor:
    """``x [M, K] bf16``, ``w_bf16 [N, K]``; weight/bias gradients go to ``w_param.grad``
    / ``b_param.grad`` (fp32) when given."""
    return _LinearFn.apply(x, w_bf16, bias, w_param, b_param)
