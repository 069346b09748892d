"""The reference's fused-op functions and modules (layers/kernels/fused_ops.py:237-465:
``fused_rmsnorm``, ``fused_silu_multiply``, ``fused_add_rmsnorm``,
``fused_rotary_embedding``, ``FusedRMSNorm``, ``FusedSiLUMLP``) on this framework's
kernels.

On CUDA tensors the RMSNorm runs on the AdaLN-RMSNorm kernel (``csrc/fused/norm.cu``, the
modulation set to zero) for widths that kernel takes (multiples of 256 up to 2048, not
1280 or 1792), and the MLP projections on the tcgen05 GEMM (``ops.linear``). Everything
else, and every CPU tensor, is computed with PyTorch: the multiply of ``silu(gate) * up``
and the rotary rotation are single elementwise passes either way, and in the fused engine
they live in GEMM epilogues (SwiGLU, rotary) rather than in kernels of their own. The
outputs keep the input dtype. None of the functions records an autograd graph through the
kernel path except :class:`FusedSiLUMLP` (``ops.linear`` is differentiable).
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

_ADALN_WIDTHS = {256, 512, 768, 1024, 1536, 2048}


def _rmsnorm_torch(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).to(x.dtype)


def fused_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``x / rms(x) * weight`` over the last dim; ``x`` is ``[..., D]``."""
    D = x.shape[-1]
    if x.is_cuda and D in _ADALN_WIDTHS and not torch.is_grad_enabled():
        from ..ops.fused import adaln_rmsnorm

        x2 = x.reshape(-1, D).to(torch.bfloat16).contiguous()
        mod = torch.zeros(1, 2 * D, device=x.device, dtype=torch.float32)
        h, _ = adaln_rmsnorm(x2, weight.float().contiguous(), mod, 0, D, x2.shape[0], eps)
        return h.view(x.shape).to(x.dtype)
    return _rmsnorm_torch(x, weight, eps)


def fused_silu_multiply(x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """``silu(x) * gate``."""
    return F.silu(x) * gate


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float = 1e-6) -> torch.Tensor:
    """``rmsnorm(x + residual) * weight``."""
    return fused_rmsnorm(x + residual, weight, eps)


def fused_rotary_embedding(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor,
                           sin: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotary embedding of ``[B, T, H, D]`` q and k with interleaved pairs (channels 2i,
    2i + 1 rotate together); ``cos`` / ``sin`` are ``[T, D/2]``."""
    c = cos[None, :, None, :].to(q.dtype)
    s = sin[None, :, None, :].to(q.dtype)

    def rot(x):
        a, b = x[..., 0::2], x[..., 1::2]
        return torch.stack([a * c - b * s, a * s + b * c], dim=-1).flatten(-2)

    return rot(q), rot(k)


class FusedRMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if torch.is_grad_enabled() and self.weight.requires_grad:
            return _rmsnorm_torch(x, self.weight, self.eps)  # differentiable path
        return fused_rmsnorm(x, self.weight, self.eps)


class FusedSiLUMLP(nn.Module):
    """``down_proj(silu(gate_proj x) * up_proj x)`` (the reference's parameter names)."""

    def __init__(self, d_model: int, d_ff: int):
        super().__init__()
        self.up_proj = nn.Linear(d_model, d_ff, bias=False)
        self.gate_proj = nn.Linear(d_model, d_ff, bias=False)
        self.down_proj = nn.Linear(d_ff, d_model, bias=False)
        for lin in (self.up_proj, self.gate_proj):
            nn.init.normal_(lin.weight, std=0.02)
        nn.init.normal_(self.down_proj.weight, std=0.02 / math.sqrt(24))

    @staticmethod
    def _proj(x: torch.Tensor, lin: nn.Linear) -> torch.Tensor:
        if x.is_cuda and x.shape[-1] % 64 == 0 and lin.out_features % 64 == 0:
            from ..ops.linear import linear

            flat = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
            y = linear(flat, lin.weight.to(torch.bfloat16), None, lin.weight, None)
            return y.view(*x.shape[:-1], -1)
        return lin(x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = fused_silu_multiply(self._proj(x, self.gate_proj), self._proj(x, self.up_proj))
        return self._proj(h.contiguous(), self.down_proj)
