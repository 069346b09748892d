"""Normalisation layers: RMSNorm, LayerNorm, AdaLN (scale/shift) and AdaLN-Zero (gated).

Semantics follow the reference's ``layers/nn_helpers.py``:
  * ``RMSNorm`` (nn_helpers.py:39-65): fp32 normalise, eps 1e-6, cast back, times weight.
  * ``AdaLN`` (nn_helpers.py:92-139): ``RMSNorm(x) * (1 + scale) + shift`` where
    ``(scale, shift) = cond_proj(cond).chunk(2)``; ``cond`` is ``[B, C]`` (broadcast over
    tokens) or ``[B, T, C]``. The state-dict names (``norm.weight``,
    ``cond_proj.{weight,bias}``) match the reference so its checkpoints load unchanged.

One deliberate difference: the reference initialises ``cond_proj.bias[0::2] = 1``
while splitting the output into halves with ``chunk(2)``, which makes its "identity"
init scale every even channel by 2 and shift it by 1. Here the projection starts at
exactly zero, so a fresh AdaLN is the identity on top of the RMSNorm.

On CUDA the fused kernel ``drivedit_b200.ops.norm.adaln_rmsnorm`` computes the same
function for the per-frame modulation used by the world models.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def _norm(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._norm(x.float()).type_as(x) * self.weight.to(x.dtype)


class LayerNorm(nn.Module):
    def __init__(self, dim: int, bias: bool = False, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))
        self.bias = nn.Parameter(torch.zeros(dim)) if bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.layer_norm(x, self.weight.shape, self.weight, self.bias, self.eps)


def _split_modulation(params: torch.Tensor, n: int):
    chunks = params.chunk(n, dim=-1)
    if params.dim() == 2:  # [B, n*D] -> broadcast over tokens
        chunks = tuple(c.unsqueeze(1) for c in chunks)
    return chunks


class AdaLN(nn.Module):
    """Adaptive RMSNorm: ``norm(x) * (1 + scale) + shift`` from a conditioning vector."""

    def __init__(self, dim: int, cond_dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.norm = RMSNorm(dim, eps)
        self.cond_proj = nn.Linear(cond_dim, 2 * dim, bias=True)
        nn.init.zeros_(self.cond_proj.weight)
        nn.init.zeros_(self.cond_proj.bias)

    def modulation(self, cond: torch.Tensor):
        return _split_modulation(self.cond_proj(cond), 2)

    def forward(self, x: torch.Tensor, cond: torch.Tensor) -> torch.Tensor:
        scale, shift = self.modulation(cond)
        return self.norm(x) * (1 + scale) + shift


class AdaLNZero(nn.Module):
    """AdaLN with a residual gate (DiT "adaLN-Zero"), as the reference's
    ``FlowMatchingBlock`` (blocks/flow_matching.py:131-144) uses it: returns the
    modulated input and the gate ``alpha`` for the residual branch. Zero init makes
    every residual branch start closed."""

    def __init__(self, dim: int, cond_dim: int, eps: float = 1e-6):
        super().__init__()
        self.norm = RMSNorm(dim, eps)
        self.cond_proj = nn.Linear(cond_dim, 3 * dim, bias=True)
        nn.init.zeros_(self.cond_proj.weight)
        nn.init.zeros_(self.cond_proj.bias)

    def forward(self, x: torch.Tensor, cond: torch.Tensor):
        scale, shift, gate = _split_modulation(self.cond_proj(cond), 3)
        return self.norm(x) * (1 + scale) + shift, gate


def adaln_rmsnorm_reference(
    x: torch.Tensor,
    weight: Optional[torch.Tensor],
    scale: torch.Tensor,
    shift: torch.Tensor,
    eps: float = 1e-6,
) -> torch.Tensor:
    """fp32 reference of the fused op: ``rmsnorm(x) * w * (1 + scale) + shift``.

    ``x`` is ``[B, T, D]``; ``scale``/``shift`` broadcast to it (``[B, 1, D]``,
    ``[B, T, D]``, or per-frame ``[B, F, 1, D]`` after the caller reshapes x).
    """
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.float()
    return y * (1 + scale.float()) + shift.float()
