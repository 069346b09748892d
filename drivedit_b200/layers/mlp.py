"""Feed-forward layers: MLP, SwiGLU, GeGLU, ConditionalMLP and the ``create_mlp`` factory.

Same capabilities and state-dict names as the reference's ``layers/mlp.py``
(MLP :13-83, SwiGLU :86-155 with ``w1`` gate / ``w2`` value / ``w3`` out and default
hidden ``8d/3`` rounded up to a multiple of 8 :101-105, GeGLU :158-211,
ConditionalMLP :214-272, factory :275-304).

The fused CUDA path stores the gate and value projections as one ``[2F, d]`` matrix
whose rows alternate in groups of 32 (32 gate rows, then the 32 matching value rows),
so that one 256-wide GEMM tile holds matching gate/value columns and the SwiGLU is
applied in the GEMM epilogue. :func:`pack_swiglu` / :func:`unpack_swiglu` convert.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

GROUP = 32


def pack_swiglu(w_gate: torch.Tensor, w_value: torch.Tensor) -> torch.Tensor:
    """``[F, d]`` gate and value weights -> ``[2F, d]`` with rows interleaved by 32."""
    Fh, d = w_gate.shape
    assert Fh % GROUP == 0
    return torch.stack([w_gate.view(Fh // GROUP, GROUP, d), w_value.view(Fh // GROUP, GROUP, d)],
                       1).reshape(2 * Fh, d)


def unpack_swiglu(w: torch.Tensor):
    F2, d = w.shape
    v = w.view(F2 // (2 * GROUP), 2, GROUP, d)
    return v[:, 0].reshape(F2 // 2, d), v[:, 1].reshape(F2 // 2, d)


def split_gu(gu: torch.Tensor):
    """Interleaved ``[..., 2F]`` pre-activation -> (gate, value) each ``[..., F]``."""
    *lead, F2 = gu.shape
    v = gu.view(*lead, F2 // (2 * GROUP), 2, GROUP)
    return v[..., 0, :].reshape(*lead, F2 // 2), v[..., 1, :].reshape(*lead, F2 // 2)


def swiglu_hidden(d_model: int, d_ff: Optional[int] = None, multiple_of: int = 8) -> int:
    if d_ff is not None:
        return d_ff
    h = int(8 * d_model / 3)
    return multiple_of * ((h + multiple_of - 1) // multiple_of)


_ACTIVATIONS = {"silu": F.silu, "swish": F.silu, "gelu": F.gelu, "relu": F.relu}


def _init_in_out(w_in, w_out, biases=()):
    """Input projections N(0, 0.02); the projection back into the residual stream
    N(0, 0.02 / sqrt(24)) (depth-scaled); biases zero."""
    for w in w_in:
        nn.init.normal_(w.weight, std=0.02)
    nn.init.normal_(w_out.weight, std=0.02 / math.sqrt(24.0))
    for lin in list(w_in) + [w_out]:
        if lin.bias is not None:
            nn.init.zeros_(lin.bias)


class MLP(nn.Module):
    """``w2(act(w1 x))``; ``activation`` one of silu (default), swish, gelu (exact), relu."""

    def __init__(self, d_model: int, d_ff: Optional[int] = None, activation: str = "silu",
                 dropout: float = 0.0, bias: bool = False):
        super().__init__()
        if activation not in _ACTIVATIONS:
            raise ValueError(f"Unsupported activation: {activation}")
        self.d_model, self.d_ff = d_model, d_ff or 4 * d_model
        self.activation_name = activation
        self.activation = _ACTIVATIONS[activation]
        self.w1 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w2 = nn.Linear(self.d_ff, d_model, bias=bias)
        self.drop = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        _init_in_out([self.w1], self.w2)

    def forward(self, x):
        return self.w2(self.drop(self.activation(self.w1(x))))


class SwiGLU(nn.Module):
    """``w3(silu(w1 x) * w2 x)``."""

    def __init__(self, d_model: int, d_ff: Optional[int] = None, dropout: float = 0.0,
                 bias: bool = False):
        super().__init__()
        self.d_ff = swiglu_hidden(d_model, d_ff)
        self.w1 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w2 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w3 = nn.Linear(self.d_ff, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()

    def forward(self, x):
        return self.w3(self.dropout(F.silu(self.w1(x)) * self.w2(x)))


class GeGLU(nn.Module):
    """``w3(gelu(w1 x) * w2 x)`` (exact GELU), hidden ``8d/3`` rounded up to 8 by default."""

    def __init__(self, d_model: int, d_ff: Optional[int] = None, dropout: float = 0.0,
                 bias: bool = False):
        super().__init__()
        self.d_model = d_model
        self.d_ff = swiglu_hidden(d_model, d_ff)
        self.w1 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w2 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w3 = nn.Linear(self.d_ff, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        _init_in_out([self.w1, self.w2], self.w3)

    def forward(self, x):
        return self.w3(self.dropout(F.gelu(self.w1(x)) * self.w2(x)))


class ConditionalMLP(nn.Module):
    """A standard :class:`MLP` applied to ``x + cond_proj(cond)``; ``cond`` is per token
    ``[B, T, d_cond]`` or per sample ``[B, d_cond]`` (broadcast over the tokens)."""

    def __init__(self, d_model: int, d_cond: int, d_ff: Optional[int] = None,
                 activation: str = "silu", dropout: float = 0.0, bias: bool = False):
        super().__init__()
        self.d_model, self.d_cond = d_model, d_cond
        self.mlp = MLP(d_model, d_ff or 4 * d_model, activation, dropout, bias)
        self.d_ff = self.mlp.d_ff
        self.cond_proj = nn.Linear(d_cond, d_model, bias=bias)
        nn.init.normal_(self.cond_proj.weight, std=0.02)
        if bias:
            nn.init.zeros_(self.cond_proj.bias)

    def forward(self, x, cond):
        c = self.cond_proj(cond)
        return self.mlp(x + (c[:, None] if c.dim() == 2 else c))


def create_mlp(d_model: int, mlp_type: str = "standard", d_ff: Optional[int] = None,
               activation: str = "silu", dropout: float = 0.0, bias: bool = False,
               d_cond: Optional[int] = None) -> nn.Module:
    """``standard`` (an :class:`MLP` with ``activation``), ``swiglu``, ``geglu``; also
    ``gelu`` / ``relu`` / ``silu`` (a standard MLP with that activation) and
    ``conditional`` (needs ``d_cond``)."""
    if mlp_type == "standard":
        return MLP(d_model, d_ff, activation, dropout, bias)
    if mlp_type == "swiglu":
        return SwiGLU(d_model, d_ff, dropout, bias)
    if mlp_type == "geglu":
        return GeGLU(d_model, d_ff, dropout, bias)
    if mlp_type in ("gelu", "relu", "silu"):
        return MLP(d_model, d_ff, mlp_type, dropout, bias)
    if mlp_type == "conditional":
        if d_cond is None:
            raise ValueError("the conditional MLP needs d_cond")
        return ConditionalMLP(d_model, d_cond, d_ff, activation, dropout, bias)
    raise ValueError(f"Unsupported MLP type: {mlp_type}")
