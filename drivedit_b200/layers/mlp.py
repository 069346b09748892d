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


class MLP(nn.Module):
    def __init__(self, d_model: int, d_ff: Optional[int] = None, activation: str = "gelu",
                 dropout: float = 0.0, bias: bool = True):
        super().__init__()
        d_ff = d_ff or 4 * d_model
        self.fc1 = nn.Linear(d_model, d_ff, bias=bias)
        self.fc2 = nn.Linear(d_ff, d_model, bias=bias)
        self.act = {"gelu": nn.GELU(approximate="tanh"), "relu": nn.ReLU(),
                    "silu": nn.SiLU()}[activation]
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()

    def forward(self, x):
        return self.fc2(self.dropout(self.act(self.fc1(x))))


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
    def __init__(self, d_model: int, d_ff: Optional[int] = None, dropout: float = 0.0,
                 bias: bool = False):
        super().__init__()
        self.d_ff = swiglu_hidden(d_model, d_ff)
        self.w1 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w2 = nn.Linear(d_model, self.d_ff, bias=bias)
        self.w3 = nn.Linear(self.d_ff, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()

    def forward(self, x):
        return self.w3(self.dropout(F.gelu(self.w1(x), approximate="tanh") * self.w2(x)))


class ConditionalMLP(nn.Module):
    """SwiGLU whose hidden activations are FiLM-modulated by a conditioning vector."""

    def __init__(self, d_model: int, cond_dim: int, d_ff: Optional[int] = None,
                 dropout: float = 0.0, bias: bool = False):
        super().__init__()
        self.mlp = SwiGLU(d_model, d_ff, dropout, bias)
        self.film = nn.Linear(cond_dim, 2 * self.mlp.d_ff)
        nn.init.zeros_(self.film.weight)
        nn.init.zeros_(self.film.bias)

    def forward(self, x, cond):
        gamma, beta = self.film(cond).chunk(2, -1)
        if gamma.dim() == 2:
            gamma, beta = gamma[:, None], beta[:, None]
        h = F.silu(self.mlp.w1(x)) * self.mlp.w2(x)
        h = h * (1 + gamma) + beta
        return self.mlp.w3(self.mlp.dropout(h))


def create_mlp(d_model: int, mlp_type: str = "swiglu", d_ff: Optional[int] = None,
               dropout: float = 0.0, bias: bool = False, **kw) -> nn.Module:
    if mlp_type == "swiglu":
        return SwiGLU(d_model, d_ff, dropout, bias)
    if mlp_type == "geglu":
        return GeGLU(d_model, d_ff, dropout, bias)
    if mlp_type in ("gelu", "relu", "silu", "mlp"):
        return MLP(d_model, d_ff, "gelu" if mlp_type == "mlp" else mlp_type, dropout, bias)
    if mlp_type == "conditional":
        return ConditionalMLP(d_model, kw["cond_dim"], d_ff, dropout, bias)
    raise ValueError(f"unknown mlp_type {mlp_type!r}")
