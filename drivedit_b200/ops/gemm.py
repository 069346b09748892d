"""tcgen05 GEMM entry points (``csrc/gemm/gemm.cu``).

``gemm(a, b)`` computes ``a @ b.T`` for bf16 ``a [M, K]`` and ``b [N, K]``. ``a_t`` /
``b_t`` say the operand is stored transposed (``a`` as ``[K, M]``, ``b`` as ``[K, N]``),
which is how the backward pass reads activations and weights without a transpose copy.
The epilogue is fused into the kernel:

=============  ==============================================================
``bf16``       ``out = acc (+ bias) (+ residual)``, bf16
``f32``        ``out = acc (+ bias)``, fp32
``f32_acc``    ``out += acc`` with fp32 vector reductions (split-K, grad accumulation)
``swiglu``     ``gu = acc`` (gate/up interleaved in groups of 32), ``act = silu(g) * u``
``dswiglu``    ``acc = d(act)``; writes ``d(gu)`` using the saved ``gu``
``rope``       rotary pairs applied to the q/k columns, then bf16
``gate_res``   ``out = residual + gate[row // rows_per_group] * acc`` (AdaLN-Zero)
=============  ==============================================================
"""
from __future__ import annotations

from typing import Optional

import torch

from ._ext import ext

EPI = {
    "bf16": 0,
    "f32": 1,
    "f32_acc": 2,
    "swiglu": 3,
    "dswiglu": 4,
    "rope": 5,
    "gate_res": 6,
    "gelu": 7,
}


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: Optional[torch.Tensor] = None,
    *,
    epi: str = "bf16",
    a_t: bool = False,
    b_t: bool = False,
    residual: Optional[torch.Tensor] = None,
    bias: Optional[torch.Tensor] = None,
    out2: Optional[torch.Tensor] = None,
    rope_tab: Optional[torch.Tensor] = None,
    rope_cols: int = 0,
    rope_rows_per_seq: int = 1,
    rope_pos_offset: int = 0,
    rope_head_dim: int = 64,
    gate: Optional[torch.Tensor] = None,
    gate_rows_per_group: int = 1,
    splits: int = 0,
    bn: int = 0,
    gather=None,
) -> torch.Tensor:
    """``gather``: a :class:`WeightGather` handle when ``b`` is a sharded weight whose
    peer-owned pieces this GEMM all-gathers into the local buffer before using them
    (FSDP all-gather fused with the consuming GEMM)."""
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[1] if b_t else b.shape[0]
    if out is None:
        if epi in ("f32", "f32_acc"):
            out = (torch.zeros if epi == "f32_acc" else torch.empty)(
                M, N, device=a.device, dtype=torch.float32
            )
        elif epi == "dswiglu":
            out = torch.empty(M, 2 * N, device=a.device, dtype=torch.bfloat16)
        else:
            out = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
    if epi == "swiglu" and out2 is None:
        out2 = torch.empty(M, N // 2, device=a.device, dtype=torch.bfloat16)
    if gather is not None:
        g = gather.launch_args(b)
    else:
        g = (None, [], 0, 0, 0, 0)
    ext().gemm(
        a, b, out, EPI[epi], a_t, b_t, residual, bias, out2, rope_tab, rope_cols,
        rope_rows_per_seq, rope_pos_offset, rope_head_dim, gate, gate_rows_per_group,
        splits, bn, *g,
    )
    return out
