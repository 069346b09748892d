"""Attention entry points of the fused block path.

``attention_fwd(qkv, bc)`` takes the ``[M, 3d]`` output of the QKV GEMM (q, k already
rotated) and returns ``(o [M, d] bf16, o_lin or None, lse, aux)``;
``attention_bwd`` returns ``dqkv [M, 3d]`` (q/k gradients still in the rotated frame).

Modes: ``dense`` (frame-causal / token-causal / bidirectional softmax attention) and
``sla`` (top-k block routing, block-sparse softmax, linear branch).

CUDA tensors always run the sm_100a kernels; a missing or incomplete extension raises
instead of falling back. CPU tensors run the PyTorch reference (dense only), which is
what the CPU tests and the CPU oracles use.
"""
from __future__ import annotations

import torch

from ._ext import ext


def _kernels(t: torch.Tensor) -> bool:
    """True for CUDA tensors; raises when the extension lacks the attention kernels."""
    if not t.is_cuda:
        return False
    if getattr(ext(), "attn_fwd", None) is None:
        raise RuntimeError("the drivedit_b200 extension was built without the attention "
                           "kernels; rebuild it with `python setup.py build_ext --inplace`")
    return True


def _split(qkv, bc):
    B, T, H, Dh = bc.B, bc.T, bc.H, bc.Dh
    q, k, v = qkv.view(B, T, 3, H, Dh).unbind(2)
    return q, k, v


def _torch_dense(q, k, v, bc):
    from ..layers.attention import frame_causal_mask

    T = q.shape[1]
    if bc.causal == "frame":
        mask = frame_causal_mask(T, bc.tpf, device=q.device)
    elif bc.causal == "token":
        mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=q.device))[None, None]
    else:
        mask = None
    o = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), attn_mask=mask)
    return o.transpose(1, 2)


def attention_fwd(qkv: torch.Tensor, bc):
    if _kernels(qkv):
        from .attention_kernels import attention_fwd_kernel

        return attention_fwd_kernel(qkv, bc)
    if bc.attn_mode != "dense":
        raise RuntimeError("SLA attention on the fused block path needs CUDA tensors")
    q, k, v = _split(qkv, bc)
    o = _torch_dense(q, k, v, bc)
    return o.reshape(qkv.shape[0], -1).contiguous(), None, None, None


def attention_bwd(qkv, o, lse, do, do_lin, aux, bc):
    if _kernels(qkv):
        from .attention_kernels import attention_bwd_kernel

        return attention_bwd_kernel(qkv, o, lse, do, do_lin, aux, bc)
    q, k, v = (t.detach().requires_grad_(True) for t in _split(qkv, bc))
    with torch.enable_grad():
        out = _torch_dense(q, k, v, bc)
        gq, gk, gv = torch.autograd.grad(out, (q, k, v), do.view_as(out))
    return torch.stack([gq, gk, gv], 2).reshape(qkv.shape).contiguous()
