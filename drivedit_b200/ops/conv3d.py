"""Video-VAE convolutions and GroupNorm on the hand-written sm_100a kernels.

``causal_conv3d`` computes the reference ``CausalConv3d`` (front temporal padding
``kt - 1``, symmetric spatial padding ``k // 2``; reference models/vae3d.py:119-173)
on channels-last activations with ``csrc/vae/conv3d.cu``:

* stride 1: one implicit-GEMM launch; padding is the TMA unit's zero fill;
* stride s > 1 (``Downsample3D``): the input is rearranged space-to-depth (each
  s-block of a strided dimension becomes channels) and the weights are re-indexed so the
  same stride-1 kernel computes the strided convolution exactly;
* backward: ``dx`` is the stride-1 kernel again on ``dy`` with flipped, transposed
  weights and mirrored padding; ``dw`` is the weight-gradient mode of the same kernel
  (K = output positions), accumulated in fp32.

``group_norm_silu`` is ``csrc/vae/groupnorm.cu`` (GroupNorm, optionally followed by
SiLU) with its own backward. Tensors keep the reference's logical ``[B, C, T, H, W]``
shape; on the GPU they are stored channels-last (``torch.channels_last_3d``) so every
kernel reads them without a copy.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from ._ext import ext


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def to_cl(x: torch.Tensor) -> torch.Tensor:
    """``[B, C, T, H, W]`` -> contiguous channels-last ``[B, T, H, W, C]`` bf16."""
    return x.to(torch.bfloat16).permute(0, 2, 3, 4, 1).contiguous()


def from_cl(y: torch.Tensor) -> torch.Tensor:
    """``[B, T, H, W, C]`` -> a ``[B, C, T, H, W]`` view (channels_last_3d strides)."""
    return y.permute(0, 4, 1, 2, 3)


def _pad_channels(x_cl: torch.Tensor, c: int) -> torch.Tensor:
    if x_cl.shape[-1] == c:
        return x_cl
    return torch.nn.functional.pad(x_cl, (0, c - x_cl.shape[-1]))


def _kernel_weight(w: torch.Tensor, cin_pad: int, cout_pad: int) -> torch.Tensor:
    """``[Cout, Cin, kt, kh, kw]`` -> bf16 ``[Cout_pad, kt*kh*kw*Cin_pad]`` (tap-major)."""
    Cout, Cin = w.shape[:2]
    wk = w.permute(0, 2, 3, 4, 1)
    wk = torch.nn.functional.pad(wk, (0, cin_pad - Cin))
    wk = wk.reshape(Cout, -1)
    if cout_pad != Cout:
        wk = torch.nn.functional.pad(wk, (0, 0, 0, cout_pad - Cout))
    return wk.to(torch.bfloat16).contiguous()


class _Conv3dFn(torch.autograd.Function):
    """Stride-1 conv on channels-last ``x [B,T,H,W,Cin_pad]`` with explicit output
    extents; input coordinate = output coordinate + tap - pad."""

    @staticmethod
    def forward(ctx, x_cl, w, bias, residual, ksize, pads, out_thw):
        kt, kh, kw = ksize
        pt, ph, pw = pads
        Cout, Cin = w.shape[:2]
        cin_pad = x_cl.shape[-1]
        wk = _kernel_weight(w.detach(), cin_pad, Cout)
        B = x_cl.shape[0]
        To, Ho, Wo = out_thw
        y = torch.empty(B, To, Ho, Wo, Cout, device=x_cl.device, dtype=torch.bfloat16)
        b32 = None if bias is None else bias.detach().float().contiguous()
        res = None if residual is None else residual.contiguous()
        ext().conv3d_fwd(x_cl, wk, y, kt, kh, kw, pt, ph, pw, b32, res)
        ctx.save_for_backward(x_cl, wk)
        ctx.meta = (ksize, pads, Cout, Cin, w.dtype, bias is not None and bias.requires_grad,
                    residual is not None)
        return y

    @staticmethod
    def backward(ctx, dy):
        x_cl, wk = ctx.saved_tensors
        (kt, kh, kw), (pt, ph, pw), Cout, Cin, wdtype, need_db, has_res = ctx.meta
        dy = dy.to(torch.bfloat16).contiguous()
        B, T, H, W, cin_pad = x_cl.shape
        cout_pad = _round_up(Cout, 128)
        dy_p = _pad_channels(dy, cout_pad)
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            # dx[i] = sum_k dy[i + k - (K-1-p)] * W[K-1-k]^T
            wf = wk.view(Cout, kt, kh, kw, cin_pad).flip(1, 2, 3).permute(4, 1, 2, 3, 0)
            wf = torch.nn.functional.pad(wf, (0, cout_pad - Cout)).reshape(cin_pad, -1).contiguous()
            dx = torch.empty_like(x_cl)
            ext().conv3d_fwd(dy_p, wf, dx, kt, kh, kw, kt - 1 - pt, kh - 1 - ph, kw - 1 - pw,
                             None, None)
        if ctx.needs_input_grad[1]:
            acc = torch.zeros(cout_pad, kt * kh * kw * cin_pad, device=dy.device,
                              dtype=torch.float32)
            ext().conv3d_wgrad(x_cl, dy_p, acc, kt, kh, kw, pt, ph, pw, 0)
            dw = acc[:Cout].view(Cout, kt, kh, kw, cin_pad)[..., :Cin].permute(0, 4, 1, 2, 3)
            dw = dw.to(wdtype)
        if need_db:
            db = dy.float().sum((0, 1, 2, 3))
        dres = dy if has_res else None
        return dx, dw, db, dres, None, None, None


def _s2d_index(k: int, s: int, p: int) -> Tuple[torch.Tensor, int, int]:
    """Re-index one dimension of a stride-``s`` kernel for a space-to-depth input.

    Output ``o`` reads original index ``o*s + k - p``; in blocks of ``s`` that is block
    ``o + q`` at phase ``r`` with ``k = q*s + r + p``. Returns an index table
    ``[s, K']`` into the kernel dimension (``k`` = K for a zero tap), ``K'`` and the new
    front padding ``p' = -q_min``."""
    qmin = (-p) // s
    qmax = (k - 1 - p) // s
    kn = qmax - qmin + 1
    idx = torch.full((s, kn), k, dtype=torch.long)
    for r in range(s):
        for qi in range(kn):
            kk = (qi + qmin) * s + r + p
            if 0 <= kk < k:
                idx[r, qi] = kk
    return idx, kn, -qmin


def s2d_weight(w: torch.Tensor, stride: Sequence[int], pads: Sequence[int]):
    """Weights of a strided conv -> weights of the equivalent stride-1 conv on the
    space-to-depth input (channel order (rt, rh, rw, c)). Differentiable in ``w``."""
    Cout, Cin, kt, kh, kw = w.shape
    wp = torch.nn.functional.pad(w, (0, 1, 0, 1, 0, 1))  # index k -> zero tap
    ks, news = [], []
    for d, (k, s, p) in enumerate(zip((kt, kh, kw), stride, pads)):
        idx, kn, pn = _s2d_index(k, s, p)
        wp = wp.index_select(2 + d, idx.flatten().to(w.device))  # (r, q') pairs, r-major
        ks.append((s, kn))
        news.append(pn)
    st, sh, sw = stride
    (_, knt), (_, knh), (_, knw) = ks
    wp = wp.view(Cout, Cin, st, knt, sh, knh, sw, knw)
    # -> [Cout, (rt, rh, rw, c), K't, K'h, K'w]
    wp = wp.permute(0, 2, 4, 6, 1, 3, 5, 7).reshape(Cout, st * sh * sw * Cin, knt, knh, knw)
    return wp, (knt, knh, knw), tuple(news)


def space_to_depth(x_cl: torch.Tensor, stride: Sequence[int]) -> torch.Tensor:
    """``[B, T, H, W, C]`` -> ``[B, T/st, H/sh, W/sw, st*sh*sw*C]`` (zero-padding the end
    of each strided dimension to a multiple of its stride)."""
    st, sh, sw = stride
    B, T, H, W, C = x_cl.shape
    Tp, Hp, Wp = _round_up(T, st), _round_up(H, sh), _round_up(W, sw)
    if (Tp, Hp, Wp) != (T, H, W):
        x_cl = torch.nn.functional.pad(x_cl, (0, 0, 0, Wp - W, 0, Hp - H, 0, Tp - T))
    x = x_cl.view(B, Tp // st, st, Hp // sh, sh, Wp // sw, sw, C)
    return x.permute(0, 1, 3, 5, 2, 4, 6, 7).reshape(B, Tp // st, Hp // sh, Wp // sw,
                                                      st * sh * sw * C)


def conv_stride1_reference(x_cl: torch.Tensor, w: torch.Tensor, pads: Sequence[int],
                           out_thw: Sequence[int]) -> torch.Tensor:
    """PyTorch statement of what one ``conv3d_fwd`` launch computes (fp32): channels-last
    ``x``, input coordinate = output coordinate + tap - pad, zero outside the input."""
    B, T, H, W, C = x_cl.shape
    Cout, Cin, kt, kh, kw = w.shape
    To, Ho, Wo = out_thw
    pt, ph, pw = pads
    x = x_cl.permute(0, 4, 1, 2, 3).float()[:, :Cin]
    # pad front by `pad` and back so that every read index exists
    x = torch.nn.functional.pad(x, (pw, max(0, Wo + kw - 1 - pw - W), ph,
                                    max(0, Ho + kh - 1 - ph - H), pt,
                                    max(0, To + kt - 1 - pt - T)))
    y = torch.nn.functional.conv3d(x, w.float())
    return y[:, :, :To, :Ho, :Wo].permute(0, 2, 3, 4, 1)


def causal_conv3d(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                  stride: Sequence[int] = (1, 1, 1), temporal_pad: Optional[int] = None,
                  residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x [B, Cin, T, H, W]`` -> ``[B, Cout, To, Ho, Wo]`` (channels-last storage).

    Same output as ``F.conv3d(F.pad(x, (0,0,0,0,tp,0)), weight, bias, stride,
    padding=(0, kh//2, kw//2))`` with ``tp = kt - 1`` unless ``temporal_pad`` says
    otherwise; ``residual`` (output-shaped) is added in the epilogue."""
    Cout, Cin, kt, kh, kw = weight.shape
    st, sh, sw = stride
    tp = kt - 1 if temporal_pad is None else temporal_pad
    pads = (tp, kh // 2, kw // 2)
    B, _, T, H, W = x.shape
    To = (T + tp - kt) // st + 1
    Ho = (H + 2 * pads[1] - kh) // sh + 1
    Wo = (W + 2 * pads[2] - kw) // sw + 1
    x_cl = to_cl(x)
    if (st, sh, sw) != (1, 1, 1):
        w2, ks, pads = s2d_weight(weight, (st, sh, sw), pads)
        x_cl = space_to_depth(x_cl, (st, sh, sw))
    else:
        w2, ks = weight, (kt, kh, kw)
    x_cl = _pad_channels(x_cl, _round_up(x_cl.shape[-1], 128))
    res_cl = None if residual is None else to_cl(residual)
    y = _Conv3dFn.apply(x_cl, w2, bias, res_cl, ks, pads, (To, Ho, Wo))
    return from_cl(y)


class _GroupNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_cl3, weight, bias, groups, eps, silu):
        w32 = weight.detach().float().contiguous()
        b32 = None if bias is None else bias.detach().float().contiguous()
        y, stats = ext().groupnorm_fwd(x_cl3, w32, b32, groups, eps, silu)
        ctx.save_for_backward(x_cl3, w32, stats)
        ctx.b32 = b32
        ctx.silu = silu
        ctx.dtypes = (weight.dtype, None if bias is None else bias.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w32, stats = ctx.saved_tensors
        dx, acc = ext().groupnorm_bwd(dy.to(torch.bfloat16).contiguous(), x, w32, ctx.b32, stats,
                                      ctx.silu)
        dw = acc[..., 1].sum(0).to(ctx.dtypes[0])
        db = None if ctx.dtypes[1] is None else acc[..., 0].sum(0).to(ctx.dtypes[1])
        return dx, dw, db, None, None, None


def group_norm_silu(x: torch.Tensor, groups: int, weight: torch.Tensor,
                    bias: Optional[torch.Tensor], eps: float = 1e-5, silu: bool = True):
    """``silu(GroupNorm(x))`` (or plain GroupNorm) for ``x [B, C, T, H, W]``."""
    B, C = x.shape[:2]
    x_cl = to_cl(x)
    shp = x_cl.shape
    y = _GroupNormFn.apply(x_cl.view(B, -1, C), weight, bias, groups, eps, silu)
    return from_cl(y.view(shp))
