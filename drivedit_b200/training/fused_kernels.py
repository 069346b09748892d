"""The reference's training-side fused kernels API (training/kernels/fused_normalize.py:
194-360, training/kernels/fused_augment.py:199-470) on this framework's CUDA kernels.

* Normalisation: :func:`fused_normalize_kernel` / :class:`FusedNormalizeFunction`
  (LayerNorm without affine parameters), :class:`FusedNormalize` (optional affine) and
  :class:`FusedRMSNorm`. On CUDA tensors whose width is a multiple of 256 they run on the
  LayerNorm kernel (``csrc/fused/layernorm.cu``, bf16 out, fp32 statistics,
  differentiable); otherwise PyTorch's ``layer_norm``.
* Augmentation: :func:`fused_augment_kernel`, :class:`FusedAugmentation`,
  :class:`VideoAugmentation`: per-sample horizontal flip, brightness shift and contrast
  around 0.5, clamped to [0, 1], optional per-channel standardisation; one pass of the
  clip-augmentation kernel (``csrc/fused/augment.cu``) on CUDA, its PyTorch statement
  (:func:`drivedit_b200.data.transforms.clip_augment_reference`) on the CPU. A video gets
  the same parameters on every frame.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..data.transforms import clip_augment_reference
from ..layers.fused_ops import FusedRMSNorm  # noqa: F401  (also exported here by the reference)


def _kernel_ok(x: torch.Tensor) -> bool:
    return x.is_cuda and x.shape[-1] % 256 == 0


class FusedNormalizeFunction(torch.autograd.Function):
    """LayerNorm without affine parameters, differentiable (CUDA kernel when the width is
    a multiple of 256)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
        from ..ops.fused import layer_norm

        with torch.enable_grad():
            xi = x.detach().requires_grad_(True)
            y = layer_norm(xi, None, None, eps) if _kernel_ok(x) else F.layer_norm(xi, (x.shape[-1],), eps=eps)
        ctx.save_for_backward(xi, y)
        return y.detach().to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        xi, y = ctx.saved_tensors
        (dx,) = torch.autograd.grad(y, xi, dy.to(y.dtype))
        return dx, None


def fused_normalize_kernel(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    if _kernel_ok(x):
        from ..ops.fused import layer_norm

        return layer_norm(x, None, None, eps).to(x.dtype)
    return F.layer_norm(x, (x.shape[-1],), eps=eps)


class FusedNormalize(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5, affine: bool = True):
        super().__init__()
        self.dim, self.eps, self.affine = dim, eps, affine
        if affine:
            self.weight = nn.Parameter(torch.ones(dim))
            self.bias = nn.Parameter(torch.zeros(dim))
        else:
            self.register_parameter("weight", None)
            self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _kernel_ok(x):
            from ..ops.fused import layer_norm

            return layer_norm(x, self.weight, self.bias, self.eps).to(x.dtype)
        return F.layer_norm(x, (self.dim,), self.weight, self.bias, self.eps)


def fused_augment_kernel(x: torch.Tensor, flip_flags: torch.Tensor, brightness: torch.Tensor,
                         contrast: torch.Tensor) -> torch.Tensor:
    """``x [B, C, H, W]`` in [0, 1]; per-sample ``flip_flags`` (bool), ``brightness``
    (added) and ``contrast`` (scaled around 0.5)."""
    v = x[:, None]
    if x.is_cuda:
        from ..data.transforms import AugmentationPipeline

        y = AugmentationPipeline.fused_clip_augment(v.float(), flip_flags, brightness, contrast)
    else:
        y = clip_augment_reference(v.float(), flip_flags, brightness, contrast)
    return y[:, 0].to(x.dtype)


class FusedAugmentation(nn.Module):
    def __init__(self, flip_prob: float = 0.5, brightness_range: Tuple[float, float] = (-0.1, 0.1),
                 contrast_range: Tuple[float, float] = (0.9, 1.1), normalize: bool = False,
                 mean: Sequence[float] = (0.485, 0.456, 0.406),
                 std: Sequence[float] = (0.229, 0.224, 0.225)):
        super().__init__()
        self.flip_prob = flip_prob
        self.brightness_range = tuple(brightness_range)
        self.contrast_range = tuple(contrast_range)
        self.normalize = normalize
        self.register_buffer("mean", torch.tensor(mean).view(1, -1, 1, 1))
        self.register_buffer("std", torch.tensor(std).view(1, -1, 1, 1))

    def _sample_params(self, n: int, device, deterministic: bool = False):
        if deterministic:
            return (torch.zeros(n, dtype=torch.bool, device=device),
                    torch.zeros(n, device=device), torch.ones(n, device=device))
        lo_b, hi_b = self.brightness_range
        lo_c, hi_c = self.contrast_range
        return (torch.rand(n, device=device) < self.flip_prob,
                torch.rand(n, device=device) * (hi_b - lo_b) + lo_b,
                torch.rand(n, device=device) * (hi_c - lo_c) + lo_c)

    def forward(self, x: torch.Tensor, deterministic: bool = False,
                flip_override: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``x [B, C, H, W]`` or a video ``[B, T, C, H, W]`` (one parameter set per clip)."""
        video = x.dim() == 5
        v = x if video else x[:, None]
        flip, bright, contr = self._sample_params(v.shape[0], x.device, deterministic)
        if flip_override is not None:
            flip = flip_override.to(x.device).bool()
        mean = self.mean.flatten().tolist() if self.normalize else None
        std = self.std.flatten().tolist() if self.normalize else None
        if x.is_cuda:
            from ..data.transforms import AugmentationPipeline

            y = AugmentationPipeline.fused_clip_augment(v.float().contiguous(), flip, bright, contr,
                                                        mean, std)
        else:
            y = clip_augment_reference(v.float(), flip, bright, contr, mean, std)
        y = y.to(x.dtype)
        return y if video else y[:, 0]


class VideoAugmentation(nn.Module):
    """:class:`FusedAugmentation` of clips ``[B, T, C, H, W]`` plus, with probability
    ``color_jitter_prob`` per call, a per-clip per-channel gain in ``color_range``
    (the same on every frame), clamped to [0, 1]."""

    def __init__(self, flip_prob: float = 0.5, brightness_range: Tuple[float, float] = (-0.1, 0.1),
                 contrast_range: Tuple[float, float] = (0.9, 1.1), color_jitter_prob: float = 0.3,
                 color_range: Tuple[float, float] = (0.9, 1.1)):
        super().__init__()
        self.fused_aug = FusedAugmentation(flip_prob, brightness_range, contrast_range)
        self.color_jitter_prob = color_jitter_prob
        self.color_range = tuple(color_range)

    def forward(self, frames: torch.Tensor, deterministic: bool = False) -> torch.Tensor:
        B, T, C = frames.shape[:3]
        flip = (torch.zeros(B, dtype=torch.bool, device=frames.device) if deterministic
                else torch.rand(B, device=frames.device) < self.fused_aug.flip_prob)
        out = self.fused_aug(frames, deterministic=deterministic, flip_override=flip)
        if not deterministic and self.color_jitter_prob > 0 and float(torch.rand(())) < self.color_jitter_prob:
            lo, hi = self.color_range
            gain = torch.rand(B, 1, C, 1, 1, device=frames.device) * (hi - lo) + lo
            out = (out * gain).clamp(0, 1)
        return out
