"""Offline / online preprocessing stages.

API of the reference ``data/preprocessing.py``: ``VideoPreprocessor`` (resize, centre
crop, normalise, fixed clip length, :14-150), ``LatentPreprocessor`` (VAE encoding with
a scale factor, patch tokenisation, :153-275), ``ControlPreprocessor`` (clipping,
normalisation, smoothing, derivatives, :278-443) and ``DataPreprocessingPipeline``
(:446-508).
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .transforms import FrameTransforms


class VideoPreprocessor:
    def __init__(self, image_size: Tuple[int, int] = (256, 256), sequence_length: Optional[int] = None,
                 normalize: bool = False, center_crop: bool = False):
        self.image_size, self.sequence_length = tuple(image_size), sequence_length
        self.normalize, self.center_crop = normalize, center_crop

    def __call__(self, video: torch.Tensor) -> torch.Tensor:
        """``[T, C, H, W]`` (float in [0,1] or uint8) -> ``[T', C, h, w]`` float."""
        v = video.float() / 255.0 if video.dtype == torch.uint8 else video.float()
        if self.center_crop:
            H, W = v.shape[-2:]
            ar = self.image_size[1] / self.image_size[0]
            h, w = (H, int(H * ar)) if W / H > ar else (int(W / ar), W)
            v = FrameTransforms.center_crop(v, (h, w))
        if tuple(v.shape[-2:]) != self.image_size:
            v = F.interpolate(v, size=self.image_size, mode="bilinear", align_corners=False)
        if self.sequence_length is not None:
            T = v.shape[0]
            if T >= self.sequence_length:
                v = v[:self.sequence_length]
            else:
                v = torch.cat([v, v[-1:].expand(self.sequence_length - T, -1, -1, -1)], 0)
        return FrameTransforms.normalize(v) if self.normalize else v


class LatentPreprocessor:
    """Frames -> VAE latents (mean, times ``scale_factor``) -> optional patch tokens."""

    def __init__(self, vae=None, scale_factor: float = 1.0, patch_size: int = 2):
        self.vae, self.scale_factor, self.patch_size = vae, scale_factor, patch_size

    @torch.no_grad()
    def encode(self, frames: torch.Tensor) -> torch.Tensor:
        """``[B, T, 3, H, W]`` in [0,1] -> ``[B, T', C, h, w]``."""
        if self.vae is None:
            raise ValueError("LatentPreprocessor needs a VAE to encode")
        x = frames.transpose(1, 2) * 2 - 1
        mean, _ = self.vae.encode(x)
        return (mean * self.scale_factor).transpose(1, 2)

    @torch.no_grad()
    def decode(self, latents: torch.Tensor) -> torch.Tensor:
        x = self.vae.decode((latents / self.scale_factor).transpose(1, 2))
        return ((x.float() + 1) / 2).clamp(0, 1).transpose(1, 2)

    def tokenize(self, latents: torch.Tensor) -> torch.Tensor:
        from ..models.world_dit import patchify

        return patchify(latents, self.patch_size)

    def detokenize(self, tokens: torch.Tensor, frames: int, C: int, H: int, W: int) -> torch.Tensor:
        from ..models.world_dit import unpatchify

        return unpatchify(tokens, frames, C, H, W, self.patch_size)


class ControlPreprocessor:
    def __init__(self, ranges: Optional[Sequence[Tuple[float, float]]] = None, smooth_window: int = 1,
                 add_derivatives: bool = False, fps: float = 10.0):
        self.ranges, self.smooth_window = ranges, smooth_window
        self.add_derivatives, self.fps = add_derivatives, fps

    def normalize(self, controls: torch.Tensor) -> torch.Tensor:
        if self.ranges is None:
            return controls
        lo = torch.tensor([r[0] for r in self.ranges], dtype=controls.dtype, device=controls.device)
        hi = torch.tensor([r[1] for r in self.ranges], dtype=controls.dtype, device=controls.device)
        return 2 * (torch.maximum(torch.minimum(controls, hi), lo) - lo) / (hi - lo + 1e-8) - 1

    def smooth(self, controls: torch.Tensor) -> torch.Tensor:
        k = self.smooth_window
        if k <= 1:
            return controls
        x = controls.transpose(-1, -2).reshape(-1, 1, controls.shape[-2])
        y = F.avg_pool1d(F.pad(x, (k // 2, (k - 1) // 2), mode="replicate"), k, 1)
        return y.reshape(*controls.shape[:-2], controls.shape[-1], -1).transpose(-1, -2)

    def derivatives(self, controls: torch.Tensor) -> torch.Tensor:
        d = torch.zeros_like(controls)
        d[..., 1:, :] = (controls[..., 1:, :] - controls[..., :-1, :]) * self.fps
        return d

    def __call__(self, controls: torch.Tensor) -> torch.Tensor:
        c = self.smooth(self.normalize(controls.float()))
        return torch.cat([c, self.derivatives(c)], -1) if self.add_derivatives else c


class DataPreprocessingPipeline:
    def __init__(self, video: Optional[VideoPreprocessor] = None, controls: Optional[ControlPreprocessor] = None,
                 latents: Optional[LatentPreprocessor] = None):
        self.video, self.controls, self.latents = video, controls, latents

    def __call__(self, sample: Dict[str, Any]) -> Dict[str, Any]:
        out = dict(sample)
        if self.video is not None and "frames" in out:
            out["frames"] = self.video(out["frames"])
        if self.controls is not None and "controls" in out:
            out["controls"] = self.controls(out["controls"])
        if self.latents is not None and self.latents.vae is not None and "frames" in out:
            out["latents"] = self.latents.encode(out["frames"][None])[0]
        return out
