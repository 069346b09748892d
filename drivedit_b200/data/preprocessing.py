"""Batch preprocessing stages with the reference's API (``data/preprocessing.py``):
``VideoPreprocessor`` (:14-150), ``LatentPreprocessor`` (:153-275), ``ControlPreprocessor``
(:278-443) and ``DataPreprocessingPipeline`` (:446-508).

Frames ``[B, T, C, H, W]`` / ``[T, C, H, W]``: scaled to [0, 1] when given as 0-255,
resized bilinearly, standardised per channel. Latents: resized, standardised over their
spatial dims per map, optionally clamped; flattened to one token per frame and back.
Controls ``[B, T, C]`` / ``[T, C]``: a centred moving average over time (zero padding at
the ends, as a same-size convolution), then each listed channel mapped from its range to
[-1, 1] and clamped.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

IMAGENET_MEAN = [0.485, 0.456, 0.406]
IMAGENET_STD = [0.229, 0.224, 0.225]


def _channel_view(v: Sequence[float], like: torch.Tensor) -> torch.Tensor:
    """Per-channel values shaped to broadcast over the channel dim (third from last)."""
    t = torch.as_tensor(v, dtype=like.dtype, device=like.device)
    return t.view((1,) * max(like.dim() - 3, 0) + (-1, 1, 1))


def _resize_maps(x: torch.Tensor, size: Tuple[int, int]) -> torch.Tensor:
    """Bilinear resize of the last two dims of a 4-D or 5-D tensor."""
    if x.dim() not in (4, 5):
        raise ValueError(f"Unsupported dimensions: {x.dim()}")
    lead = x.shape[:-3]
    y = F.interpolate(x.reshape(-1, *x.shape[-3:]), size=tuple(size), mode="bilinear", align_corners=False)
    return y.reshape(*lead, *y.shape[1:])


def _stats(x: torch.Tensor) -> Dict[str, Any]:
    xf = x.float()
    return {"mean": float(xf.mean()), "std": float(xf.std()), "min": float(xf.min()),
            "max": float(xf.max()), "shape": list(x.shape)}


class VideoPreprocessor:
    def __init__(self, target_size: Tuple[int, int] = (256, 256), normalize: bool = True,
                 mean: Optional[List[float]] = None, std: Optional[List[float]] = None,
                 dtype: torch.dtype = torch.float32):
        self.target_size = tuple(target_size)
        self.normalize, self.dtype = normalize, dtype
        self.mean = list(mean) if mean is not None else list(IMAGENET_MEAN)
        self.std = list(std) if std is not None else list(IMAGENET_STD)

    def preprocess_batch(self, frames: torch.Tensor) -> torch.Tensor:
        x = frames.to(self.dtype)
        if x.max() > 1.0:
            x = x / 255.0
        if tuple(x.shape[-2:]) != self.target_size:
            x = _resize_maps(x, self.target_size)
        return (x - _channel_view(self.mean, x)) / _channel_view(self.std, x) if self.normalize else x

    __call__ = preprocess_batch

    def denormalize(self, frames: torch.Tensor) -> torch.Tensor:
        if not self.normalize:
            return frames
        return frames * _channel_view(self.std, frames) + _channel_view(self.mean, frames)

    def get_frame_statistics(self, frames: torch.Tensor) -> Dict[str, Any]:
        return _stats(frames)


class LatentPreprocessor:
    def __init__(self, latent_dim: int = 64, spatial_size: Tuple[int, int] = (32, 32),
                 normalize_latents: bool = True, clamp_range: Optional[Tuple[float, float]] = None):
        self.latent_dim, self.spatial_size = latent_dim, tuple(spatial_size)
        self.normalize_latents, self.clamp_range = normalize_latents, clamp_range

    def preprocess_latents(self, latents: torch.Tensor) -> torch.Tensor:
        x = latents
        if tuple(x.shape[-2:]) != self.spatial_size:
            x = _resize_maps(x, self.spatial_size)
        if self.normalize_latents:
            m = x.mean((-2, -1), keepdim=True)
            s = x.std((-2, -1), keepdim=True).clamp_min(1e-8)
            x = (x - m) / s
        if self.clamp_range is not None:
            x = x.clamp(*self.clamp_range)
        return x

    __call__ = preprocess_latents

    def tokenize_latents(self, latents: torch.Tensor) -> torch.Tensor:
        """``[B, T, C, H, W]`` -> ``[B, T, C*H*W]`` (``[B, C, H, W]`` -> ``[B, C*H*W]``)."""
        if latents.dim() not in (4, 5):
            raise ValueError(f"Unsupported latent dimensions: {latents.dim()}")
        return latents.flatten(-3)

    def detokenize_latents(self, tokens: torch.Tensor) -> torch.Tensor:
        if tokens.dim() not in (2, 3):
            raise ValueError(f"Unsupported token dimensions: {tokens.dim()}")
        return tokens.unflatten(-1, (self.latent_dim, *self.spatial_size))

    def compute_latent_statistics(self, latents: torch.Tensor) -> Dict[str, Any]:
        return _stats(latents)


class ControlPreprocessor:
    DEFAULT_RANGES = {0: (-1.0, 1.0), 1: (-1.0, 1.0), 2: (-10.0, 10.0), 3: (-10.0, 10.0)}

    def __init__(self, control_dim: int = 4, normalize_controls: bool = True,
                 control_ranges: Optional[Dict[int, Tuple[float, float]]] = None,
                 smooth_controls: bool = True, smooth_window: int = 3):
        """Default ranges: steering and acceleration in [-1, 1], goal x / y in [-10, 10]."""
        self.control_dim, self.normalize_controls = control_dim, normalize_controls
        self.smooth_controls, self.smooth_window = smooth_controls, smooth_window
        self.control_ranges = dict(control_ranges) if control_ranges is not None else dict(self.DEFAULT_RANGES)

    def preprocess_controls(self, controls: torch.Tensor) -> torch.Tensor:
        x = controls
        if self.smooth_controls:
            x = self._smooth_controls(x)
        if self.normalize_controls:
            x = self._normalize_controls(x)
        return x

    __call__ = preprocess_controls

    def _smooth_controls(self, controls: torch.Tensor) -> torch.Tensor:
        k = self.smooth_window
        if k <= 1:
            return controls
        if controls.dim() not in (2, 3):
            raise ValueError(f"Unsupported control dimensions: {controls.dim()}")
        x = controls if controls.dim() == 3 else controls[None]
        B, T, C = x.shape
        w = torch.full((C, 1, k), 1.0 / k, dtype=x.dtype, device=x.device)
        y = F.conv1d(x.transpose(1, 2), w, padding=k // 2, groups=C)[..., :T].transpose(1, 2)
        return y if controls.dim() == 3 else y[0]

    def _normalize_controls(self, controls: torch.Tensor) -> torch.Tensor:
        out = controls.clone()
        for c, (lo, hi) in self.control_ranges.items():
            if c < controls.shape[-1]:
                out[..., c] = (2 * (controls[..., c] - lo) / (hi - lo) - 1).clamp(-1.0, 1.0)
        return out

    def denormalize_controls(self, controls: torch.Tensor) -> torch.Tensor:
        if not self.normalize_controls:
            return controls
        out = controls.clone()
        for c, (lo, hi) in self.control_ranges.items():
            if c < controls.shape[-1]:
                out[..., c] = (controls[..., c] + 1) * (hi - lo) / 2 + lo
        return out

    def compute_control_statistics(self, controls: torch.Tensor) -> Dict[str, Any]:
        return {f"dim_{c}": {k: v for k, v in _stats(controls[..., c]).items() if k != "shape"}
                for c in range(controls.shape[-1])}

    def interpolate_controls(self, controls: torch.Tensor, target_length: int) -> torch.Tensor:
        """Linear resampling of ``[B, T, C]`` / ``[T, C]`` to ``target_length`` steps (sample
        centres aligned, as bilinear interpolation without corner alignment)."""
        x = controls if controls.dim() == 3 else controls[None]
        y = F.interpolate(x.transpose(1, 2), size=target_length, mode="linear", align_corners=False)
        y = y.transpose(1, 2)
        return y if controls.dim() == 3 else y[0]

    def add_control_noise(self, controls: torch.Tensor, noise_std: float = 0.01) -> torch.Tensor:
        return controls + torch.randn_like(controls) * noise_std


class DataPreprocessingPipeline:
    """Applies the three stages to the ``frames``, ``latents`` and ``controls`` of a
    batch (default-configured stages when not given); other keys pass through."""

    def __init__(self, video_preprocessor: Optional[VideoPreprocessor] = None,
                 latent_preprocessor: Optional[LatentPreprocessor] = None,
                 control_preprocessor: Optional[ControlPreprocessor] = None):
        self.video_preprocessor = video_preprocessor or VideoPreprocessor()
        self.latent_preprocessor = latent_preprocessor or LatentPreprocessor()
        self.control_preprocessor = control_preprocessor or ControlPreprocessor()

    def __call__(self, batch: Dict[str, Any]) -> Dict[str, Any]:
        stages = {"frames": self.video_preprocessor.preprocess_batch,
                  "latents": self.latent_preprocessor.preprocess_latents,
                  "controls": self.control_preprocessor.preprocess_controls}
        return {k: stages[k](v) if k in stages else v for k, v in batch.items()}

    def get_preprocessor_configs(self) -> Dict[str, Dict[str, Any]]:
        v, l, c = self.video_preprocessor, self.latent_preprocessor, self.control_preprocessor
        return {"video": {"target_size": v.target_size, "normalize": v.normalize, "mean": v.mean, "std": v.std},
                "latent": {"latent_dim": l.latent_dim, "spatial_size": l.spatial_size,
                           "normalize_latents": l.normalize_latents},
                "control": {"control_dim": c.control_dim, "normalize_controls": c.normalize_controls,
                            "control_ranges": c.control_ranges}}
