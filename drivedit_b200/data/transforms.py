"""Frame / video transforms and the training augmentation pipeline.

API of the reference ``data/transforms.py`` (``FrameTransforms`` :15-198,
``VideoTransforms`` :201-275, ``AugmentationPipeline`` :278-423). Frames are
``[..., C, H, W]`` floats in [0, 1]. ``AugmentationPipeline.fused_clip_augment`` applies
per-clip flip + brightness/contrast + normalisation to a whole batch in one sm_100a
kernel (csrc/fused/augment.cu; uint8 HWC input supported) with the same arithmetic as
``clip_augment_reference``.
"""
from __future__ import annotations

import math
import random
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

IMAGENET_MEAN = [0.485, 0.456, 0.406]
IMAGENET_STD = [0.229, 0.224, 0.225]


def _cview(v, x):
    return torch.tensor(v, dtype=x.dtype, device=x.device).view(-1, 1, 1)


class FrameTransforms:
    @staticmethod
    def normalize(frame, mean=None, std=None):
        return (frame - _cview(mean or IMAGENET_MEAN, frame)) / _cview(std or IMAGENET_STD, frame)

    @staticmethod
    def denormalize(frame, mean=None, std=None):
        return frame * _cview(std or IMAGENET_STD, frame) + _cview(mean or IMAGENET_MEAN, frame)

    @staticmethod
    def resize(frame, size: Tuple[int, int], mode: str = "bilinear"):
        x = frame if frame.dim() == 4 else frame[None]
        y = F.interpolate(x, size=size, mode=mode, align_corners=False if mode in ("bilinear", "bicubic") else None)
        return y if frame.dim() == 4 else y[0]

    @staticmethod
    def crop(frame, top: int, left: int, height: int, width: int):
        return frame[..., top:top + height, left:left + width]

    @staticmethod
    def center_crop(frame, size):
        H, W = frame.shape[-2:]
        h, w = size
        return FrameTransforms.crop(frame, (H - h) // 2, (W - w) // 2, h, w)

    @staticmethod
    def random_crop(frame, size):
        H, W = frame.shape[-2:]
        h, w = size
        return FrameTransforms.crop(frame, random.randint(0, max(0, H - h)), random.randint(0, max(0, W - w)), h, w)

    @staticmethod
    def horizontal_flip(frame):
        return frame.flip(-1)

    @staticmethod
    def vertical_flip(frame):
        return frame.flip(-2)

    @staticmethod
    def rotate(frame, angle: float, mode: str = "bilinear"):
        x = frame if frame.dim() == 4 else frame[None]
        a = math.radians(angle)
        theta = torch.tensor([[math.cos(a), -math.sin(a), 0.0], [math.sin(a), math.cos(a), 0.0]],
                             dtype=x.dtype, device=x.device)[None].expand(x.shape[0], 2, 3)
        grid = F.affine_grid(theta, list(x.shape), align_corners=False)
        y = F.grid_sample(x, grid, mode=mode, padding_mode="zeros", align_corners=False)
        return y if frame.dim() == 4 else y[0]

    @staticmethod
    def brightness(frame, factor: float):
        return (frame * factor).clamp(0, 1)

    @staticmethod
    def contrast(frame, factor: float):
        m = frame.mean(dim=(-3, -2, -1), keepdim=True)
        return ((frame - m) * factor + m).clamp(0, 1)

    @staticmethod
    def saturation(frame, factor: float):
        gray = (0.299 * frame[..., 0:1, :, :] + 0.587 * frame[..., 1:2, :, :] + 0.114 * frame[..., 2:3, :, :])
        return ((frame - gray) * factor + gray).clamp(0, 1)

    @staticmethod
    def hue(frame, factor: float):
        """Rotate hue by ``factor`` turns (YIQ rotation)."""
        a = 2 * math.pi * factor
        c, s = math.cos(a), math.sin(a)
        T = torch.tensor([[0.299, 0.587, 0.114], [0.596, -0.274, -0.322], [0.211, -0.523, 0.312]],
                         dtype=frame.dtype, device=frame.device)
        R = torch.tensor([[1, 0, 0], [0, c, -s], [0, s, c]], dtype=frame.dtype, device=frame.device)
        M = torch.linalg.inv(T) @ R @ T
        y = torch.einsum("ij,...jhw->...ihw", M, frame)
        return y.clamp(0, 1)

    @staticmethod
    def gaussian_noise(frame, std: float = 0.01):
        return (frame + torch.randn_like(frame) * std).clamp(0, 1)


class VideoTransforms:
    """Video ``[T, C, H, W]``."""

    @staticmethod
    def temporal_crop(video, length: int, start: Optional[int] = None):
        T = video.shape[0]
        if T <= length:
            return video
        s = random.randint(0, T - length) if start is None else start
        return video[s:s + length]

    @staticmethod
    def temporal_subsample(video, factor: int):
        return video[::factor]

    @staticmethod
    def temporal_flip(video):
        return video.flip(0)

    @staticmethod
    def apply_frame_transform(video, transform_fn: Callable, **kwargs):
        return torch.stack([transform_fn(f, **kwargs) for f in video])

    @staticmethod
    def temporal_jitter(video, max_jitter: int = 2):
        T = video.shape[0]
        idx = torch.clamp(torch.arange(T) + torch.randint(-max_jitter, max_jitter + 1, (T,)), 0, T - 1)
        return video[idx.sort().values]


def clip_augment_reference(x: torch.Tensor, flip: torch.Tensor, brightness: torch.Tensor,
                           contrast: torch.Tensor, mean=None, std=None) -> torch.Tensor:
    """PyTorch statement of the fused kernel: ``x [B, T, C, H, W]`` in [0, 1]."""
    B = x.shape[0]
    y = torch.where(flip.view(B, 1, 1, 1, 1).bool(), x.flip(-1), x)
    y = (contrast.view(B, 1, 1, 1, 1) * (y + brightness.view(B, 1, 1, 1, 1) - 0.5) + 0.5).clamp(0, 1)
    if mean is not None:
        y = (y - torch.tensor(mean, device=x.device).view(1, 1, -1, 1, 1)) / \
            torch.tensor(std, device=x.device).view(1, 1, -1, 1, 1)
    return y


class AugmentationPipeline:
    """List of ``{"name": ..., **params}`` transforms, each applied with probability
    ``p`` (per transform ``prob`` overrides) to a video ``[T, C, H, W]``."""

    def __init__(self, transforms: List[Dict[str, Any]], p: float = 0.5):
        self.transforms, self.p = transforms, p

    def __call__(self, video: torch.Tensor, **kwargs) -> torch.Tensor:
        for t in self.transforms:
            t = dict(t)
            name = t.pop("name")
            prob = t.pop("prob", self.p)
            if random.random() < prob:
                video = self._apply_transform(video, name, t)
        return video

    def _apply_transform(self, video, name, params):
        ft = FrameTransforms
        if name == "horizontal_flip":
            return video.flip(-1)
        if name == "vertical_flip":
            return video.flip(-2)
        if name == "brightness":
            return ft.brightness(video, random.uniform(*params.get("range", (0.9, 1.1))))
        if name == "contrast":
            f = random.uniform(*params.get("range", (0.9, 1.1)))
            return torch.stack([ft.contrast(fr, f) for fr in video])
        if name == "saturation":
            return ft.saturation(video, random.uniform(*params.get("range", (0.9, 1.1))))
        if name == "hue":
            return ft.hue(video, random.uniform(*params.get("range", (-0.05, 0.05))))
        if name == "rotate":
            return ft.rotate(video, random.uniform(*params.get("range", (-5.0, 5.0))))
        if name == "random_crop":
            size = params["size"]
            H, W = video.shape[-2:]
            top, left = random.randint(0, max(0, H - size[0])), random.randint(0, max(0, W - size[1]))
            return video[..., top:top + size[0], left:left + size[1]]
        if name == "center_crop":
            return ft.center_crop(video, params["size"])
        if name == "resize":
            return ft.resize(video, tuple(params["size"]))
        if name == "gaussian_noise":
            return ft.gaussian_noise(video, params.get("std", 0.01))
        if name == "temporal_jitter":
            return VideoTransforms.temporal_jitter(video, params.get("max_jitter", 2))
        if name == "normalize":
            return ft.normalize(video, params.get("mean"), params.get("std"))
        raise ValueError(f"unknown transform {name!r}")

    @staticmethod
    def fused_clip_augment(x: torch.Tensor, flip: torch.Tensor, brightness: torch.Tensor,
                           contrast: torch.Tensor, mean=None, std=None, out_bf16: bool = False,
                           input_u8_hwc: bool = False) -> torch.Tensor:
        """Batch augmentation on the GPU kernel; ``x`` is float ``[B, T, C, H, W]`` in
        [0, 1] or uint8 ``[B, T, H, W, C]`` (``input_u8_hwc``)."""
        from ..ops._ext import ext

        dev = x.device
        m = None if mean is None else torch.tensor(mean, device=dev, dtype=torch.float32)
        s = None if std is None else torch.tensor(std, device=dev, dtype=torch.float32)
        return ext().video_augment(x.contiguous(), input_u8_hwc, out_bf16,
                                   flip.to(dev, torch.int32).contiguous(),
                                   brightness.to(dev, torch.float32).contiguous(),
                                   contrast.to(dev, torch.float32).contiguous(), m, s)

    @classmethod
    def create_training_pipeline(cls, image_size=(256, 256)) -> "AugmentationPipeline":
        return cls([{"name": "resize", "size": image_size, "prob": 1.0},
                    {"name": "horizontal_flip", "prob": 0.5},
                    {"name": "brightness", "range": (0.9, 1.1)}, {"name": "contrast", "range": (0.9, 1.1)},
                    {"name": "saturation", "range": (0.9, 1.1), "prob": 0.3},
                    {"name": "gaussian_noise", "std": 0.01, "prob": 0.2}], p=0.5)

    @classmethod
    def create_validation_pipeline(cls, image_size=(256, 256)) -> "AugmentationPipeline":
        return cls([{"name": "resize", "size": image_size, "prob": 1.0}], p=1.0)
