"""Depth maps (the reference's Rust ``depth.rs``: ``DepthLoaderConfig``, ``DepthMap``,
``DepthLoader`` with ``load / load_npz / load_npy / load_png_16bit / load_exr /
load_batch / load_batch_contiguous`` and the ``utils`` conversions).

Decoding, resizing and normalisation run in the native runtime (``csrc/data/depth.cpp``,
threads without the GIL); the conversions below are vectorised torch ops.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import List, Sequence, Tuple, Union

import torch

from .native import native

PathLike = Union[str, Path]


@dataclass
class DepthLoaderConfig:
    target_width: int = 640
    target_height: int = 360
    min_depth: float = 0.0          # both 0: range from the map's finite values
    max_depth: float = 0.0
    clip_depth: bool = True
    invert_depth: bool = False
    npz_array_name: str = "depth"   # "" = the first array of the archive

    @classmethod
    def with_resolution(cls, width: int, height: int) -> "DepthLoaderConfig":
        return cls(target_width=width, target_height=height)

    def with_depth_range(self, lo: float, hi: float) -> "DepthLoaderConfig":
        self.min_depth, self.max_depth = lo, hi
        return self

    def with_inversion(self) -> "DepthLoaderConfig":
        self.invert_depth = True
        return self

    def with_npz_array(self, name: str) -> "DepthLoaderConfig":
        self.npz_array_name = name
        return self

    def _kw(self):
        return dict(target_width=self.target_width, target_height=self.target_height, min_depth=self.min_depth,
                    max_depth=self.max_depth, clip_depth=self.clip_depth, invert_depth=self.invert_depth,
                    npz_array_name=self.npz_array_name)


@dataclass
class DepthMap:
    data: torch.Tensor               # [H, W] float32 in [0, 1]
    original_min: float
    original_max: float

    def shape(self) -> Tuple[int, int]:
        return tuple(self.data.shape)

    def original_range(self) -> Tuple[float, float]:
        return self.original_min, self.original_max

    def sample(self, x: float, y: float) -> float:
        """Bilinear value at continuous pixel coordinates (clamped to the map)."""
        H, W = self.data.shape
        x = min(max(x, 0.0), W - 1.0)
        y = min(max(y, 0.0), H - 1.0)
        x0, y0 = int(x), int(y)
        x1, y1 = min(x0 + 1, W - 1), min(y0 + 1, H - 1)
        fx, fy = x - x0, y - y0
        d = self.data
        top = d[y0, x0] * (1 - fx) + d[y0, x1] * fx
        bot = d[y1, x0] * (1 - fx) + d[y1, x1] * fx
        return float(top * (1 - fy) + bot * fy)


class DepthLoader:
    def __init__(self, config: DepthLoaderConfig = None):
        self.config = config or DepthLoaderConfig()

    @classmethod
    def default_loader(cls) -> "DepthLoader":
        return cls(DepthLoaderConfig())

    def load(self, path: PathLike) -> DepthMap:
        t, lo, hi = native().load_depth(str(path), **self.config._kw())
        return DepthMap(t, lo, hi)

    load_npz = load_npy = load_png_16bit = load

    def load_exr(self, path: PathLike) -> DepthMap:
        raise NotImplementedError("EXR depth is not supported; convert to .npy / .npz / 16-bit PNG")

    def load_batch(self, paths: Sequence[PathLike]) -> List[DepthMap]:
        return [self.load(p) for p in paths]

    def load_batch_contiguous(self, paths: Sequence[PathLike], threads: int = 0) -> torch.Tensor:
        """``[N, target_height, target_width]`` float32, decoded in parallel."""
        kw = self.config._kw()
        return native().load_depth_batch([str(p) for p in paths], threads=threads, **kw)

    def target_dimensions(self) -> Tuple[int, int]:
        return self.config.target_width, self.config.target_height


# ----------------------------------------------------------------------------- utils
def depth_to_disparity(depth: torch.Tensor, baseline: float, focal_length: float, min_depth: float = 1e-3):
    return torch.where(depth > min_depth, baseline * focal_length / depth.clamp_min(min_depth), torch.zeros_like(depth))


def disparity_to_depth(disp: torch.Tensor, baseline: float, focal_length: float, min_disparity: float = 1e-6):
    return torch.where(disp > min_disparity, baseline * focal_length / disp.clamp_min(min_disparity),
                       torch.full_like(disp, float("inf")))


def log_depth(depth: torch.Tensor, near: float, far: float) -> torch.Tensor:
    ln, lf = torch.log(torch.tensor(near)), torch.log(torch.tensor(far))
    r = float(lf - ln)
    return (depth.clamp(near, far).log() - ln) / (r if abs(r) > 1e-8 else 1.0)


def depth_gradient(depth: torch.Tensor) -> torch.Tensor:
    """Central-difference gradient magnitude of ``[H, W]`` (zero on the border)."""
    g = torch.zeros_like(depth)
    dx = depth[1:-1, 2:] - depth[1:-1, :-2]
    dy = depth[2:, 1:-1] - depth[:-2, 1:-1]
    g[1:-1, 1:-1] = torch.sqrt(dx * dx + dy * dy)
    return g


def fill_invalid(depth: torch.Tensor, invalid_value: float = 0.0, iterations: int = 10) -> torch.Tensor:
    """Fills invalid pixels with the mean of their valid 3x3 neighbours, repeatedly."""
    d = depth.clone().float()
    valid = (d != invalid_value) & torch.isfinite(d)
    d[~valid] = 0
    k = torch.ones(1, 1, 3, 3)
    for _ in range(iterations):
        if bool(valid.all()):
            break
        s = torch.nn.functional.conv2d((d * valid)[None, None], k, padding=1)[0, 0]
        c = torch.nn.functional.conv2d(valid.float()[None, None], k, padding=1)[0, 0]
        fill = (~valid) & (c > 0)
        d[fill] = s[fill] / c[fill]
        valid = valid | fill
    return d
