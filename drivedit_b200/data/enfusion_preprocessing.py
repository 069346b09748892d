"""Per-file processors of Enfusion capture sessions with the reference's API
(data/enfusion_preprocessing.py): telemetry parsing and control normalisation (the
native parser, :mod:`drivedit_b200.data.telemetry`), frames, depth maps, scene graphs,
session quality scoring, anchor frames, and the factory that builds them all.

Frames decode through the native PNG decoder (threaded, resize included) when every path
is a PNG, else through OpenCV; depth maps through the native depth loader
(:mod:`drivedit_b200.data.depth`). The dataset that combines them per sample is
:class:`drivedit_b200.data.enfusion.EnfusionDataset`.
"""
from __future__ import annotations

import json
import warnings
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch
import torch.nn.functional as F

from .native import available as native_available
from .native import native
from .telemetry import (ControlNormalizer, EnfusionControlNormalizer,  # noqa: F401
                        EnfusionTelemetryConfig, EnfusionTelemetryParser, TelemetryConfig,
                        TelemetryParser)

PathLike = Union[str, Path]
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def _view(stats: torch.Tensor, dim: int) -> torch.Tensor:
    """Per-channel statistics shaped to broadcast over [C, H, W], [T, C, H, W] or
    [B, T, C, H, W]."""
    return stats.view((1,) * (dim - 3) + (-1, 1, 1))


class EnfusionFrameProcessor:
    """RGB frames resized to ``target_size`` (H, W), in [0, 1], optionally standardised
    per channel (ImageNet statistics by default)."""

    def __init__(self, target_size: Tuple[int, int] = (256, 256), normalize: bool = True,
                 mean: Optional[Sequence[float]] = None, std: Optional[Sequence[float]] = None,
                 threads: int = 0):
        self.target_size = tuple(target_size)
        self.normalize = normalize
        self.mean = list(mean or IMAGENET_MEAN)
        self.std = list(std or IMAGENET_STD)
        self.threads = threads

    def _standardise(self, x: torch.Tensor) -> torch.Tensor:
        if not self.normalize:
            return x
        m = _view(torch.tensor(self.mean, dtype=x.dtype), x.dim())
        s = _view(torch.tensor(self.std, dtype=x.dtype), x.dim())
        return (x - m) / s

    def _decode(self, paths: List[str]) -> torch.Tensor:
        """uint8 ``[T, H, W, 3]``; raises ValueError on an unreadable file."""
        H, W = self.target_size
        if native_available() and all(p.lower().endswith(".png") for p in paths):
            return native().load_frames(paths, H, W, self.threads)
        import cv2

        out = []
        for p in paths:
            im = cv2.imread(p, cv2.IMREAD_COLOR)
            if im is None:
                raise ValueError(f"Failed to load frame: {p}")
            if im.shape[:2] != (H, W):
                im = cv2.resize(im, (W, H), interpolation=cv2.INTER_LINEAR)
            out.append(np.ascontiguousarray(im[:, :, ::-1]))
        return torch.from_numpy(np.stack(out))

    def load_frame(self, frame_path: PathLike) -> torch.Tensor:
        """``[3, H, W]``."""
        u8 = self._decode([str(frame_path)])
        return self._standardise(u8[0].permute(2, 0, 1).float() / 255.0)

    def load_frames(self, frame_paths: Sequence[PathLike], max_frames: Optional[int] = None) -> torch.Tensor:
        """``[T, 3, H, W]``; frames that fail to load are skipped with a warning (all at
        once when the batch decodes in one native call; one by one otherwise)."""
        paths = [str(p) for p in frame_paths][:max_frames]
        try:
            u8 = self._decode(paths)
        except Exception:
            good = []
            for p in paths:
                try:
                    good.append(self._decode([p]))
                except Exception as e:
                    warnings.warn(f"Skipping frame {p}: {e}")
            if not good:
                raise ValueError("No frames could be loaded")
            u8 = torch.cat(good)
        return self._standardise(u8.permute(0, 3, 1, 2).float() / 255.0)

    def denormalize(self, frames: torch.Tensor) -> torch.Tensor:
        if not self.normalize:
            return frames
        m = _view(torch.tensor(self.mean, dtype=frames.dtype, device=frames.device), frames.dim())
        s = _view(torch.tensor(self.std, dtype=frames.dtype, device=frames.device), frames.dim())
        return (frames * s + m).clamp(0.0, 1.0)


class EnfusionDepthProcessor:
    """Depth maps (``npz`` / ``npy`` arrays in metres, or 16-bit PNG scaled to
    ``[0, max_depth]``) resized to ``target_size`` and divided by ``max_depth`` into [0, 1]."""

    def __init__(self, target_size: Tuple[int, int] = (256, 256), max_depth: float = 100.0,
                 depth_format: str = "npz"):
        if depth_format not in ("npz", "npy", "png16"):
            raise ValueError(f"Unsupported depth format: {depth_format}")
        self.target_size = tuple(target_size)
        self.max_depth = float(max_depth)
        self.depth_format = depth_format

    def _metres(self, path: str) -> np.ndarray:
        if self.depth_format == "png16":
            import cv2

            d = cv2.imread(path, cv2.IMREAD_ANYDEPTH)
            if d is None:
                raise ValueError(f"Failed to load depth: {path}")
            return d.astype(np.float32) / 65535.0 * self.max_depth
        d = np.load(path)
        if hasattr(d, "files"):
            d = d["depth"] if "depth" in d.files else d[d.files[0]]
        return np.asarray(d, np.float32)

    def load_depth(self, depth_path: PathLike) -> torch.Tensor:
        """``[1, H, W]`` in [0, 1]."""
        d = self._metres(str(depth_path))
        if d.ndim == 3:
            d = d[..., 0]
        t = torch.from_numpy(np.ascontiguousarray(d))[None, None]
        if tuple(t.shape[-2:]) != self.target_size:
            t = F.interpolate(t, size=self.target_size, mode="bilinear", align_corners=False)
        return (t[0] / self.max_depth).clamp(0.0, 1.0)

    def load_depth_sequence(self, depth_paths: Sequence[PathLike]) -> torch.Tensor:
        """``[T, 1, H, W]``; a map that fails to load becomes zeros (with a warning)."""
        out = []
        for p in depth_paths:
            try:
                out.append(self.load_depth(p))
            except Exception as e:
                warnings.warn(f"Skipping depth {p}: {e}")
                out.append(torch.zeros(1, *self.target_size))
        return torch.stack(out)

    def denormalize(self, depth: torch.Tensor) -> torch.Tensor:
        return depth * self.max_depth


class EnfusionSceneParser:
    """Scene-graph JSON files -> ``{'entities': [...], 'timestamp', 'weather',
    'time_of_day'}`` with at most ``max_entities`` entities, each carrying id, class,
    position, rotation, velocity, 2-D and 3-D boxes, visibility and distance (defaults
    for missing keys). The typed scene graph is :class:`drivedit_b200.data.scene.SceneParser`."""

    _ENTITY_DEFAULTS = (("id", ""), ("class", "unknown"), ("position", [0, 0, 0]),
                        ("rotation", [0, 0, 0]), ("velocity", [0, 0, 0]), ("bbox", [0, 0, 0, 0]),
                        ("bbox_3d", [0, 0, 0, 0, 0, 0]), ("visible", True), ("distance", 0.0))

    def __init__(self, max_entities: int = 64):
        self.max_entities = max_entities

    def parse_scene(self, scene_path: PathLike) -> Dict[str, Any]:
        data = json.loads(Path(scene_path).read_text())
        ents = [{k: e.get(k, dflt) for k, dflt in self._ENTITY_DEFAULTS}
                for e in data.get("entities", [])[:self.max_entities]]
        return {"entities": ents, "timestamp": data.get("timestamp", 0.0),
                "weather": data.get("weather", "clear"), "time_of_day": data.get("time_of_day", 12.0)}

    def parse_scene_sequence(self, scene_paths: Sequence[PathLike]) -> List[Dict[str, Any]]:
        out = []
        for p in scene_paths:
            try:
                out.append(self.parse_scene(p))
            except Exception as e:
                warnings.warn(f"Skipping scene {p}: {e}")
                out.append({"entities": [], "timestamp": 0.0})
        return out


class EnfusionQualityFilter:
    """Session quality in [0, 1]: the mean of frame completeness (frames against
    duration x frame rate), speed and steering variation (std over their thresholds,
    capped at 1), continuity (1 - 10 x the fraction of position jumps above
    ``max_position_jump``, floored at 0) and motion (1 - stationary fraction over
    ``max_stationary_ratio``). The same components and weights as the reference
    (data/enfusion_preprocessing.py:710-837), so sessions rank the same."""

    def __init__(self, config: Optional[TelemetryConfig] = None):
        self.config = config or TelemetryConfig()

    def _expected_frames(self, tel: Dict[str, np.ndarray]) -> int:
        ts = np.asarray(tel.get("timestamp", []))
        return int((ts[-1] - ts[0]) * self.config.frame_rate) if ts.size else 0

    def _continuity(self, tel: Dict[str, np.ndarray]) -> float:
        pos = np.asarray(tel.get("position", np.zeros((0, 3))))
        if pos.size < 2 or pos.shape[0] < 2:
            return 1.0
        jumps = np.linalg.norm(np.diff(pos, axis=0), axis=1) > self.config.max_position_jump
        return 1.0 - min(float(jumps.mean()) * 10.0, 1.0)

    def compute_quality_score(self, telemetry: Dict[str, np.ndarray], frame_paths: Sequence) -> float:
        c = self.config
        parts = [min(len(frame_paths) / max(self._expected_frames(telemetry), 1), 1.0)]
        speed = np.asarray(telemetry.get("speed", []))
        steer = np.asarray(telemetry.get("steering", []))
        if speed.size:
            parts.append(min(float(speed.std()) / c.min_speed_variation, 1.0))
        if steer.size:
            parts.append(min(float(steer.std()) / c.min_steering_variation, 1.0))
        parts.append(self._continuity(telemetry))
        if speed.size:
            parts.append(1.0 - min(float((speed < 0.5).mean()) / c.max_stationary_ratio, 1.0))
        return float(np.mean(parts))

    def filter_sessions(self, session_dirs: Sequence[PathLike], min_quality: float = 0.5) -> List[Tuple[Path, float]]:
        """``(session, score)`` of the sessions with ``telemetry.csv`` scoring at least
        ``min_quality``, best first (all telemetry files parsed by the native parser)."""
        parser = TelemetryParser(self.config)
        out = []
        for d in map(Path, session_dirs):
            tp = d / "telemetry.csv"
            if not tp.exists():
                continue
            try:
                tel = parser.parse_csv(tp)
                frames = sorted((d / "frames").glob("*.png")) if (d / "frames").exists() else []
                q = self.compute_quality_score(tel, frames)
            except Exception as e:
                warnings.warn(f"Error processing session {d}: {e}")
                continue
            if q >= min_quality:
                out.append((d, q))
        out.sort(key=lambda x: x[1], reverse=True)
        return out


class EnfusionAnchorDetector:
    """Anchor frames of a control sequence ``[T, D]``: first and last frame (optional),
    and every frame whose steering (channel 0) or speed (channel 5) change from the
    previous frame exceeds its threshold, at least ``min_interval`` frames after the
    previous anchor."""

    def __init__(self, min_steering_change: float = 0.1, min_speed_change: float = 2.0,
                 min_interval: int = 10):
        self.min_steering_change = min_steering_change
        self.min_speed_change = min_speed_change
        self.min_interval = min_interval

    def detect_anchors(self, controls: torch.Tensor, include_first_last: bool = True) -> torch.Tensor:
        T = controls.shape[0]
        out = torch.zeros(T, dtype=torch.bool)
        if T == 0:
            return out
        if include_first_last:
            out[0] = out[-1] = True
        d = (controls[1:] - controls[:-1]).abs()
        big = d[:, 0] > self.min_steering_change
        if controls.shape[1] > 5:
            big |= d[:, 5] > self.min_speed_change
        last = 0
        for i in range(1, T):   # sequential: each anchor pushes the next window
            if i - last >= self.min_interval and bool(big[i - 1]):
                out[i] = True
                last = i
        return out


def create_enfusion_preprocessors(config: Optional[TelemetryConfig] = None,
                                  target_size: Tuple[int, int] = (256, 256),
                                  max_depth: float = 100.0) -> Dict[str, Any]:
    """Every processor above, keyed as in the reference."""
    config = config or TelemetryConfig()
    return {"telemetry_parser": TelemetryParser(config),
            "control_normalizer": ControlNormalizer(config),
            "frame_processor": EnfusionFrameProcessor(target_size=target_size),
            "depth_processor": EnfusionDepthProcessor(target_size=target_size, max_depth=max_depth),
            "scene_parser": EnfusionSceneParser(),
            "quality_filter": EnfusionQualityFilter(config),
            "anchor_detector": EnfusionAnchorDetector()}
