"""Telemetry parsing (native CSV parser) and control normalisation.

``TelemetryParser`` maps the reference's Python parser API
(data/enfusion_preprocessing.py:59-248: ``parse_csv``, ``interpolate_to_frame_rate``,
``compute_ego_transform``) onto the native parser (csrc/data/telemetry.cpp, the column
alias lists of rust/drivedit-data/src/telemetry.rs:353-520). ``ControlNormalizer``
produces the 6-D control vector of ``EnfusionControlNormalizer``
(data/enfusion_preprocessing.py:251-419).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

import numpy as np
import torch

from .native import native


@dataclass
class TelemetryConfig:
    """Normalisation ranges, the reference's column names and rates, and the session
    quality thresholds (the reference's ``EnfusionTelemetryConfig`` fields and defaults,
    data/enfusion_preprocessing.py:20-56, so its configs load). The native parser finds
    columns by its alias lists; the ``*_col`` names are kept for the reference's code."""
    steering_range: Tuple[float, float] = (-1.0, 1.0)
    throttle_range: Tuple[float, float] = (0.0, 1.0)
    brake_range: Tuple[float, float] = (0.0, 1.0)
    speed_range: Tuple[float, float] = (0.0, 50.0)  # m/s
    speed_unit_kmh: bool = True                      # the `speed` column is km/h
    timestamp_col: str = "timestamp"
    position_cols: Tuple[str, str, str] = ("pos_x", "pos_y", "pos_z")
    rotation_cols: Tuple[str, str, str] = ("rot_pitch", "rot_yaw", "rot_roll")
    velocity_cols: Tuple[str, str, str] = ("vel_x", "vel_y", "vel_z")
    throttle_col: str = "throttle"
    brake_col: str = "brake"
    steering_col: str = "steering"
    gear_col: str = "gear"
    rpm_col: str = "rpm"
    speed_col: str = "speed"
    telemetry_rate: float = 5.0       # Hz
    frame_rate: float = 30.0          # Hz
    min_speed_variation: float = 0.1  # speed std (m/s) of a "dynamic" session
    max_stationary_ratio: float = 0.8
    min_steering_variation: float = 0.01
    max_position_jump: float = 10.0   # m between rows
    max_rotation_jump: float = 90.0   # degrees between rows


EnfusionTelemetryConfig = TelemetryConfig


class TelemetryParser:
    def __init__(self, config: TelemetryConfig = None):
        self.config = config or TelemetryConfig()

    @staticmethod
    def parse_raw(path) -> Dict[str, torch.Tensor]:
        """All recognised columns as float64 tensors (native parser)."""
        return native().parse_telemetry(str(path))

    @staticmethod
    def parse_files(paths, threads: int = 0):
        return native().parse_telemetry_files([str(p) for p in paths], threads)

    def parse_csv(self, path) -> Dict[str, np.ndarray]:
        raw = self.parse_raw(path)
        n = int(raw["_rows"])
        g = lambda k: raw[k].numpy().astype(np.float32) if k in raw else np.zeros(n, np.float32)
        speed = g("speed_ms") if "speed_ms" in raw else g("speed_kmh") / 3.6
        out = {
            "timestamp": (raw["timestamp_ms"].numpy() / 1000.0).astype(np.float32) if "timestamp_ms" in raw
            else np.arange(n, dtype=np.float32),
            "position": np.stack([g("latitude"), g("longitude"), g("altitude")], 1),
            "rotation": np.stack([g("heading"), g("pitch"), g("roll")], 1),
            "steering": g("steering"), "throttle": g("throttle"), "brake": g("brake"),
            "speed": speed, "yaw_rate": g("yaw_rate"),
            "acceleration": np.stack([g("acceleration_x"), g("acceleration_y"), g("acceleration_z")], 1),
        }
        if "velocity_x" in raw and "velocity_y" in raw:
            out["velocity"] = np.stack([g("velocity_x"), g("velocity_y"), np.zeros(n, np.float32)], 1)
        if "frame_id" in raw:
            out["frame_id"] = raw["frame_id"].numpy().astype(np.int64)
        return out

    @staticmethod
    def interpolate_to_frame_rate(telemetry: Dict[str, np.ndarray], num_frames: int) -> Dict[str, np.ndarray]:
        """Linear resampling of every per-row array to ``num_frames`` rows."""
        out = {}
        for k, v in telemetry.items():
            v = np.asarray(v)
            n = v.shape[0]
            if n == num_frames or n == 0:
                out[k] = v
                continue
            src = np.linspace(0.0, 1.0, n)
            dst = np.linspace(0.0, 1.0, num_frames)
            if v.ndim == 1:
                out[k] = np.interp(dst, src, v.astype(np.float64)).astype(v.dtype if v.dtype.kind == "f" else np.float32)
            else:
                out[k] = np.stack([np.interp(dst, src, v[:, j]) for j in range(v.shape[1])], 1).astype(np.float32)
        return out

    @staticmethod
    def compute_ego_transform(position: np.ndarray, rotation: np.ndarray) -> np.ndarray:
        """``[N, 4, 4]`` from positions and (heading, pitch, roll) in degrees (Z-Y-X)."""
        N = position.shape[0]
        y, p, r = (np.deg2rad(rotation[:, i].astype(np.float64)) for i in range(3))
        cy, sy, cp, sp, cr, sr = np.cos(y), np.sin(y), np.cos(p), np.sin(p), np.cos(r), np.sin(r)
        R = np.empty((N, 3, 3))
        R[:, 0, 0] = cy * cp
        R[:, 0, 1] = cy * sp * sr - sy * cr
        R[:, 0, 2] = cy * sp * cr + sy * sr
        R[:, 1, 0] = sy * cp
        R[:, 1, 1] = sy * sp * sr + cy * cr
        R[:, 1, 2] = sy * sp * cr - cy * sr
        R[:, 2, 0] = -sp
        R[:, 2, 1] = cp * sr
        R[:, 2, 2] = cp * cr
        T = np.tile(np.eye(4), (N, 1, 1))
        T[:, :3, :3] = R
        T[:, :3, 3] = position
        return T.astype(np.float32)


EnfusionTelemetryParser = TelemetryParser


def _to_range(v, in_rng, out_rng):
    lo, hi = in_rng
    olo, ohi = out_rng
    v = np.clip(v, lo, hi)
    n = (v - lo) / (hi - lo) if hi - lo > 1e-8 else np.zeros_like(v)
    return (n * (ohi - olo) + olo).astype(np.float32)


class ControlNormalizer:
    """6-D controls ``[steering, throttle-brake, brake, forward-vel|speed proxy,
    lateral-vel, speed]`` in [-1, 1] / [0, 1]."""

    def __init__(self, config: TelemetryConfig = None):
        self.config = config or TelemetryConfig()

    def normalize_controls(self, telemetry: Dict[str, np.ndarray], output_dim: int = 6) -> torch.Tensor:
        c = self.config
        T = len(telemetry.get("timestamp", []))
        if T == 0:
            return torch.zeros(1, output_dim)
        out = np.zeros((T, output_dim), np.float32)
        z = np.zeros(T, np.float32)
        thr, brk = np.asarray(telemetry.get("throttle", z)), np.asarray(telemetry.get("brake", z))
        if "steering" in telemetry:
            out[:, 0] = _to_range(np.asarray(telemetry["steering"]), c.steering_range, (-1.0, 1.0))
        out[:, 1] = (thr - brk).astype(np.float32)
        if "brake" in telemetry:
            out[:, 2] = _to_range(brk, c.brake_range, (0.0, 1.0))
        if "velocity" in telemetry and output_dim > 4:
            vel = np.asarray(telemetry["velocity"])
            out[:, 3] = _to_range(vel[:, 0], (-c.speed_range[1], c.speed_range[1]), (-1.0, 1.0))
            out[:, 4] = _to_range(vel[:, 1], (-0.5 * c.speed_range[1], 0.5 * c.speed_range[1]), (-1.0, 1.0))
        elif "speed" in telemetry and output_dim > 3:
            out[:, 3] = _to_range(np.asarray(telemetry["speed"]), c.speed_range, (0.0, 1.0))
        if "speed" in telemetry and output_dim > 5:
            out[:, 5] = _to_range(np.asarray(telemetry["speed"]), c.speed_range, (0.0, 1.0))
        return torch.from_numpy(out)

    def denormalize_controls(self, controls: torch.Tensor) -> Dict[str, torch.Tensor]:
        s = self.config.speed_range[1]
        return {"steering": controls[..., 0], "acceleration": controls[..., 1], "brake": controls[..., 2],
                "velocity_forward": controls[..., 3] * s, "velocity_lateral": controls[..., 4] * 0.5 * s,
                "speed": controls[..., 5] * s}

    @staticmethod
    def normalize_native(raw_table: Dict[str, torch.Tensor], speed_range=(0.0, 50.0)) -> torch.Tensor:
        """Same 6-D vector computed in C++ straight from ``TelemetryParser.parse_raw``."""
        return native().normalize_controls(raw_table, speed_range=tuple(speed_range))


EnfusionControlNormalizer = ControlNormalizer
