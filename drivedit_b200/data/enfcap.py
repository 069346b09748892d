"""ENFCAP v1 capture files (ENFusion CAPture): native reader / writer plus a pure-Python
decoder used as the test oracle.

Same binary layout as the reference's Rust crate (rust/drivedit-data/src/enfcap.rs:61-79,
:162-222, :562-680): a 64-byte header (``ENFCAP01``, version, frame count, start
timestamp split into two f32, flags), variable-length frame records (id, timestamp,
3x4 ego transform, 10 vehicle-state floats, entity list, road-point list, flags) and a
table of u64 frame offsets at the end of the file (O(1) random access).

The header's start timestamp is written as ``lo = ts``, ``hi = ts / FLT_MAX`` (the
format's own encoding); the readers return ``ts`` for such headers where the reference
reader's ``lo + hi * FLT_MAX`` would give ``2 ts``.
"""
from __future__ import annotations

import struct
from enum import IntEnum, IntFlag
from typing import Dict, List

import numpy as np

from .native import native


class HeaderFlags(IntFlag):
    COMPRESSED = 1
    HAS_SCREENSHOTS = 2
    HAS_DEPTH = 4
    HAS_AUDIO = 8
    ANCHOR_FRAMES = 16


class FrameFlags(IntFlag):
    ANCHOR = 1
    COLLISION = 2
    MANUAL_CONTROL = 4
    SCENE_CHANGE = 8


class EntityType(IntEnum):
    VEHICLE = 0
    PEDESTRIAN = 1
    CYCLIST = 2
    ANIMAL = 3
    TRAFFIC_SIGN = 4
    TRAFFIC_LIGHT = 5
    OBSTACLE = 6
    OTHER = 7


VEHICLE_STATE_FIELDS = ("speed_kmh", "steering", "throttle", "brake", "clutch", "gear",
                        "engine_rpm", "acceleration", "yaw_rate", "slip_angle")


def ENFCAPReader(path: str):
    """Memory-mapped reader: ``frame_count``, ``start_timestamp``, ``flags``,
    ``read_frame(i)`` -> dict, ``read_frames(start, end, threads=0)`` -> dict of batched
    tensors (parallel decode), ``validate()``."""
    return native().ENFCAPReader(str(path))


def ENFCAPWriter(path: str, start_timestamp: float = 0.0, flags: int = int(HeaderFlags.ANCHOR_FRAMES)):
    """Append-only writer: ``write_frame(frame_id, timestamp, ego_transform[3,4],
    vehicle_state[10], entity_type[n], entity_pos[n,3], road_points[m,3], flags)``, then
    ``finalize()`` (writes the index table and the header's frame count)."""
    return native().ENFCAPWriter(str(path), float(start_timestamp), int(flags))


def read_enfcap_py(path: str) -> Dict[str, object]:
    """Pure-Python decode of a whole file (oracle for the native reader)."""
    with open(path, "rb") as f:
        buf = f.read()
    magic, ver, n, lo, hi, flags = struct.unpack_from("<8sIIffI", buf, 0)
    if magic != b"ENFCAP01" or ver != 1:
        raise ValueError("not an ENFCAP v1 file")
    offs = np.frombuffer(buf, dtype="<u8", count=n, offset=len(buf) - 8 * n)
    frames: List[Dict[str, object]] = []
    for o in offs.tolist():
        fid, ts = struct.unpack_from("<If", buf, o)
        ego = np.frombuffer(buf, "<f4", 12, o + 8).reshape(3, 4)
        veh = np.frombuffer(buf, "<f4", 10, o + 56)
        p = o + 96
        (ne,) = struct.unpack_from("<H", buf, p)
        p += 2
        ents = [struct.unpack_from("<Ifff", buf, p + 16 * i) for i in range(ne)]
        p += 16 * ne
        (nr,) = struct.unpack_from("<H", buf, p)
        p += 2
        road = np.frombuffer(buf, "<f4", 3 * nr, p).reshape(nr, 3)
        p += 12 * nr
        (fl,) = struct.unpack_from("<H", buf, p)
        frames.append({"frame_id": fid, "timestamp": ts, "ego_transform": ego.copy(),
                       "vehicle_state": veh.copy(), "entities": ents, "road_points": road.copy(),
                       "flags": fl})
    hi_part = float(hi) * float(np.finfo(np.float32).max)
    ts = float(lo) if hi != 0 and abs(hi_part - lo) <= 1e-3 * abs(lo) + 1e-3 else float(lo) + hi_part
    return {"frame_count": n, "start_timestamp": ts, "flags": flags, "frames": frames}
