"""Scene graphs of 3-D entities (the reference's Rust ``scene.rs``: ``BoundingBox3D`` with
corners / rotation / containment / approximate IoU, ``EntityClass``, ``Entity``, ``EgoPose``,
``SceneGraph`` queries, ``SceneParser`` with JSON parsing, frame-to-frame entity matching,
velocity estimation, ego-frame transformation, confidence filtering and feature vectors).

Quaternions are ``(w, x, y, z)`` as in the reference. Queries over many entities are
vectorised numpy over the scene's position array instead of per-entity loops; JSON goes
through the standard library parser.
"""
from __future__ import annotations

import json
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field, replace
from enum import Enum
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


def quat_to_matrix(q) -> np.ndarray:
    w, x, y, z = np.asarray(q, dtype=np.float64) / max(np.linalg.norm(q), 1e-12)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]], dtype=np.float32)


def quat_mul(a, b) -> np.ndarray:
    w1, x1, y1, z1 = a
    w2, x2, y2, z2 = b
    return np.array([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2, w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2, w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2], np.float32)


def quat_inv(q) -> np.ndarray:
    q = np.asarray(q, np.float32) / max(float(np.dot(q, q)), 1e-12)
    return np.array([q[0], -q[1], -q[2], -q[3]], np.float32)


@dataclass
class BoundingBox3D:
    center: Tuple[float, float, float] = (0.0, 0.0, 0.0)
    dimensions: Tuple[float, float, float] = (1.0, 1.0, 1.0)   # length, width, height
    rotation: Tuple[float, float, float, float] = (1.0, 0.0, 0.0, 0.0)

    @classmethod
    def axis_aligned(cls, center, dimensions) -> "BoundingBox3D":
        return cls(tuple(center), tuple(dimensions))

    def rotation_matrix(self) -> np.ndarray:
        return quat_to_matrix(self.rotation)

    def corners(self) -> np.ndarray:
        """``[8, 3]``: bottom face (z = -h/2) counter-clockwise from (-l, -w), then the top."""
        l, w, h = (np.asarray(self.dimensions, np.float32) / 2)
        local = np.array([[-l, -w, -h], [l, -w, -h], [l, w, -h], [-l, w, -h],
                          [-l, -w, h], [l, -w, h], [l, w, h], [-l, w, h]], np.float32)
        return local @ self.rotation_matrix().T + np.asarray(self.center, np.float32)

    def volume(self) -> float:
        return float(np.prod(self.dimensions))

    def contains(self, point) -> bool:
        local = self.rotation_matrix().T @ (np.asarray(point, np.float32) - np.asarray(self.center, np.float32))
        return bool(np.all(np.abs(local) <= np.asarray(self.dimensions, np.float32) / 2 + 1e-6))

    def iou_approx(self, other: "BoundingBox3D") -> float:
        """IoU of the two boxes' axis-aligned hulls (intersection) over the true volumes."""
        a, b = self.corners(), other.corners()
        lo = np.maximum(a.min(0), b.min(0))
        hi = np.minimum(a.max(0), b.max(0))
        inter = float(np.prod(np.clip(hi - lo, 0, None)))
        union = self.volume() + other.volume() - inter
        return inter / union if union > 0 else 0.0


class EntityClass(str, Enum):
    CAR = "car"
    TRUCK = "truck"
    BUS = "bus"
    MOTORCYCLE = "motorcycle"
    BICYCLE = "bicycle"
    PEDESTRIAN = "pedestrian"
    ANIMAL = "animal"
    TRAFFIC_LIGHT = "traffic_light"
    TRAFFIC_SIGN = "traffic_sign"
    BUILDING = "building"
    VEGETATION = "vegetation"
    UNKNOWN = "unknown"

    @classmethod
    def from_str(cls, s: str) -> "EntityClass":
        s = (s or "").strip().lower()
        alias = {"vehicle": "car", "person": "pedestrian", "human": "pedestrian", "bike": "bicycle",
                 "motorbike": "motorcycle", "tree": "vegetation", "sign": "traffic_sign", "light": "traffic_light"}
        s = alias.get(s, s)
        try:
            return cls(s)
        except ValueError:
            return cls.UNKNOWN

    def is_dynamic(self) -> bool:
        return self in (EntityClass.CAR, EntityClass.TRUCK, EntityClass.BUS, EntityClass.MOTORCYCLE,
                        EntityClass.BICYCLE, EntityClass.PEDESTRIAN, EntityClass.ANIMAL)

    def is_static(self) -> bool:
        return not self.is_dynamic() and self != EntityClass.UNKNOWN


@dataclass
class Entity:
    id: int
    entity_class: EntityClass
    position: np.ndarray
    bbox_3d: BoundingBox3D = field(default_factory=BoundingBox3D)
    velocity: np.ndarray = field(default_factory=lambda: np.zeros(3, np.float32))
    confidence: float = 1.0
    attributes: Dict[str, object] = field(default_factory=dict)

    def __post_init__(self):
        self.position = np.asarray(self.position, np.float32)
        self.velocity = np.asarray(self.velocity, np.float32)

    def speed(self) -> float:
        return float(np.linalg.norm(self.velocity))

    def is_moving(self, threshold: float = 0.5) -> bool:
        return self.speed() > threshold

    def distance_from_origin(self) -> float:
        return float(np.linalg.norm(self.position))

    def distance_to(self, other: "Entity") -> float:
        return float(np.linalg.norm(self.position - other.position))

    def predict_position(self, dt: float) -> np.ndarray:
        return self.position + self.velocity * dt


@dataclass
class EgoPose:
    position: np.ndarray = field(default_factory=lambda: np.zeros(3, np.float32))
    rotation: np.ndarray = field(default_factory=lambda: np.array([1, 0, 0, 0], np.float32))
    velocity: np.ndarray = field(default_factory=lambda: np.zeros(3, np.float32))


@dataclass
class SceneGraph:
    frame_id: int = 0
    timestamp: float = 0.0
    entities: List[Entity] = field(default_factory=list)
    ego_pose: Optional[EgoPose] = None

    def add_entity(self, e: Entity) -> None:
        self.entities.append(e)

    def get_entity(self, id_: int) -> Optional[Entity]:
        return next((e for e in self.entities if e.id == id_), None)

    def get_by_class(self, cls: EntityClass) -> List[Entity]:
        return [e for e in self.entities if e.entity_class == cls]

    def get_dynamic(self) -> List[Entity]:
        return [e for e in self.entities if e.entity_class.is_dynamic()]

    def get_static(self) -> List[Entity]:
        return [e for e in self.entities if e.entity_class.is_static()]

    def positions(self) -> np.ndarray:
        return np.stack([e.position for e in self.entities]) if self.entities else np.zeros((0, 3), np.float32)

    def get_within_distance(self, point, max_distance: float) -> List[Entity]:
        d2 = ((self.positions() - np.asarray(point, np.float32)) ** 2).sum(1)
        return [self.entities[i] for i in np.nonzero(d2 <= max_distance ** 2)[0]]

    def get_in_fov(self, fov_deg: float, max_range: float) -> List[Entity]:
        """Entities within ``max_range`` (xy plane) and ``fov_deg`` of the ego's +x axis."""
        p = self.positions()
        dist = np.hypot(p[:, 0], p[:, 1])
        ang = np.abs(np.arctan2(p[:, 1], p[:, 0]))
        keep = (dist <= max_range) & (ang <= np.radians(fov_deg) / 2)
        return [self.entities[i] for i in np.nonzero(keep)[0]]

    def __len__(self) -> int:
        return len(self.entities)

    def is_empty(self) -> bool:
        return not self.entities

    def class_histogram(self) -> Dict[EntityClass, int]:
        h: Dict[EntityClass, int] = {}
        for e in self.entities:
            h[e.entity_class] = h.get(e.entity_class, 0) + 1
        return h


class SceneParser:
    """JSON scenes: ``{"frame_id", "timestamp", "entities": [{"id", "class", "position",
    "bbox"/"bbox_3d": {"center", "dimensions", "rotation"}, "velocity", "confidence"}],
    "ego_pose": {"position", "rotation", "velocity"}}``."""

    def __init__(self):
        self.parsed = 0

    def parse_str(self, s: str) -> SceneGraph:
        return self._from_dict(json.loads(s))

    def parse_bytes(self, b: bytes) -> SceneGraph:
        return self.parse_str(b.decode("utf-8"))

    def parse_file(self, path) -> SceneGraph:
        return self.parse_str(Path(path).read_text())

    def parse_batch(self, paths: Sequence, threads: int = 8) -> List[object]:
        """One result per path: the scene or the exception raised parsing it."""
        def one(p):
            try:
                return self.parse_file(p)
            except Exception as e:  # noqa: BLE001 - reported per file
                return e

        with ThreadPoolExecutor(threads) as ex:
            return list(ex.map(one, paths))

    def parse_batch_ok(self, paths: Sequence, threads: int = 8) -> List[SceneGraph]:
        return [s for s in self.parse_batch(paths, threads) if isinstance(s, SceneGraph)]

    def _from_dict(self, d: Dict) -> SceneGraph:
        self.parsed += 1
        ents = []
        for i, e in enumerate(d.get("entities", [])):
            bb = e.get("bbox_3d", e.get("bbox", {})) or {}
            box = BoundingBox3D(tuple(bb.get("center", e.get("position", (0, 0, 0)))),
                                tuple(bb.get("dimensions", (1, 1, 1))), tuple(bb.get("rotation", (1, 0, 0, 0))))
            ents.append(Entity(int(e.get("id", i)), EntityClass.from_str(e.get("class", e.get("type", ""))),
                               e.get("position", box.center), box, e.get("velocity", (0, 0, 0)),
                               float(e.get("confidence", 1.0)),
                               {k: v for k, v in e.items() if k not in ("id", "class", "type", "position", "bbox",
                                                                        "bbox_3d", "velocity", "confidence")}))
        ego = None
        if "ego_pose" in d and d["ego_pose"]:
            ep = d["ego_pose"]
            ego = EgoPose(np.asarray(ep.get("position", (0, 0, 0)), np.float32),
                          np.asarray(ep.get("rotation", (1, 0, 0, 0)), np.float32),
                          np.asarray(ep.get("velocity", (0, 0, 0)), np.float32))
        return SceneGraph(int(d.get("frame_id", 0)), float(d.get("timestamp", 0.0)), ents, ego)

    # ---------------------------------------------------------------- temporal / frames
    @staticmethod
    def match_entities(prev: SceneGraph, curr: SceneGraph, max_distance: float) -> List[Tuple[int, int]]:
        """Greedy nearest match of same-class entities within ``max_distance``."""
        if not prev.entities or not curr.entities:
            return []
        pp, cp = prev.positions(), curr.positions()
        dist = np.linalg.norm(pp[:, None] - cp[None], axis=-1)
        same = np.array([[a.entity_class == b.entity_class for b in curr.entities] for a in prev.entities])
        dist = np.where(same & (dist <= max_distance), dist, np.inf)
        used = np.zeros(len(curr.entities), bool)
        out = []
        for i in range(len(prev.entities)):
            row = np.where(used, np.inf, dist[i])
            j = int(np.argmin(row))
            if np.isfinite(row[j]):
                used[j] = True
                out.append((prev.entities[i].id, curr.entities[j].id))
        return out

    @staticmethod
    def compute_velocities(prev: SceneGraph, curr: SceneGraph, matches: List[Tuple[int, int]]) -> None:
        dt = curr.timestamp - prev.timestamp
        if dt <= 0:
            return
        pm = {e.id: e for e in prev.entities}
        cm = {e.id: e for e in curr.entities}
        for a, b in matches:
            if a in pm and b in cm:
                cm[b].velocity = (cm[b].position - pm[a].position) / dt

    @staticmethod
    def transform_to_ego(scene: SceneGraph) -> SceneGraph:
        """Positions, velocities and boxes in the ego frame (no-op without an ego pose)."""
        if scene.ego_pose is None:
            return scene
        R = quat_to_matrix(scene.ego_pose.rotation)
        t = np.asarray(scene.ego_pose.position, np.float32)
        inv_q = quat_inv(scene.ego_pose.rotation)
        ents = []
        for e in scene.entities:
            box = replace(e.bbox_3d, center=tuple(R.T @ (np.asarray(e.bbox_3d.center, np.float32) - t)),
                          rotation=tuple(quat_mul(inv_q, e.bbox_3d.rotation)))
            ents.append(replace(e, position=R.T @ (e.position - t), velocity=R.T @ e.velocity, bbox_3d=box))
        return SceneGraph(scene.frame_id, scene.timestamp, ents, EgoPose())

    @staticmethod
    def filter_by_confidence(scene: SceneGraph, min_confidence: float) -> None:
        scene.entities = [e for e in scene.entities if e.confidence >= min_confidence]

    @staticmethod
    def to_feature_vector(scene: SceneGraph, max_entities: int = 64, max_distance: float = 100.0) -> np.ndarray:
        """``[max_entities, 16]``: one-hot-free compact rows (class index, position / max
        distance, velocity, box dimensions, yaw sin/cos, confidence, valid flag) for the
        nearest entities; zero rows pad."""
        out = np.zeros((max_entities, 16), np.float32)
        ents = sorted(scene.entities, key=lambda e: e.distance_from_origin())[:max_entities]
        classes = list(EntityClass)
        for i, e in enumerate(ents):
            w, x, y, z = e.bbox_3d.rotation
            yaw = np.arctan2(2 * (w * z + x * y), 1 - 2 * (y * y + z * z))
            out[i, 0] = classes.index(e.entity_class) / len(classes)
            out[i, 1:4] = e.position / max_distance
            out[i, 4:7] = e.velocity
            out[i, 7:10] = e.bbox_3d.dimensions
            out[i, 10], out[i, 11] = np.sin(yaw), np.cos(yaw)
            out[i, 12] = e.confidence
            out[i, 13] = 1.0
            out[i, 14] = float(e.entity_class.is_dynamic())
            out[i, 15] = e.speed()
        return out
