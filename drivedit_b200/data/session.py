"""Session discovery and dataset presets (the reference's Rust ``session.rs``
``SessionMetadata`` / ``find_sessions`` and ``config.rs`` ``DatasetConfig`` with its
``minimal`` / ``production`` presets)."""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import List, Union

_IMG = (".png", ".jpg", ".jpeg")


@dataclass
class DatasetConfig:
    sequence_length: int = 16
    image_height: int = 256
    image_width: int = 512
    control_dim: int = 4
    frame_stride: int = 1
    context_frames: int = 4
    load_depth: bool = True
    load_flow: bool = False
    normalize_images: bool = True
    use_fp16: bool = False
    seed: int = 42
    augment_prob: float = 0.0

    @classmethod
    def minimal(cls) -> "DatasetConfig":
        return cls(4, 64, 128, 4, 1, 2, False, False, True, False, 42, 0.0)

    @classmethod
    def production(cls) -> "DatasetConfig":
        return cls(16, 256, 512, 4, 1, 4, True, True, True, True, 42, 0.2)

    def to_enfusion_config(self):
        """The Python dataset's config with these sizes."""
        from .enfusion import EnfusionDatasetConfig

        return EnfusionDatasetConfig(sequence_length=self.sequence_length, frame_skip=self.frame_stride,
                                     image_size=(self.image_height, self.image_width), load_depth=self.load_depth,
                                     control_dim=self.control_dim, normalize_frames=self.normalize_images,
                                     augment=self.augment_prob > 0)


@dataclass
class SessionMetadata:
    session_id: str
    num_frames: int
    duration_seconds: float
    fps: float
    width: int
    height: int
    has_telemetry: bool
    has_depth: bool
    path: str

    def __repr__(self) -> str:
        return (f"SessionMetadata(id='{self.session_id}', frames={self.num_frames}, "
                f"duration={self.duration_seconds:.1f}s, {self.width}x{self.height})")

    @classmethod
    def from_dir(cls, d: Union[str, Path]) -> "SessionMetadata":
        d = Path(d)
        frames_dir = next((d / s for s in ("frames", "images") if (d / s).exists()), d)
        frames = sorted(p for p in frames_dir.iterdir() if p.suffix.lower() in _IMG) if frames_dir.exists() else []
        info = {}
        if (d / "metadata.json").exists():
            try:
                info = json.loads((d / "metadata.json").read_text())
            except json.JSONDecodeError:
                info = {}
        fps = float(info.get("fps", 20.0))
        w = int(info.get("width", 0))
        h = int(info.get("height", 0))
        if (not w or not h) and frames and frames[0].suffix.lower() == ".png":
            head = frames[0].read_bytes()[:24]
            w, h = int.from_bytes(head[16:20], "big"), int.from_bytes(head[20:24], "big")
        n = len(frames)
        if not n and (d / "video.enfcap").exists():
            from .enfcap import read_enfcap_py

            n = len(read_enfcap_py(str(d / "video.enfcap"))["frames"])
        return cls(d.name, n, n / fps if fps > 0 else 0.0, fps, w, h,
                   any((d / f).exists() for f in ("telemetry.csv", "telemetry.txt")) or (d / "video.enfcap").exists(),
                   (d / "depth").exists(), str(d))


def is_session_dir(path: Path) -> bool:
    if (path / "video.enfcap").exists() or (path / "frames").exists() or (path / "images").exists():
        return True
    try:
        return any(p.suffix.lower() in _IMG for p in path.iterdir())
    except OSError:
        return False


def find_sessions(root: Union[str, Path]) -> List[Path]:
    """Session directories: ``root`` itself, or its children / grandchildren that are."""
    root = Path(root)
    if not root.exists():
        raise FileNotFoundError(f"Root path does not exist: {root}")
    if is_session_dir(root):
        return [root]
    out: List[Path] = []
    for c in sorted(p for p in root.iterdir() if p.is_dir()):
        if is_session_dir(c):
            out.append(c)
        else:
            out.extend(g for g in sorted(p for p in c.iterdir() if p.is_dir()) if is_session_dir(g))
    return out
