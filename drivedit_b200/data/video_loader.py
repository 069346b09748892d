"""Image-folder video sequences with the reference's API and on-disk layout
(``data/video_loader.py``: ``FrameBuffer`` :19-91, ``VideoDataset`` :94-366,
``VideoLoader`` :369-425).

Layout: ``<root>/<split>/<sequence>/`` (or ``<root>/<sequence>/`` when there is no split
folder) holding the frames (``.jpg`` / ``.jpeg`` / ``.png`` / ``.bmp``, in name order), an
optional ``controls.json`` (``{"controls": [{"steering", "acceleration", "goal_x",
"goal_y"}, ...]}``, one entry per frame) or ``controls.npy`` (``[N, A]``), and an optional
``depth/`` folder of 16-bit PNGs, one per frame. A ``<root>/<split>_metadata.json`` with
``{"sequences": [{"sequence_id", "frame_paths", "num_frames", "control_path",
"depth_paths"}]}`` replaces the scan.

Samples start every ``sequence_length // 2`` frames and take ``sequence_length`` frames
``frame_skip`` apart (the last frame repeats past a sequence's end). All the frames of a
sample decode in one call of the native PNG decoder (threads, resize included) when they
are PNGs; other formats go through OpenCV. Decoded frames can be kept in a
:class:`FrameBuffer` (LRU, bounded by count and by megabytes).
"""
from __future__ import annotations

import json
import threading
from collections import OrderedDict
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple, Union

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset


class FrameBuffer:
    """Least-recently-used cache of decoded frames, bounded by ``max_frames`` entries
    and ``max_memory_mb`` megabytes; thread-safe (loader workers are processes, but a
    threaded caller shares one buffer)."""

    def __init__(self, max_frames: int = 1000, max_memory_mb: float = 500.0):
        self.max_frames, self.max_memory_mb = max_frames, max_memory_mb
        self._d: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        self._mb = 0.0
        self._lock = threading.Lock()
        self.hits = self.misses = 0

    @staticmethod
    def _size_mb(t: torch.Tensor) -> float:
        return t.numel() * t.element_size() / 2 ** 20

    def get(self, key: str) -> Optional[torch.Tensor]:
        with self._lock:
            t = self._d.get(key)
            if t is None:
                self.misses += 1
                return None
            self._d.move_to_end(key)
            self.hits += 1
            return t

    def put(self, key: str, frame: torch.Tensor) -> None:
        with self._lock:
            old = self._d.pop(key, None)
            if old is not None:
                self._mb -= self._size_mb(old)
            self._d[key] = frame
            self._mb += self._size_mb(frame)
            while self._d and (len(self._d) > self.max_frames or self._mb > self.max_memory_mb):
                _, t = self._d.popitem(last=False)
                self._mb -= self._size_mb(t)

    def clear(self) -> None:
        with self._lock:
            self._d.clear()
            self._mb = 0.0

    def stats(self) -> Dict[str, Any]:
        with self._lock:
            return {"num_frames": len(self._d), "memory_mb": self._mb,
                    "memory_utilization": self._mb / self.max_memory_mb if self.max_memory_mb else 0.0,
                    "capacity_utilization": len(self._d) / self.max_frames if self.max_frames else 0.0,
                    "hits": self.hits, "misses": self.misses}

    def __len__(self):
        return len(self._d)


class VideoDataset(Dataset):
    def __init__(self, data_root: Union[str, Path], sequence_length: int = 16, frame_skip: int = 1,
                 image_size: Tuple[int, int] = (256, 256), split: str = "train", cache_frames: bool = True,
                 load_controls: bool = True, load_depth: bool = False,
                 supported_formats: Optional[Sequence[str]] = None, max_cache_mb: float = 500.0,
                 decode_threads: int = 0):
        self.data_root = Path(data_root)
        self.sequence_length, self.frame_skip = sequence_length, max(1, frame_skip)
        self.image_size, self.split = tuple(image_size), split
        self.load_controls, self.load_depth = load_controls, load_depth
        self.supported_formats = [f.lower() for f in (supported_formats or [".jpg", ".jpeg", ".png", ".bmp"])]
        self.cache_frames, self.decode_threads = cache_frames, decode_threads
        self.frame_buffer = FrameBuffer(max_memory_mb=max_cache_mb) if cache_frames else None
        self.sequences = self._load_sequences()
        self.sequence_indices = self._build_sequence_indices()

    # ------------------------------------------------------------------ discovery
    def _load_sequences(self) -> List[Dict[str, Any]]:
        meta = self.data_root / f"{self.split}_metadata.json"
        if meta.exists():
            return json.loads(meta.read_text()).get("sequences", [])
        return self._scan_directories()

    def _scan_directories(self) -> List[Dict[str, Any]]:
        base = self.data_root / self.split
        if not base.is_dir():
            base = self.data_root
        out = []
        for d in sorted(p for p in base.iterdir() if p.is_dir()):
            frames = sorted(p for p in d.iterdir() if p.suffix.lower() in self.supported_formats)
            if len(frames) < self.sequence_length:
                continue
            seq: Dict[str, Any] = {"sequence_id": d.name, "frame_paths": [str(p) for p in frames],
                                   "num_frames": len(frames)}
            for name in ("controls.json", "controls.npy"):
                if (d / name).exists():
                    seq["control_path"] = str(d / name)
                    break
            depth = sorted((d / "depth").glob("*.png")) if (d / "depth").is_dir() else []
            if len(depth) == len(frames):
                seq["depth_paths"] = [str(p) for p in depth]
            out.append(seq)
        return out

    def _build_sequence_indices(self) -> List[Tuple[int, int]]:
        step = max(1, self.sequence_length // 2)
        idx = []
        for si, seq in enumerate(self.sequences):
            last = seq["num_frames"] - (self.sequence_length - 1) * self.frame_skip - 1
            idx += [(si, s) for s in range(0, last + 1, step)]
        return idx

    # ------------------------------------------------------------------ loading
    def _decode(self, paths: List[str]) -> torch.Tensor:
        H, W = self.image_size
        if all(p.lower().endswith(".png") for p in paths):
            from .native import available, native

            if available():
                return native().load_frames(paths, H, W, self.decode_threads)
        import cv2

        out = []
        for p in paths:
            im = cv2.imread(p, cv2.IMREAD_COLOR)
            if im is None:
                raise ValueError(f"Could not load frame: {p}")
            if im.shape[:2] != (H, W):
                im = cv2.resize(im, (W, H), interpolation=cv2.INTER_LINEAR)
            out.append(np.ascontiguousarray(im[:, :, ::-1]))
        return torch.from_numpy(np.stack(out))

    def _load_frames(self, paths: List[str]) -> torch.Tensor:
        """``[T, 3, H, W]`` in [0, 1]; cached frames are reused, the rest decoded together."""
        got = [self.frame_buffer.get(p) if self.frame_buffer is not None else None for p in paths]
        missing = sorted({p for p, g in zip(paths, got) if g is None})
        if missing:
            dec = self._decode(missing).permute(0, 3, 1, 2).float().div_(255.0)
            new = dict(zip(missing, dec))
            if self.frame_buffer is not None:
                for p, f in new.items():
                    self.frame_buffer.put(p, f)
            got = [g if g is not None else new[p] for p, g in zip(paths, got)]
        return torch.stack(got)

    def _load_controls(self, control_path: str, start_idx: int) -> torch.Tensor:
        """``[T, 4]`` (steering, acceleration, goal x, goal y) from ``controls.json``, or
        ``[T, A]`` rows of ``controls.npy``; zeros past the recorded frames."""
        frames = [start_idx + i * self.frame_skip for i in range(self.sequence_length)]
        if control_path.endswith(".npy"):
            arr = np.load(control_path).astype(np.float32)
            out = np.zeros((self.sequence_length, arr.shape[1]), np.float32)
            for i, f in enumerate(frames):
                if f < len(arr):
                    out[i] = arr[f]
            return torch.from_numpy(out)
        rows = json.loads(Path(control_path).read_text()).get("controls", [])
        out = np.zeros((self.sequence_length, 4), np.float32)
        for i, f in enumerate(frames):
            if f < len(rows):
                c = rows[f]
                out[i] = [c.get("steering", 0.0), c.get("acceleration", 0.0),
                          c.get("goal_x", 0.0), c.get("goal_y", 0.0)]
        return torch.from_numpy(out)

    def _load_depth(self, depth_paths: List[str], start_idx: int) -> torch.Tensor:
        """``[T, 1, H, W]``: 16-bit PNG depth divided by 65535 (zeros past the end)."""
        import cv2

        H, W = self.image_size
        out = torch.zeros(self.sequence_length, 1, H, W)
        for i in range(self.sequence_length):
            f = start_idx + i * self.frame_skip
            if f >= len(depth_paths):
                continue
            d = cv2.imread(depth_paths[f], cv2.IMREAD_ANYDEPTH)
            if d is None:
                continue
            if d.shape != (H, W):
                d = cv2.resize(d, (W, H), interpolation=cv2.INTER_NEAREST)
            out[i, 0] = torch.from_numpy(d.astype(np.float32) / 65535.0)
        return out

    def __len__(self) -> int:
        return len(self.sequence_indices)

    def __getitem__(self, idx: int) -> Dict[str, Any]:
        si, start = self.sequence_indices[idx]
        seq = self.sequences[si]
        fp = seq["frame_paths"]
        paths = [fp[min(start + i * self.frame_skip, len(fp) - 1)] for i in range(self.sequence_length)]
        sample: Dict[str, Any] = {"frames": self._load_frames(paths), "sequence_id": seq["sequence_id"],
                                  "start_idx": start}
        if self.load_controls:
            cp = seq.get("control_path")
            sample["controls"] = (self._load_controls(cp, start) if cp
                                  else torch.zeros(self.sequence_length, 4))
        if self.load_depth and "depth_paths" in seq:
            sample["depth"] = self._load_depth(seq["depth_paths"], start)
        return sample

    def get_sequence_info(self, idx: int) -> Dict[str, Any]:
        si, start = self.sequence_indices[idx]
        seq = self.sequences[si]
        return {"sequence_id": seq["sequence_id"], "start_idx": start, "num_frames": seq["num_frames"],
                "sequence_length": self.sequence_length, "frame_skip": self.frame_skip}


class VideoLoader:
    """A ``DataLoader`` over a :class:`VideoDataset` with the collate function that
    stacks tensors and keeps the rest as lists."""

    def __init__(self, dataset: VideoDataset, batch_size: int = 8, shuffle: bool = True,
                 num_workers: int = 4, pin_memory: bool = True, drop_last: bool = True,
                 prefetch_factor: int = 2):
        from .collate import custom_collate_fn

        self.dataset = dataset
        kw = dict(prefetch_factor=prefetch_factor, persistent_workers=True) if num_workers > 0 else {}
        self.dataloader = DataLoader(dataset, batch_size=batch_size, shuffle=shuffle, num_workers=num_workers,
                                     pin_memory=pin_memory and torch.cuda.is_available(), drop_last=drop_last,
                                     collate_fn=custom_collate_fn, **kw)

    def __iter__(self):
        return iter(self.dataloader)

    def __len__(self):
        return len(self.dataloader)

    def get_cache_stats(self) -> Dict[str, Any]:
        fb = getattr(self.dataset, "frame_buffer", None)
        return fb.stats() if fb is not None else {}
