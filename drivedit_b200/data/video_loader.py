"""Image-folder video sequences (reference ``data/video_loader.py``: ``FrameBuffer``
LRU cache :19-91, ``VideoDataset`` :94-366, ``VideoLoader`` :369-425). Sequences are
sub-directories of frames (``*.png`` / ``*.jpg``) with optional ``controls.npy`` /
``depth/``; PNG sequences are decoded natively in parallel."""
from __future__ import annotations

from collections import OrderedDict
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset


class FrameBuffer:
    def __init__(self, max_frames: int = 1000):
        self.max_frames = max_frames
        self._d: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        self.hits = self.misses = 0

    def get(self, key: str) -> Optional[torch.Tensor]:
        if key in self._d:
            self._d.move_to_end(key)
            self.hits += 1
            return self._d[key]
        self.misses += 1
        return None

    def put(self, key: str, frame: torch.Tensor):
        self._d[key] = frame
        self._d.move_to_end(key)
        while len(self._d) > self.max_frames:
            self._d.popitem(last=False)

    def clear(self):
        self._d.clear()

    def __len__(self):
        return len(self._d)


class VideoDataset(Dataset):
    def __init__(self, root: str, sequence_length: int = 16, image_size: Tuple[int, int] = (256, 256),
                 stride: int = 1, cache_frames: int = 0, load_controls: bool = True):
        self.root = Path(root)
        self.sequence_length, self.image_size, self.stride = sequence_length, tuple(image_size), stride
        self.load_controls = load_controls
        self.buffer = FrameBuffer(cache_frames) if cache_frames else None
        self.sequences: List[Tuple[Path, List[Path]]] = []
        for d in sorted(p for p in self.root.iterdir() if p.is_dir()):
            frames = sorted(list(d.glob("*.png")) + list(d.glob("*.jpg")))
            if len(frames) >= sequence_length:
                self.sequences.append((d, frames))
        self.index = [(si, s) for si, (_, fr) in enumerate(self.sequences)
                      for s in range(0, len(fr) - sequence_length + 1, stride)]

    def __len__(self):
        return len(self.index)

    def _load(self, paths: List[Path]) -> torch.Tensor:
        H, W = self.image_size
        if self.buffer is not None:
            hit = [self.buffer.get(str(p)) for p in paths]
            if all(h is not None for h in hit):
                return torch.stack(hit)
        if all(p.suffix.lower() == ".png" for p in paths):
            from .native import native

            u8 = native().load_frames([str(p) for p in paths], H, W, 0)
        else:
            import cv2

            u8 = torch.from_numpy(np.stack([cv2.resize(cv2.imread(str(p))[:, :, ::-1], (W, H)) for p in paths]))
        fr = u8.permute(0, 3, 1, 2).float().div_(255.0)
        if self.buffer is not None:
            for p, f in zip(paths, fr):
                self.buffer.put(str(p), f)
        return fr

    def __getitem__(self, i) -> Dict[str, Any]:
        si, s = self.index[i]
        d, frames = self.sequences[si]
        out: Dict[str, Any] = {"frames": self._load(frames[s:s + self.sequence_length]),
                               "sequence": d.name, "start": s}
        cp = d / "controls.npy"
        if self.load_controls and cp.exists():
            out["controls"] = torch.from_numpy(np.load(cp)[s:s + self.sequence_length].astype(np.float32))
        return out


class VideoLoader:
    def __init__(self, root: str, batch_size: int = 4, num_workers: int = 2, shuffle: bool = True, **kw):
        self.dataset = VideoDataset(root, **kw)
        self.loader = DataLoader(self.dataset, batch_size=batch_size, shuffle=shuffle, num_workers=num_workers,
                                 drop_last=shuffle)

    def __iter__(self):
        return iter(self.loader)

    def __len__(self):
        return len(self.loader)
