"""Memory-mapped video datasets and a prefetching device loader.

Capabilities of the reference ``data/pipeline.py`` (``VideoMemoryMap`` :20-131,
``DrivingDataset`` :134-226, ``StreamingDataLoader`` :229-265, ``DatasetSplitter``
:268-311, ``create_efficient_pipeline`` :341+). Differences by design: the frame cache
is raw uint8 ``[N, H, W, 3]`` in a ``numpy.memmap`` (no JPEG re-decode on every access;
the reference's index header format string ``'IFII'`` is not a valid ``struct`` format),
and the loader overlaps host->device copies with compute on a side CUDA stream from
pinned buffers.
"""
from __future__ import annotations

import json
import queue
import random
import threading
from pathlib import Path
from typing import Any, Dict, Iterator, List, Optional, Sequence, Tuple

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset, Subset


class VideoMemoryMap:
    """Frames of a video (or of an image array) cached once as a uint8 memmap."""

    def __init__(self, video_path: str, cache_dir: Optional[str] = None, frames: Optional[np.ndarray] = None):
        self.video_path = Path(video_path)
        self.cache_dir = Path(cache_dir) if cache_dir else self.video_path.parent / "cache"
        self.cache_dir.mkdir(parents=True, exist_ok=True)
        self.index_path = self.cache_dir / f"{self.video_path.stem}.json"
        self.data_path = self.cache_dir / f"{self.video_path.stem}.u8"
        if not (self.index_path.exists() and self.data_path.exists()):
            self._build_cache(frames)
        meta = json.loads(self.index_path.read_text())
        self.frame_count, self.fps = meta["frame_count"], meta["fps"]
        self.height, self.width = meta["height"], meta["width"]
        self.data = np.memmap(self.data_path, dtype=np.uint8, mode="r",
                              shape=(self.frame_count, self.height, self.width, 3))

    def _build_cache(self, frames: Optional[np.ndarray]):
        fps = 30.0
        if frames is None:
            import cv2

            cap = cv2.VideoCapture(str(self.video_path))
            fps = cap.get(cv2.CAP_PROP_FPS) or fps
            fr = []
            while True:
                ok, f = cap.read()
                if not ok:
                    break
                fr.append(f[:, :, ::-1])
            cap.release()
            if not fr:
                raise IOError(f"could not decode {self.video_path}")
            frames = np.stack(fr)
        frames = np.ascontiguousarray(frames, dtype=np.uint8)
        mm = np.memmap(self.data_path, dtype=np.uint8, mode="w+", shape=frames.shape)
        mm[:] = frames
        mm.flush()
        self.index_path.write_text(json.dumps({"frame_count": int(frames.shape[0]), "fps": float(fps),
                                               "height": int(frames.shape[1]), "width": int(frames.shape[2])}))

    def __len__(self):
        return self.frame_count

    def get_frame(self, idx: int) -> np.ndarray:
        if idx >= self.frame_count:
            raise IndexError(f"Frame {idx} >= {self.frame_count}")
        return np.asarray(self.data[idx])

    def get_batch(self, indices: Sequence[int]) -> torch.Tensor:
        """``[B, 3, H, W]`` float in [0, 1]."""
        u8 = torch.from_numpy(np.ascontiguousarray(self.data[list(indices)]))
        return u8.permute(0, 3, 1, 2).float().div_(255.0)


class DrivingDataset(Dataset):
    """Windows of ``sequence_length`` frames (+ per-frame controls) over memory-mapped
    videos; ``controls[i]`` is an ``[N_i, A]`` array for video ``i``."""

    def __init__(self, videos: List[VideoMemoryMap], controls: Optional[List[np.ndarray]] = None,
                 sequence_length: int = 16, stride: int = 1):
        self.videos, self.controls = videos, controls
        self.sequence_length, self.stride = sequence_length, stride
        self.index = [(vi, s) for vi, v in enumerate(videos)
                      for s in range(0, len(v) - sequence_length + 1, stride)]

    def __len__(self):
        return len(self.index)

    def __getitem__(self, i):
        vi, s = self.index[i]
        idx = list(range(s, s + self.sequence_length))
        out = {"frames": self.videos[vi].get_batch(idx)}
        if self.controls is not None:
            out["controls"] = torch.from_numpy(np.asarray(self.controls[vi][s:s + self.sequence_length],
                                                          dtype=np.float32))
        return out


class StreamingDataLoader:
    """Iterates a DataLoader and stages each batch on the device ahead of use: a
    background thread pins host tensors, copies run on a side stream, and the consumer
    waits on that stream's event only when it takes the batch."""

    def __init__(self, loader: DataLoader, device="cuda", prefetch: int = 2):
        self.loader, self.device, self.prefetch = loader, torch.device(device), prefetch

    def __len__(self):
        return len(self.loader)

    def _to_device(self, batch, stream):
        def mv(x):
            if torch.is_tensor(x):
                x = x.pin_memory() if not x.is_pinned() else x
                return x.to(self.device, non_blocking=True)
            if isinstance(x, dict):
                return {k: mv(v) for k, v in x.items()}
            if isinstance(x, (list, tuple)):
                return type(x)(mv(v) for v in x)
            return x

        if stream is None:
            return mv(batch), None
        with torch.cuda.stream(stream):
            b = mv(batch)
            ev = torch.cuda.Event()
            ev.record(stream)
        return b, ev

    def __iter__(self) -> Iterator[Any]:
        use_cuda = self.device.type == "cuda" and torch.cuda.is_available()
        stream = torch.cuda.Stream(device=self.device) if use_cuda else None
        q: "queue.Queue" = queue.Queue(maxsize=self.prefetch)
        stop = object()

        def producer():
            try:
                for b in self.loader:
                    q.put(self._to_device(b, stream))
            finally:
                q.put((stop, None))

        th = threading.Thread(target=producer, daemon=True)
        th.start()
        while True:
            b, ev = q.get()
            if b is stop:
                break
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
            yield b
        th.join()


class DatasetSplitter:
    @staticmethod
    def split(dataset: Dataset, ratios: Sequence[float] = (0.8, 0.1, 0.1), seed: int = 0) -> List[Subset]:
        n = len(dataset)
        perm = torch.randperm(n, generator=torch.Generator().manual_seed(seed)).tolist()
        out, s = [], 0
        for i, r in enumerate(ratios):
            e = n if i == len(ratios) - 1 else s + int(round(r * n))
            out.append(Subset(dataset, perm[s:e]))
            s = e
        return out


def create_efficient_pipeline(videos: List[VideoMemoryMap], controls=None, sequence_length: int = 16,
                              batch_size: int = 4, num_workers: int = 2, device="cuda",
                              split=(0.9, 0.1), seed: int = 0):
    ds = DrivingDataset(videos, controls, sequence_length)
    parts = DatasetSplitter.split(ds, split, seed)
    mk = lambda d, sh: StreamingDataLoader(DataLoader(d, batch_size=batch_size, shuffle=sh,
                                                      num_workers=num_workers, drop_last=sh), device)
    return [mk(p, i == 0) for i, p in enumerate(parts)]
