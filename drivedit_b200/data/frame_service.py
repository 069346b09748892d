"""Background frame loading (the reference's Rust ``frame_loader.rs`` ``FrameLoaderService``
and ``frame.rs`` ``FrameRingBuffer``): decode + resize in native worker threads while the
trainer runs, with an LRU cache of decoded frames shared by overlapping clips."""
from __future__ import annotations

from collections import deque
from typing import List, Optional, Sequence, Tuple

import torch

from .native import native


class FrameRequest:
    """A submitted batch; ``result()`` blocks until its frames are decoded."""

    def __init__(self, service, rid: int, out: torch.Tensor):
        self._svc, self._id, self._out, self._done = service, rid, out, False

    def done(self) -> bool:
        return self._done or self._svc.done(self._id)

    def result(self) -> torch.Tensor:
        """``uint8 [N, H, W, 3]``; raises the decode error if a frame failed."""
        if not self._done:
            self._svc.wait(self._id)
            self._done = True
        return self._out


class FrameLoaderService:
    def __init__(self, threads: int = 0, cache_frames: int = 256):
        self._svc = native().FrameLoaderService(threads, cache_frames)

    def submit(self, paths: Sequence[str], height: int, width: int) -> FrameRequest:
        rid, out = self._svc.submit([str(p) for p in paths], height, width)
        return FrameRequest(self._svc, rid, out)

    def load(self, paths: Sequence[str], height: int, width: int) -> torch.Tensor:
        return self.submit(paths, height, width).result()

    def pending(self) -> int:
        return self._svc.pending()

    def cache_stats(self):
        return self._svc.cache_stats()

    def clear_cache(self):
        self._svc.clear_cache()


class FrameRingBuffer:
    """The newest ``capacity`` frames (e.g. a streaming context window)."""

    def __init__(self, capacity: int):
        self.capacity = capacity
        self._buf: deque = deque(maxlen=capacity)

    def push(self, frame: torch.Tensor) -> None:
        self._buf.append(frame)

    def latest(self, n: Optional[int] = None) -> torch.Tensor:
        items = list(self._buf)[-(n or len(self._buf)):]
        return torch.stack(items)

    def __len__(self) -> int:
        return len(self._buf)

    def is_full(self) -> bool:
        return len(self._buf) == self.capacity

    def clear(self) -> None:
        self._buf.clear()
