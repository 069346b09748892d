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
from typing import Any, Dict, Iterator, List, Optional, Sequence, Tuple, Union

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
    """Windows of ``sequence_length`` frames ``stride`` frames apart over memory-mapped
    videos (the reference's arguments, data/pipeline.py:134-226): ``video_paths`` are
    video files (cached on first use under ``cache_dir``) or :class:`VideoMemoryMap`
    objects; a window may start at any frame that leaves room for it. Frames are resized
    to ``image_size``; with ``augment``, half of the windows get one brightness /
    contrast change and one horizontal flip decision for all their frames.
    ``controls[i]`` (``[N_i, A]``) adds per-frame controls. Returns ``frames``,
    ``video_idx``, ``start_frame`` (and ``controls``)."""

    def __init__(self, video_paths: Sequence, sequence_length: int = 16,
                 image_size: Tuple[int, int] = (256, 256), cache_dir: Optional[str] = None,
                 stride: int = 1, augment: bool = True, controls: Optional[List[np.ndarray]] = None):
        self.videos = [v if isinstance(v, VideoMemoryMap) else VideoMemoryMap(str(v), cache_dir)
                       for v in video_paths]
        self.video_paths = [str(v.video_path) for v in self.videos]
        self.sequence_length, self.stride = sequence_length, max(1, stride)
        self.image_size = tuple(image_size) if image_size is not None else None
        self.augment, self.controls = augment, controls
        span = (sequence_length - 1) * self.stride + 1
        self.index = [(vi, s) for vi, v in enumerate(self.videos) for s in range(0, len(v) - span + 1)]

    def __len__(self):
        return len(self.index)

    def _augment_sequence(self, frames: torch.Tensor) -> torch.Tensor:
        if random.random() < 0.3:
            gain = 0.8 + 0.4 * random.random()       # contrast
            shift = 0.8 + 0.4 * random.random() - 1  # brightness
            frames = (frames * gain + shift).clamp(0, 1)
        if random.random() < 0.5:
            frames = frames.flip(-1)
        return frames

    def __getitem__(self, i):
        vi, s = self.index[i]
        idx = list(range(s, s + self.sequence_length * self.stride, self.stride))
        frames = self.videos[vi].get_batch(idx)
        if self.image_size is not None and tuple(frames.shape[-2:]) != self.image_size:
            frames = torch.nn.functional.interpolate(frames, size=self.image_size, mode="bilinear",
                                                     align_corners=False)
        if self.augment and random.random() < 0.5:
            frames = self._augment_sequence(frames)
        out = {"frames": frames, "video_idx": vi, "start_frame": s}
        if self.controls is not None:
            out["controls"] = torch.from_numpy(np.asarray(self.controls[vi][idx], dtype=np.float32))
        return out


class StreamingDataLoader:
    """Batches of a dataset staged on the device ahead of use: a background thread pins
    host tensors, copies run on a side stream, and the consumer waits on that stream's
    event only when it takes the batch. Built as the reference's (``dataset, batch_size,
    num_workers, prefetch_factor, pin_memory``, data/pipeline.py:229-265: shuffled, last
    partial batch dropped) or around an existing ``DataLoader`` (``device``, ``prefetch``)."""

    def __init__(self, dataset, batch_size: int = 8, num_workers: int = 4, prefetch_factor: int = 2,
                 pin_memory: bool = True, device="cuda", prefetch: Optional[int] = None):
        if isinstance(dataset, DataLoader):
            loader = dataset
        else:
            kw = dict(prefetch_factor=prefetch_factor, persistent_workers=True) if num_workers > 0 else {}
            loader = DataLoader(dataset, batch_size=batch_size, shuffle=True, num_workers=num_workers,
                                drop_last=True, **kw)
        self.dataset = getattr(loader, "dataset", dataset)
        self.batch_size, self.pin_memory = batch_size, pin_memory
        self.loader = self.dataloader = loader
        self.device = torch.device(device if (str(device) != "cuda" or torch.cuda.is_available()) else "cpu")
        self.prefetch = prefetch if prefetch is not None else max(1, prefetch_factor)

    def __len__(self):
        return len(self.loader)

    def _to_device(self, batch, stream):
        def mv(x):
            if torch.is_tensor(x):
                if self.device.type == "cuda" and not x.is_pinned():
                    x = x.pin_memory()
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
    def split_by_video(video_paths: Sequence[str], train_ratio: float = 0.8, val_ratio: float = 0.1,
                       seed: Optional[int] = None) -> Tuple[List[str], List[str], List[str]]:
        """Whole videos to train / val / test (no window of one video in two splits)."""
        paths = list(video_paths)
        random.Random(seed).shuffle(paths)
        n_tr, n_va = int(len(paths) * train_ratio), int(len(paths) * val_ratio)
        return paths[:n_tr], paths[n_tr:n_tr + n_va], paths[n_tr + n_va:]

    @staticmethod
    def create_datasets(video_paths: Sequence[str], sequence_length: int = 16,
                        image_size: Tuple[int, int] = (256, 256), cache_dir: Optional[str] = None,
                        seed: Optional[int] = None, **kwargs):
        """(train, val, test) :class:`DrivingDataset` of a video-level split; augmentation
        on the training set only."""
        tr, va, te = DatasetSplitter.split_by_video(video_paths, seed=seed)
        return tuple(DrivingDataset(p, sequence_length, image_size, cache_dir, augment=(i == 0), **kwargs)
                     for i, p in enumerate((tr, va, te)))

    @staticmethod
    def split(dataset: Dataset, ratios: Sequence[float] = (0.8, 0.1, 0.1), seed: int = 0) -> List[Subset]:
        """Random subsets of a dataset's items in the given proportions."""
        n = len(dataset)
        perm = torch.randperm(n, generator=torch.Generator().manual_seed(seed)).tolist()
        out, s = [], 0
        for i, r in enumerate(ratios):
            e = n if i == len(ratios) - 1 else s + int(round(r * n))
            out.append(Subset(dataset, perm[s:e]))
            s = e
        return out


def create_efficient_pipeline(video_dir: Union[str, Path, Sequence], batch_size: int = 8,
                              sequence_length: int = 16, image_size: Tuple[int, int] = (256, 256),
                              cache_dir: Optional[str] = None, num_workers: int = 4, device="cuda",
                              seed: Optional[int] = None):
    """(train, val, test) :class:`StreamingDataLoader` over the ``*.mp4`` / ``*.avi`` /
    ``*.mov`` videos of ``video_dir`` (or a list of paths / :class:`VideoMemoryMap`),
    split by video (data/pipeline.py:341-381)."""
    if isinstance(video_dir, (str, Path)):
        d = Path(video_dir)
        videos = sorted(str(p) for ext in ("*.mp4", "*.avi", "*.mov") for p in d.glob(ext))
    else:
        videos = list(video_dir)
    splits = DatasetSplitter.create_datasets(videos, sequence_length, image_size, cache_dir, seed=seed)
    return tuple(StreamingDataLoader(ds, batch_size, num_workers, device=device) for ds in splits)
