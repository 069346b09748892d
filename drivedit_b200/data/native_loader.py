"""Native-runtime dataset front ends (the reference's ``data/rust_loader.py`` and
``data/hybrid_loader.py`` interfaces: ``RustDatasetConfig``, ``RustEnfusionDataset``,
``RustCollator``, ``RustDataLoader``, ``RustBatchLoader``, ``create_rust_dataloaders``,
``benchmark_rust_vs_python``, ``check_rust_available``, ``get_rust_version``;
``HybridLoaderConfig``, ``PerformanceTracker``, ``HybridDataLoader``,
``create_hybrid_dataloaders``, ``get_best_loader``).

The compiled runtime here is the C++ extension ``drivedit_b200._data`` (ENFCAP, telemetry,
PNG / depth decoding, the background frame service), so the ``Rust*`` names are aliases of
the ``Native*`` classes. :class:`NativeBatchLoader` assembles a batch by submitting every
frame of every sample in one request to the native :class:`FrameLoaderService` (decode +
resize on worker threads without the GIL) and prefetches the next batch while the current
one is consumed. The reference's ``GoPrefetchClient`` is a gRPC stub that never prefetches;
its role is taken by that service.
"""
from __future__ import annotations

import logging
import random
import time
from collections import defaultdict, deque
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np
import torch
from torch.utils.data import DataLoader

from .enfusion import EnfusionCollator, EnfusionDataset, EnfusionDatasetConfig
from .native import available


def check_native_available() -> bool:
    return available()


def get_native_version() -> Optional[str]:
    return "drivedit_b200._data (C++ data runtime)" if available() else None


@dataclass
class NativeDatasetConfig:
    sequence_length: int = 16
    frame_skip: int = 1
    image_height: int = 256
    image_width: int = 256
    load_depth: bool = True
    load_controls: bool = True
    control_dim: int = 6
    normalize_frames: bool = True
    cache_frames: bool = True
    max_cache_mb: float = 1000.0
    num_workers: int = 4

    @property
    def image_size(self) -> Tuple[int, int]:
        return (self.image_height, self.image_width)

    def to_enfusion_config(self) -> EnfusionDatasetConfig:
        return EnfusionDatasetConfig(sequence_length=self.sequence_length, frame_skip=self.frame_skip,
                                     image_size=self.image_size, load_depth=self.load_depth,
                                     load_controls=self.load_controls, control_dim=self.control_dim,
                                     normalize_frames=self.normalize_frames, cache_frames=self.cache_frames,
                                     max_cache_memory_mb=self.max_cache_mb, loader_threads=self.num_workers,
                                     augment=False, load_scene=False)


class NativeEnfusionDataset(EnfusionDataset):
    """:class:`EnfusionDataset` configured from a :class:`NativeDatasetConfig`."""

    def __init__(self, data_root, config: Optional[NativeDatasetConfig] = None, split: str = "train", **kw):
        self.native_config = config or NativeDatasetConfig()
        super().__init__(data_root, self.native_config.to_enfusion_config(), split, **kw)

    def frame_paths(self, i: int) -> List[str]:
        c = self.config
        si, st = self.index[i]
        s = self.sessions[si]
        return [str(s.frame_paths[st + k * c.frame_skip]) for k in range(c.sequence_length)]


class NativeCollator(EnfusionCollator):
    def __init__(self, include_depth: bool = True):
        super().__init__()
        self.include_depth = include_depth

    def __call__(self, batch):
        out = super().__call__(batch)
        if not self.include_depth:
            out.pop("depth", None)
        return out


class NativeDataLoader(DataLoader):
    """A torch DataLoader over a native dataset with its collator."""

    def __init__(self, dataset: NativeEnfusionDataset, batch_size: int = 8, shuffle: bool = True,
                 num_workers: int = 0, drop_last: bool = True, **kw):
        super().__init__(dataset, batch_size=batch_size, shuffle=shuffle, num_workers=num_workers,
                         drop_last=drop_last, collate_fn=NativeCollator(dataset.config.load_depth), **kw)


class NativeBatchLoader:
    """Batches without a DataLoader: one frame-service request per batch (all samples'
    frames decoded in parallel), the next batch in flight while this one is used."""

    def __init__(self, dataset: NativeEnfusionDataset, batch_size: int = 8, shuffle: bool = True,
                 drop_last: bool = True, threads: int = 0, seed: int = 0):
        from .frame_service import FrameLoaderService

        self.dataset, self.batch_size, self.shuffle, self.drop_last = dataset, batch_size, shuffle, drop_last
        self.service = FrameLoaderService(threads, cache_frames=0)
        self.rng = random.Random(seed)

    def __len__(self) -> int:
        n = len(self.dataset)
        return n // self.batch_size if self.drop_last else (n + self.batch_size - 1) // self.batch_size

    def _submit(self, idxs: List[int]):
        H, W = self.dataset.config.image_size
        paths = [p for i in idxs for p in self.dataset.frame_paths(i)]
        if not all(p.lower().endswith(".png") for p in paths):
            return idxs, None
        return idxs, self.service.submit(paths, H, W)

    def _finish(self, idxs, req) -> Dict[str, object]:
        ds = self.dataset
        c = ds.config
        T = c.sequence_length
        if req is None:               # non-PNG frames: the dataset's own decoder
            frames = torch.stack([ds.sessions[ds.index[i][0]].load_frames(
                [ds.index[i][1] + k * c.frame_skip for k in range(T)]) for i in idxs])
        else:
            u8 = req.result()
            frames = u8.view(len(idxs), T, *u8.shape[1:]).permute(0, 1, 4, 2, 3).float().div_(255.0)
        ctrl, ego, anchors, depth = [], [], [], []
        for i in idxs:
            si, st = ds.index[i]
            s = ds.sessions[si]
            idx = [st + k * c.frame_skip for k in range(T)]
            ctrl.append(s.controls[idx])
            ego.append(s.ego_transforms[idx])
            anchors.append(s.anchor_mask(st, idx))
            if c.load_depth:
                d = s.load_depth(idx)
                if d is not None:
                    depth.append(d)
        out = {"frames": frames, "controls": torch.stack(ctrl), "ego_transform": torch.stack(ego),
               "anchor_mask": torch.stack(anchors)}
        if depth and len(depth) == len(idxs):
            out["depth"] = torch.stack(depth)
        return out

    def __iter__(self) -> Iterator[Dict[str, object]]:
        order = list(range(len(self.dataset)))
        if self.shuffle:
            self.rng.shuffle(order)
        batches = [order[i:i + self.batch_size] for i in range(0, len(order), self.batch_size)]
        if self.drop_last and batches and len(batches[-1]) < self.batch_size:
            batches.pop()
        pending = deque()
        for b in batches[:2]:
            pending.append(self._submit(b))
        nxt = 2
        while pending:
            idxs, req = pending.popleft()
            if nxt < len(batches):
                pending.append(self._submit(batches[nxt]))
                nxt += 1
            yield self._finish(idxs, req)


def create_native_dataloaders(data_root, config: Optional[NativeDatasetConfig] = None, batch_size: int = 8,
                              val_fraction: float = 0.1, seed: int = 0):
    """(train, val) batch loaders split by session."""
    cfg = config or NativeDatasetConfig()
    full = NativeEnfusionDataset(data_root, cfg)
    names = sorted({s.session_dir.name for s in full.sessions})
    rng = random.Random(seed)
    rng.shuffle(names)
    n_val = max(1, int(len(names) * val_fraction)) if len(names) > 1 else 0
    val_ids, train_ids = names[:n_val], names[n_val:]
    train = NativeEnfusionDataset(data_root, cfg, "train", session_ids=train_ids)
    loaders = [NativeBatchLoader(train, batch_size, True, True, seed=seed)]
    if val_ids:
        val = NativeEnfusionDataset(data_root, cfg, "val", session_ids=val_ids)
        loaders.append(NativeBatchLoader(val, batch_size, False, False))
    else:
        loaders.append(None)
    return tuple(loaders)


def benchmark_native_vs_python(data_root, config: Optional[NativeDatasetConfig] = None, batch_size: int = 4,
                               num_batches: int = 5) -> Dict[str, float]:
    """Batches per second of the native batch loader and of a plain per-sample Python path
    (PIL decode + resize) over the same samples."""
    from PIL import Image

    cfg = config or NativeDatasetConfig()
    ds = NativeEnfusionDataset(data_root, cfg)
    nb = min(num_batches, len(ds) // batch_size)
    t0 = time.perf_counter()
    for k, _ in enumerate(NativeBatchLoader(ds, batch_size, shuffle=False)):
        if k + 1 >= nb:
            break
    t_native = time.perf_counter() - t0
    H, W = cfg.image_size
    t0 = time.perf_counter()
    for b in range(nb):
        for i in range(b * batch_size, (b + 1) * batch_size):
            np.stack([np.asarray(Image.open(p).convert("RGB").resize((W, H), Image.BILINEAR))
                      for p in ds.frame_paths(i)])
    t_py = time.perf_counter() - t0
    return {"native_batches_per_s": nb / max(t_native, 1e-9), "python_batches_per_s": nb / max(t_py, 1e-9),
            "speedup": t_py / max(t_native, 1e-9)}


# ----------------------------------------------------------------------------- hybrid
@dataclass
class HybridLoaderConfig:
    """The reference's loader settings (data/hybrid_loader.py:63-125). ``prefer_rust``
    selects the native (C++) runtime when it is built; ``use_batch_loader`` its batch
    loader (one native call decodes a whole batch). The Go prefetch-service fields are
    accepted and unused: there is no such service; the native loader prefetches."""
    sequence_length: int = 16
    frame_skip: int = 1
    image_size: Tuple[int, int] = (256, 256)
    load_depth: bool = True
    load_controls: bool = True
    control_dim: int = 6
    batch_size: int = 8
    num_workers: int = 4
    shuffle: bool = True
    drop_last: bool = True
    pin_memory: bool = True
    prefetch_factor: int = 2
    cache_frames: bool = True
    max_cache_mb: float = 1000.0
    prefer_rust: bool = True
    use_batch_loader: bool = True
    go_prefetch_enabled: bool = False
    go_prefetch_address: str = "localhost:50051"
    go_prefetch_buffer_size: int = 16
    track_performance: bool = True
    log_interval: int = 100

    @property
    def prefer_native(self) -> bool:
        return self.prefer_rust

    def to_rust_config(self) -> NativeDatasetConfig:
        return NativeDatasetConfig(sequence_length=self.sequence_length, frame_skip=self.frame_skip,
                                   image_height=self.image_size[0], image_width=self.image_size[1],
                                   load_depth=self.load_depth, load_controls=self.load_controls,
                                   control_dim=self.control_dim, cache_frames=self.cache_frames,
                                   max_cache_mb=self.max_cache_mb, num_workers=self.num_workers)

    to_native_config = to_rust_config

    def to_python_config(self) -> EnfusionDatasetConfig:
        return self.to_rust_config().to_enfusion_config()


class PerformanceTracker:
    """Batch load times and throughput; a summary is logged every ``log_interval``
    batches."""

    def __init__(self, log_interval: int = 100):
        self.log_interval = log_interval
        self.reset()

    def reset(self):
        self.load_times: List[float] = []
        self.batch_count = self.total_samples = 0
        self.start_time = time.time()

    def record_batch(self, load_time: float, batch_size: int):
        self.load_times.append(load_time)
        self.batch_count += 1
        self.total_samples += batch_size
        if self.log_interval and self.batch_count % self.log_interval == 0:
            st = self.get_stats()
            logging.getLogger(__name__).info("batch %d: %.1f ms per batch, %.1f samples/s", self.batch_count,
                                             st["avg_load_time_ms"], st["samples_per_sec"])

    def get_stats(self) -> Dict[str, float]:
        if not self.load_times:
            return {}
        dt = time.time() - self.start_time
        return {"batch_count": self.batch_count, "total_samples": self.total_samples, "total_time_sec": dt,
                "avg_load_time_ms": float(np.mean(self.load_times)) * 1000.0,
                "samples_per_sec": self.total_samples / dt if dt > 0 else 0.0}


class HybridDataLoader:
    """The native batch loader when the runtime is built (and preferred), else a torch
    DataLoader over the Python dataset (data/hybrid_loader.py:255-427); records the time
    each batch took to arrive."""

    def __init__(self, data_root, config: Optional[HybridLoaderConfig] = None, split: str = "train",
                 session_ids: Optional[List[str]] = None):
        self.data_root = Path(data_root)
        self.config = c = config or HybridLoaderConfig()
        self.split, self.session_ids = split, session_ids
        self._use_native = c.prefer_rust and available()
        self._backend_name = "rust" if self._use_native else "python"
        self._performance_tracker = PerformanceTracker(c.log_interval) if c.track_performance else None
        self._loader = self._create_loader()

    def _create_loader(self):
        c = self.config
        if self._use_native:
            ds = NativeEnfusionDataset(self.data_root, c.to_rust_config(), self.split, session_ids=self.session_ids)
            if c.use_batch_loader:
                return NativeBatchLoader(ds, c.batch_size, shuffle=c.shuffle and len(ds) > 0)
            return NativeDataLoader(ds, c.batch_size, shuffle=c.shuffle and len(ds) > 0, num_workers=c.num_workers)
        ds = EnfusionDataset(self.data_root, c.to_python_config(), self.split, self.session_ids)
        kw = dict(prefetch_factor=c.prefetch_factor) if c.num_workers > 0 else {}
        return DataLoader(ds, batch_size=c.batch_size, shuffle=c.shuffle and len(ds) > 0,
                          drop_last=c.drop_last, num_workers=c.num_workers,
                          pin_memory=c.pin_memory and torch.cuda.is_available(),
                          collate_fn=EnfusionCollator(), **kw)

    @property
    def backend(self) -> str:
        return self._backend_name

    @property
    def is_rust(self) -> bool:
        return self._use_native

    def __iter__(self):
        t = time.perf_counter()
        for b in self._loader:
            now = time.perf_counter()
            if self._performance_tracker is not None:
                x = b.get("frames", b.get("controls")) if isinstance(b, dict) else None
                self._performance_tracker.record_batch(now - t, int(x.shape[0]) if x is not None else 0)
            t = now
            yield b

    def __len__(self):
        return len(self._loader)

    def get_performance_stats(self) -> Dict[str, float]:
        return self._performance_tracker.get_stats() if self._performance_tracker is not None else {}

    def reset_performance_stats(self):
        if self._performance_tracker is not None:
            self._performance_tracker.reset()

    def cache_stats(self) -> Dict[str, float]:
        for obj in (self._loader, getattr(self._loader, "dataset", None)):
            if obj is not None and hasattr(obj, "cache_stats"):
                return obj.cache_stats()
        return {}

    def clear_cache(self):
        for obj in (self._loader, getattr(self._loader, "dataset", None)):
            if obj is not None and hasattr(obj, "clear_cache"):
                obj.clear_cache()
                return

    def close(self):
        pass


def create_hybrid_dataloaders(data_root, config: Optional[HybridLoaderConfig] = None,
                              train_ratio: float = 0.8, val_ratio: float = 0.1, seed: Optional[int] = None):
    """(train, val, test) loaders from ``train/`` / ``val/`` (/ ``test/``) folders or a
    session-level split of ``session_*``; validation and test are not shuffled."""
    from dataclasses import replace

    root = Path(data_root)
    config = config or HybridLoaderConfig()
    evalc = replace(config, shuffle=False)
    if (root / "train").is_dir() and (root / "val").is_dir():
        return (HybridDataLoader(root / "train", config, "train"),
                HybridDataLoader(root / "val", evalc, "val"),
                HybridDataLoader(root / "test" if (root / "test").is_dir() else root / "val", evalc, "test"))
    names = sorted(p.name for p in root.glob("session_*") if p.is_dir())
    random.Random(seed).shuffle(names)
    n_tr, n_va = int(len(names) * train_ratio), int(len(names) * val_ratio)
    return (HybridDataLoader(root, config, "train", names[:n_tr]),
            HybridDataLoader(root, evalc, "val", names[n_tr:n_tr + n_va]),
            HybridDataLoader(root, evalc, "test", names[n_tr + n_va:]))


def get_best_loader(data_root, batch_size: int = 8, sequence_length: int = 16,
                    image_size: Tuple[int, int] = (256, 256), **kwargs) -> HybridDataLoader:
    """One loader on the fastest available backend (other :class:`HybridLoaderConfig`
    fields by keyword)."""
    return HybridDataLoader(data_root, HybridLoaderConfig(batch_size=batch_size, sequence_length=sequence_length,
                                                          image_size=tuple(image_size), **kwargs))


# names of the reference's compiled-loader API
RustDatasetConfig = NativeDatasetConfig
RustEnfusionDataset = NativeEnfusionDataset
RustCollator = NativeCollator
RustDataLoader = NativeDataLoader
RustBatchLoader = NativeBatchLoader
create_rust_dataloaders = create_native_dataloaders
benchmark_rust_vs_python = benchmark_native_vs_python
check_rust_available = check_native_available
get_rust_version = get_native_version
