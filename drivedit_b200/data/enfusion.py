"""Enfusion capture sessions as a PyTorch dataset.

Session layout and sample contract of the reference (data/enfusion_loader.py:6-30,
:59-296, :299-615): a session directory holds ``telemetry.csv``, ``frames/*.png|jpg``,
optionally ``capture.enfcap``, ``depth/*.npz``, ``scene/*.json`` and
``session_info.txt`` / ``metadata.json``. A sample is a window of ``sequence_length``
frames (stride ``frame_skip``):

    {'frames': [T, 3, H, W] float [0,1], 'controls': [T, 6] [-1,1],
     'ego_transform': [T, 4, 4], 'depth': [T, 1, H, W] (optional),
     'anchor_mask': [T] bool, 'scene_entities': list, 'metadata': dict}

PNG frames are decoded and resized by the native loader on worker threads
(csrc/data/frames.cpp); other formats fall back to OpenCV. Telemetry is parsed natively
and resampled to the frame count. When a session has a ``capture.enfcap`` file, ego
transforms, anchor flags and scene entities come from it.
"""
from __future__ import annotations

import json
import random
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple, Union

import numpy as np
import torch
import torch.nn.functional as F
from torch.utils.data import DataLoader, Dataset

from .native import native
from .telemetry import ControlNormalizer, TelemetryConfig, TelemetryParser


@dataclass
class EnfusionDatasetConfig:
    sequence_length: int = 16
    frame_skip: int = 1
    image_size: Tuple[int, int] = (256, 256)
    load_depth: bool = True
    load_scene: bool = True
    load_controls: bool = True
    control_dim: int = 6
    normalize_frames: bool = True
    normalize_controls: bool = True
    min_quality_score: float = 0.5
    filter_sessions: bool = True
    cache_frames: bool = True
    cache_telemetry: bool = True
    max_cache_memory_mb: float = 1000.0
    max_depth: float = 100.0
    depth_format: str = "npz"
    telemetry_config: TelemetryConfig = field(default_factory=TelemetryConfig)
    augment: bool = True
    horizontal_flip_prob: float = 0.5
    brightness_range: Tuple[float, float] = (0.9, 1.1)
    contrast_range: Tuple[float, float] = (0.9, 1.1)
    loader_threads: int = 0


class AnchorDetector:
    """Anchor (key) frames: ENFCAP anchor flags when present, else frames where the
    normalised controls change sharply (steering / acceleration jumps) or every
    ``max_interval`` frames. The reference's detector, with its own thresholds and API, is
    :class:`drivedit_b200.data.enfusion_preprocessing.EnfusionAnchorDetector`."""

    def __init__(self, steering_threshold: float = 0.3, accel_threshold: float = 0.5,
                 min_interval: int = 4, max_interval: int = 32):
        self.steering_threshold, self.accel_threshold = steering_threshold, accel_threshold
        self.min_interval, self.max_interval = min_interval, max_interval

    def detect(self, controls: torch.Tensor) -> torch.Tensor:
        T = controls.shape[0]
        mask = torch.zeros(T, dtype=torch.bool)
        if T == 0:
            return mask
        mask[0] = True
        d = (controls[1:] - controls[:-1]).abs()
        jump = (d[:, 0] > self.steering_threshold) | (d[:, 1] > self.accel_threshold)
        last = 0
        for t in range(1, T):
            if (bool(jump[t - 1]) and t - last >= self.min_interval) or t - last >= self.max_interval:
                mask[t] = True
                last = t
        return mask




class EnfusionSession:
    def __init__(self, session_dir: Union[str, Path], config: EnfusionDatasetConfig):
        self.session_dir = Path(session_dir)
        self.config = config
        if not self.session_dir.exists():
            raise FileNotFoundError(f"Session directory not found: {self.session_dir}")
        if not (self.session_dir / "frames").exists():
            raise FileNotFoundError(f"Frames directory not found: {self.session_dir / 'frames'}")
        self.metadata = self._load_metadata()
        self.frame_paths = self._glob("frames", ("*.png", "*.jpg", "*.jpeg"))
        self.depth_paths = self._glob("depth", ("*.npz", "*.npy", "*.png")) if config.load_depth else []
        self.scene_paths = self._glob("scene", ("*.json",)) if config.load_scene else []
        self.parser = TelemetryParser(config.telemetry_config)
        self.normalizer = ControlNormalizer(config.telemetry_config)
        self.anchor_detector = AnchorDetector()
        self._telemetry = self._controls = self._ego = self._enfcap = None

    def _glob(self, sub: str, pats) -> List[Path]:
        d = self.session_dir / sub
        if not d.exists():
            return []
        out: List[Path] = []
        for p in pats:
            out.extend(d.glob(p))
        return sorted(out)

    def _load_metadata(self) -> Dict[str, Any]:
        md: Dict[str, Any] = {"session_id": self.session_dir.name, "path": str(self.session_dir)}
        info = self.session_dir / "session_info.txt"
        if info.exists():
            for line in info.read_text(errors="ignore").splitlines():
                if ":" in line:
                    k, v = line.split(":", 1)
                    md[k.strip()] = v.strip()
        js = self.session_dir / "metadata.json"
        if js.exists():
            try:
                md.update(json.loads(js.read_text()))
            except json.JSONDecodeError:
                pass
        return md

    @property
    def num_frames(self) -> int:
        return len(self.frame_paths)

    @property
    def enfcap(self):
        p = self.session_dir / "capture.enfcap"
        if self._enfcap is None and p.exists():
            from .enfcap import ENFCAPReader

            self._enfcap = ENFCAPReader(str(p))
        return self._enfcap

    @property
    def telemetry(self) -> Dict[str, np.ndarray]:
        if self._telemetry is None:
            p = self.session_dir / "telemetry.csv"
            N = self.num_frames
            if p.exists():
                tel = self.parser.parse_csv(p)
                self._telemetry = self.parser.interpolate_to_frame_rate(tel, N)
            else:
                z = np.zeros(N, np.float32)
                self._telemetry = {"timestamp": np.linspace(0, N / 30.0, N).astype(np.float32),
                                   "position": np.zeros((N, 3), np.float32),
                                   "rotation": np.zeros((N, 3), np.float32),
                                   "steering": z, "throttle": z, "brake": z, "speed": z}
        return self._telemetry

    @property
    def controls(self) -> torch.Tensor:
        if self._controls is None:
            self._controls = self.normalizer.normalize_controls(self.telemetry, self.config.control_dim)
        return self._controls

    @property
    def ego_transforms(self) -> torch.Tensor:
        if self._ego is None:
            r = self.enfcap
            if r is not None and r.frame_count >= self.num_frames:
                ego = r.read_frames(0, self.num_frames)["ego_transform"]
                T = torch.eye(4).repeat(self.num_frames, 1, 1)
                T[:, :3, :] = ego
                self._ego = T
            else:
                t = self.telemetry
                self._ego = torch.from_numpy(self.parser.compute_ego_transform(t["position"], t["rotation"]))
        return self._ego

    def anchor_mask(self, start: int, idx: List[int]) -> torch.Tensor:
        r = self.enfcap
        if r is not None and r.frame_count >= self.num_frames:
            fl = r.read_frames(min(idx), max(idx) + 1)["flags"]
            return (fl[torch.tensor(idx) - min(idx)] & 1).bool()
        return self.anchor_detector.detect(self.controls[idx])

    def get_valid_start_indices(self, sequence_length: int, frame_skip: int = 1) -> List[int]:
        need = (sequence_length - 1) * frame_skip + 1
        return list(range(self.num_frames - need + 1)) if self.num_frames >= need else []

    def load_frames(self, idx: List[int]) -> torch.Tensor:
        """``[T, 3, H, W]`` float in [0, 1]."""
        H, W = self.config.image_size
        paths = [str(self.frame_paths[i]) for i in idx]
        if all(p.lower().endswith(".png") for p in paths):
            u8 = native().load_frames(paths, H, W, self.config.loader_threads)
        else:
            import cv2

            arr = []
            for p in paths:
                im = cv2.imread(p, cv2.IMREAD_COLOR)[:, :, ::-1]
                arr.append(cv2.resize(im, (W, H), interpolation=cv2.INTER_LINEAR))
            u8 = torch.from_numpy(np.stack(arr))
        return u8.permute(0, 3, 1, 2).float().div_(255.0)

    def load_depth(self, idx: List[int]) -> Optional[torch.Tensor]:
        """``[T, 1, H, W]`` depth clipped to ``[0, max_depth]`` and scaled to [0, 1]; decoded
        and resized by the native depth loader when it is built."""
        if not self.depth_paths:
            return None
        H, W = self.config.image_size
        paths = [self.depth_paths[min(i, len(self.depth_paths) - 1)] for i in idx]
        from .native import available

        if available():
            from .depth import DepthLoader, DepthLoaderConfig

            cfg = DepthLoaderConfig(target_width=W, target_height=H, min_depth=0.0,
                                    max_depth=self.config.max_depth, npz_array_name="")
            return DepthLoader(cfg).load_batch_contiguous(paths, self.config.loader_threads)[:, None]
        out = []
        for p in paths:
            d = np.load(p)
            d = d[d.files[0]] if hasattr(d, "files") else d
            t = torch.from_numpy(np.asarray(d, np.float32))[None, None]
            t = F.interpolate(t, size=(H, W), mode="bilinear", align_corners=False)[0]
            out.append(t.clamp(0, self.config.max_depth) / self.config.max_depth)
        return torch.stack(out)

    def load_scene(self, idx: List[int]) -> List[Any]:
        if not self.scene_paths:
            return []
        out = []
        for i in idx:
            p = self.scene_paths[min(i, len(self.scene_paths) - 1)]
            try:
                out.append(json.loads(p.read_text()))
            except (OSError, json.JSONDecodeError):
                out.append({})
        return out


class EnfusionDataset(Dataset):
    def __init__(self, data_root: Union[str, Path, List[Union[str, Path]]],
                 config: Optional[EnfusionDatasetConfig] = None, split: str = "train",
                 session_ids: Optional[List[str]] = None, seed: int = 0):
        self.config = config or EnfusionDatasetConfig()
        self.split = split
        roots = data_root if isinstance(data_root, (list, tuple)) else [data_root]
        dirs: List[Path] = []
        for r in roots:
            r = Path(r)
            if (r / "frames").exists():
                dirs.append(r)
            else:
                dirs.extend(sorted(p for p in r.iterdir() if p.is_dir() and (p / "frames").exists()))
        if session_ids is not None:
            dirs = [d for d in dirs if d.name in set(session_ids)]
        self.sessions = [EnfusionSession(d, self.config) for d in dirs]
        self.index: List[Tuple[int, int]] = []
        c = self.config
        for si, s in enumerate(self.sessions):
            for st in s.get_valid_start_indices(c.sequence_length, c.frame_skip):
                self.index.append((si, st))
        self.rng = random.Random(seed)

    def __len__(self) -> int:
        return len(self.index)

    def __getitem__(self, i: int) -> Dict[str, Any]:
        c = self.config
        si, st = self.index[i]
        s = self.sessions[si]
        idx = [st + k * c.frame_skip for k in range(c.sequence_length)]
        frames = s.load_frames(idx)
        controls = s.controls[idx]
        out: Dict[str, Any] = {"frames": frames, "controls": controls,
                               "ego_transform": s.ego_transforms[idx],
                               "anchor_mask": s.anchor_mask(st, idx),
                               "metadata": {**s.metadata, "start": st, "session_index": si}}
        if c.load_depth:
            d = s.load_depth(idx)
            if d is not None:
                out["depth"] = d
        if c.load_scene:
            out["scene_entities"] = s.load_scene(idx)
        if c.augment and self.split == "train":
            out = self._augment(out)
        return out

    def _augment(self, sample: Dict[str, Any]) -> Dict[str, Any]:
        c = self.config
        fr = sample["frames"]
        if self.rng.random() < c.horizontal_flip_prob:
            fr = fr.flip(-1)
            sample["controls"] = sample["controls"].clone()
            sample["controls"][:, 0] = -sample["controls"][:, 0]  # mirrored steering
            if "depth" in sample:
                sample["depth"] = sample["depth"].flip(-1)
        b = self.rng.uniform(*c.brightness_range)
        k = self.rng.uniform(*c.contrast_range)
        mean = fr.mean((1, 2, 3), keepdim=True)
        sample["frames"] = ((fr * b - mean) * k + mean).clamp_(0, 1)
        return sample


class EnfusionCollator:
    """Stacks tensors, keeps lists (scene entities) and metadata as lists; scene entities
    are dropped unless ``include_scene_entities`` (the reference's collator options,
    data/enfusion_loader.py:616-663; ``pad_to_max`` / ``max_sequence_length`` are
    accepted for its call sites: samples of one dataset already share their length)."""

    def __init__(self, pad_to_max: bool = True, max_sequence_length: Optional[int] = None,
                 include_scene_entities: bool = True):
        self.pad_to_max, self.max_sequence_length = pad_to_max, max_sequence_length
        self.include_scene_entities = include_scene_entities

    def __call__(self, batch: List[Dict[str, Any]]) -> Dict[str, Any]:
        out: Dict[str, Any] = {}
        if not batch:
            return out
        for k in batch[0]:
            if k == "scene_entities" and not self.include_scene_entities:
                continue
            vals = [b[k] for b in batch if k in b]
            if torch.is_tensor(vals[0]) and len(vals) == len(batch):
                out[k] = torch.stack(vals)
            else:
                out[k] = vals
        return out


class EnfusionDataLoader:
    """Batches of an :class:`EnfusionDataset` delivered on ``device`` (CUDA when
    available): worker processes decode, the collator stacks into pinned memory, and
    every tensor moves with a non-blocking copy (data/enfusion_loader.py:666-722)."""

    def __init__(self, dataset: "EnfusionDataset", batch_size: int = 8, shuffle: bool = True,
                 num_workers: int = 4, pin_memory: bool = True, drop_last: bool = True,
                 prefetch_factor: int = 2, include_scene_entities: bool = False,
                 device: Optional[Union[str, torch.device]] = None):
        self.dataset = dataset
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda") if torch.cuda.is_available() else None)
        kw = dict(prefetch_factor=prefetch_factor, persistent_workers=True) if num_workers > 0 else {}
        pin = pin_memory and self.device is not None and self.device.type == "cuda"
        self.dataloader = DataLoader(dataset, batch_size=batch_size, shuffle=shuffle,
                                     num_workers=num_workers, pin_memory=pin, drop_last=drop_last,
                                     collate_fn=EnfusionCollator(include_scene_entities=include_scene_entities),
                                     **kw)

    def __iter__(self):
        for batch in self.dataloader:
            if self.device is None:
                yield batch
                continue
            yield {k: v.to(self.device, non_blocking=True) if torch.is_tensor(v) else v
                   for k, v in batch.items()}

    def __len__(self) -> int:
        return len(self.dataloader)


def create_enfusion_dataloaders(data_root, config: Optional[EnfusionDatasetConfig] = None,
                                batch_size: int = 8, num_workers: int = 4, train_ratio: float = 0.8,
                                val_ratio: float = 0.1, seed: Optional[int] = None, pin_memory: bool = True,
                                device=None):
    """(train, val, test) :class:`EnfusionDataLoader` (data/enfusion_loader.py:725-819):
    ``train/`` and ``val/`` (and ``test/``, else ``val/`` again) folders when the root has
    them, otherwise a session-level split of ``session_*`` by ``train_ratio`` /
    ``val_ratio``. Training batches are shuffled (last partial batch dropped) and
    augmented when the config asks; validation and test are not augmented."""
    from dataclasses import replace

    root = Path(data_root)
    config = config or EnfusionDatasetConfig()
    evalc = replace(config, augment=False)
    if (root / "train").is_dir() and (root / "val").is_dir():
        tr = EnfusionDataset(root / "train", config, "train")
        va = EnfusionDataset(root / "val", evalc, "val")
        te = EnfusionDataset(root / "test" if (root / "test").is_dir() else root / "val", evalc, "test")
    else:
        names = sorted(p.name for p in root.glob("session_*") if p.is_dir())
        random.Random(seed).shuffle(names)
        n_tr, n_va = int(len(names) * train_ratio), int(len(names) * val_ratio)
        tr = EnfusionDataset(root, config, "train", names[:n_tr])
        va = EnfusionDataset(root, evalc, "val", names[n_tr:n_tr + n_va])
        te = EnfusionDataset(root, evalc, "test", names[n_tr + n_va:])
    mk = lambda ds, train: EnfusionDataLoader(ds, batch_size, shuffle=train and len(ds) > 0,
                                              num_workers=num_workers, pin_memory=pin_memory,
                                              drop_last=train, device=device)
    return mk(tr, True), mk(va, False), mk(te, False)


class EnfusionToDriveDiTAdapter:
    """Loader batch -> training inputs (data/enfusion_loader.py:822-890): ``frames`` as
    they are, ``controls`` zero-padded or cut to ``target_control_dim`` channels, depth,
    ego transforms (when included and present) and anchor masks."""

    def __init__(self, target_control_dim: int = 6, include_depth: bool = True,
                 include_ego_transform: bool = True):
        self.target_control_dim = target_control_dim
        self.include_depth, self.include_ego_transform = include_depth, include_ego_transform

    def __call__(self, batch: Dict[str, Any]) -> Dict[str, torch.Tensor]:
        c = batch["controls"]
        d = self.target_control_dim
        c = F.pad(c, (0, d - c.shape[-1])) if c.shape[-1] < d else c[..., :d]
        out = {"frames": batch["frames"], "controls": c}
        if self.include_depth and batch.get("depth") is not None:
            out["depth"] = batch["depth"]
        if self.include_ego_transform and batch.get("ego_transform") is not None:
            out["ego_transform"] = batch["ego_transform"]
        if batch.get("anchor_mask") is not None:
            out["anchor_mask"] = batch["anchor_mask"]
        return out
