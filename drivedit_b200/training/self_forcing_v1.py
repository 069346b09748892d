"""Self-forcing trainer, first generation (the reference's ``training/self_forcing.py:32-493``
API: ``SelfForcingTrainer(model, optimizer, scheduler, checkpoint_dir, max_memory_gb,
mixed_precision, distributed)`` with ``train_epoch / validate / load_checkpoint /
get_training_stats / print_training_summary / log_metrics / cleanup``, plus
``create_simple_model``, ``create_dummy_dataloader`` and ``main``).

``model`` maps a frame ``[B, C, H, W]`` to the next frame. A step rolls the model out on its
own predictions from the last context frame over the prediction horizon (exposure to its own
errors is the point of self-forcing) and scores the rollout against the ground truth:
reconstruction MSE, temporal-difference consistency and a luminance L1 term.

Differences from the reference: the epoch loop reads ``checkpoint_every`` that the reference
never defines (``:175``, a crash at the first step) from the constructor here; mixed
precision is bf16 autocast (no loss scaler needed); checkpoints go through the atomic,
checksummed :class:`~drivedit_b200.training.distributed.CheckpointManager`.
"""
from __future__ import annotations

import os
import time
from collections import defaultdict
from pathlib import Path
from typing import Any, Dict, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.data import DataLoader, Dataset

from .distributed import CheckpointManager, DistributedManager, MemoryMonitor, setup_distributed_model


class SelfForcingTrainer:
    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer,
                 scheduler: Optional[Any] = None, checkpoint_dir: str = "./checkpoints",
                 max_memory_gb: float = 12.0, mixed_precision: bool = True, distributed: bool = False,
                 checkpoint_every: int = 1000, context_length: int = 8, prediction_horizon: int = 16,
                 grad_clip: float = 1.0):
        self.model, self.optimizer, self.scheduler = model, optimizer, scheduler
        self.checkpoint_dir = Path(checkpoint_dir)
        self.max_memory_gb, self.mixed_precision, self.distributed = max_memory_gb, mixed_precision, distributed
        self.checkpoint_every, self.grad_clip = checkpoint_every, grad_clip
        self.context_length, self.prediction_horizon = context_length, prediction_horizon
        self.memory_monitor = MemoryMonitor(max_memory_gb)
        self.dist_manager = DistributedManager()
        if distributed:
            self.model = setup_distributed_model(model, self.dist_manager.local_rank, find_unused_parameters=True)
        self.checkpoint_manager = CheckpointManager(str(self.checkpoint_dir), keep_checkpoints=5,
                                                    rank=self.dist_manager.rank,
                                                    world_size=self.dist_manager.world_size)
        self.loss_weights = {"reconstruction": 1.0, "temporal_consistency": 0.3, "perceptual": 0.1}
        self.global_step = 0
        self.epoch = 0
        self.best_loss = float("inf")
        self.step_times = []
        self.throughput_tracker = defaultdict(list)

    @property
    def device(self) -> torch.device:
        return next(self.model.parameters()).device

    def _autocast(self):
        on = self.mixed_precision and self.device.type == "cuda"
        return torch.autocast("cuda", dtype=torch.bfloat16, enabled=on)

    # ------------------------------------------------------------------ steps
    def _self_forcing_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        frames = batch["frames"].to(self.device)
        B, T = frames.shape[:2]
        L = min(self.context_length, T // 2)
        Hz = min(self.prediction_horizon, T - L)
        target = frames[:, L:L + Hz]
        cur = frames[:, L - 1]
        preds = []
        for _ in range(Hz):
            cur = self._predict_next_frame(cur)
            preds.append(cur)
        losses: Dict[str, torch.Tensor] = {}
        if preds:
            p = torch.stack(preds, 1).float()
            t = target.float()
            losses["reconstruction"] = F.mse_loss(p, t)
            if Hz > 1:
                losses["temporal_consistency"] = F.mse_loss(p[:, 1:] - p[:, :-1], t[:, 1:] - t[:, :-1])
            losses["perceptual"] = self._compute_perceptual_loss(p, t)
        return losses

    def _encode_frames(self, frames: torch.Tensor) -> torch.Tensor:
        return F.avg_pool2d(frames.flatten(0, 1), 8).view(frames.shape[0], frames.shape[1], -1)

    def _predict_next_frame(self, current_frame: torch.Tensor) -> torch.Tensor:
        return self.model(current_frame)

    @staticmethod
    def _compute_perceptual_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        return F.l1_loss(pred.mean(2, keepdim=True), target.mean(2, keepdim=True))

    def _compute_total_loss(self, losses: Dict[str, torch.Tensor]) -> torch.Tensor:
        total = sum(self.loss_weights.get(k, 1.0) * v for k, v in losses.items())
        return total if torch.is_tensor(total) else torch.zeros((), device=self.device)

    def train_epoch(self, dataloader) -> Dict[str, float]:
        self.model.train()
        acc = defaultdict(list)
        for batch in dataloader:
            t0 = time.perf_counter()
            with self._autocast():
                losses = self._self_forcing_step(batch)
            total = self._compute_total_loss(losses)
            self.optimizer.zero_grad(set_to_none=True)
            total.backward()
            if self.grad_clip > 0:
                torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.grad_clip)
            self.optimizer.step()
            if self.scheduler is not None:
                self.scheduler.step()
            self.global_step += 1
            for k, v in losses.items():
                acc[k].append(float(v.detach()))
            acc["total"].append(float(total.detach()))
            dt = time.perf_counter() - t0
            self.step_times.append(dt)
            self.throughput_tracker["samples_per_sec"].append(batch["frames"].shape[0] / max(dt, 1e-9))
            if self.memory_monitor.should_cleanup():
                self.memory_monitor.cleanup()
            if self.checkpoint_every and self.global_step % self.checkpoint_every == 0:
                self._save_checkpoint(float(total))
        self.epoch += 1
        return {k: float(np.mean(v)) for k, v in acc.items()}

    @torch.no_grad()
    def validate(self, val_dataloader) -> Dict[str, float]:
        self.model.eval()
        acc = defaultdict(list)
        for batch in val_dataloader:
            with self._autocast():
                losses = self._self_forcing_step(batch)
            for k, v in losses.items():
                acc[k].append(float(v))
            acc["total"].append(float(self._compute_total_loss(losses)))
        self.model.train()
        return {k: float(np.mean(v)) for k, v in acc.items()}

    # ------------------------------------------------------------------ state
    def _save_checkpoint(self, loss: float) -> None:
        best = loss < self.best_loss
        self.best_loss = min(self.best_loss, loss)
        m = self.model.module if hasattr(self.model, "module") else self.model
        self.checkpoint_manager.save_checkpoint(m, self.optimizer, self.scheduler, self.epoch,
                                                self.global_step, loss, is_best=best)

    def load_checkpoint(self, checkpoint_path: Optional[str] = None) -> Dict[str, Any]:
        m = self.model.module if hasattr(self.model, "module") else self.model
        info = self.checkpoint_manager.load_checkpoint(m, self.optimizer, self.scheduler, checkpoint_path)
        if info:
            self.epoch, self.global_step = info["epoch"], info["step"]
            self.best_loss = min(self.best_loss, info["loss"])
        return info

    def get_training_stats(self) -> Dict[str, float]:
        st = np.asarray(self.step_times[-100:] or [0.0])
        thr = self.throughput_tracker["samples_per_sec"][-100:] or [0.0]
        return {"global_step": self.global_step, "epoch": self.epoch, "best_loss": self.best_loss,
                "avg_step_time": float(st.mean()), "samples_per_sec": float(np.mean(thr)),
                **{f"memory_{k}": v for k, v in self.memory_monitor.update().items()}}

    def print_training_summary(self) -> None:
        for k, v in self.get_training_stats().items():
            print(f"  {k}: {v}")

    def log_metrics(self, metrics: Dict[str, float]) -> None:
        if self.dist_manager.is_master:
            print(f"step {self.global_step}: " + ", ".join(f"{k}={v:.4f}" for k, v in metrics.items()))

    def cleanup(self) -> None:
        self.memory_monitor.cleanup()
        self.dist_manager.cleanup()


def create_simple_model(input_channels: int = 3, hidden_dim: int = 256) -> nn.Module:
    """Three 3x3 convolutions frame -> frame with a sigmoid output."""
    return nn.Sequential(nn.Conv2d(input_channels, hidden_dim // 4, 3, padding=1), nn.ReLU(),
                         nn.Conv2d(hidden_dim // 4, hidden_dim // 2, 3, padding=1), nn.ReLU(),
                         nn.Conv2d(hidden_dim // 2, input_channels, 3, padding=1), nn.Sigmoid())


class _DummyClips(Dataset):
    def __init__(self, n: int, frames: int = 16, size: int = 64):
        self.n, self.frames, self.size = n, frames, size

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        g = torch.Generator().manual_seed(i)
        return {"frames": torch.rand(self.frames, 3, self.size, self.size, generator=g),
                "controls": torch.rand(self.frames, 6, generator=g) * 2 - 1}


def create_dummy_dataloader(batch_size: int = 4, num_batches: int = 100, frames: int = 16, size: int = 64):
    return DataLoader(_DummyClips(batch_size * num_batches, frames, size), batch_size=batch_size)


def main(rank: int = 0, world_size: int = 1, epochs: int = 1, num_batches: int = 10):
    """Trains the simple model on random clips (one process per GPU when ``world_size > 1``)."""
    if world_size > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "12355")
        DistributedManager().setup(rank, world_size, "nccl" if torch.cuda.is_available() else "gloo")
    dev = torch.device("cuda", rank) if torch.cuda.is_available() else torch.device("cpu")
    model = create_simple_model().to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.01)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(opt, T_max=1000)
    tr = SelfForcingTrainer(model, opt, sched, distributed=world_size > 1)
    try:
        for _ in range(epochs):
            tr.log_metrics(tr.train_epoch(create_dummy_dataloader(4, num_batches)))
    finally:
        tr.cleanup()
    return tr
