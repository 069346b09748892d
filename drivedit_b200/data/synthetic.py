"""Synthetic workloads of the preset shapes (random latents, actions, flow times).

The benchmarks and tests run on synthetic data: latent video ``~N(0,1)``, per-frame
actions ``~U[-1,1]``, and (for REPA) RGB frames ``~U[0,1]``. ``host_batch`` builds the
batch in pinned host memory so end-to-end timings include the host->device copy.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

from ..config import Config


@dataclass
class LatentBatch:
    latents: torch.Tensor      # [B, F, C, H, W]
    actions: torch.Tensor      # [B, F, A]
    rgb: Optional[torch.Tensor] = None  # [B, F', 3, Hi, Wi] (REPA teacher input)

    def to(self, device, non_blocking: bool = True) -> "LatentBatch":
        return LatentBatch(self.latents.to(device, non_blocking=non_blocking),
                           self.actions.to(device, non_blocking=non_blocking),
                           None if self.rgb is None else self.rgb.to(device, non_blocking=non_blocking))

    def nbytes(self) -> int:
        n = self.latents.numel() * self.latents.element_size()
        n += self.actions.numel() * self.actions.element_size()
        if self.rgb is not None:
            n += self.rgb.numel() * self.rgb.element_size()
        return n


def make_batch(cfg: Config, batch: Optional[int] = None, frames: Optional[int] = None,
               device="cpu", dtype=torch.float32, generator=None, pin: bool = False,
               rgb_frames: int = 0) -> LatentBatch:
    m, t = cfg.model, cfg.train
    B = batch or t.batch_per_gpu
    Fr = frames or t.frames
    lat = torch.randn(B, Fr, m.latent_channels, m.latent_h, m.latent_w, generator=generator,
                      dtype=torch.float32).to(dtype)
    act = torch.rand(B, Fr, m.action_dim, generator=generator) * 2 - 1
    rgb = None
    if rgb_frames and m.repa is not None:
        rgb = torch.rand(B, rgb_frames, 3, m.repa.image_h, m.repa.image_w, generator=generator).to(dtype)
    if pin:
        lat, act = lat.pin_memory(), act.pin_memory()
        rgb = rgb.pin_memory() if rgb is not None else None
    b = LatentBatch(lat, act, rgb)
    return b if str(device) == "cpu" else b.to(device)
