"""The reference's top-level system sketch (``core/base.py``: ``DriveDiTConfig``,
``TensorCache``, encoder bases, ``DriveDiTSystem`` whose forward methods are ``pass``)
made to work from this framework's parts: the causal VAE3D turns RGB frames into latents,
the latent world model predicts the next frames by flow matching under the controls, and
the VAE decodes them.

``DriveDiTSystem.forward(frames, controls, mode="train")`` returns the flow-matching loss
on the clip's latents (context frames clean, the rest noised per frame);
``mode="inference"`` rolls out ``horizon`` frames after the given ones and decodes them.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from typing import Dict, Optional

import torch
import torch.nn as nn

from ..models.world_model import ControlEncoder, DepthEncoder  # noqa: F401  (reference names)


@dataclass
class DriveDiTConfig:
    latent_channels: int = 4
    latent_spatial_size: int = 32
    model_dim: int = 1024
    n_heads: int = 16
    n_layers: int = 24
    context_length: int = 8
    max_memory_objects: int = 32
    max_memory_frames: int = 5
    flow_matching_steps: int = 4
    self_forcing_horizon: int = 16
    mixed_precision: bool = True
    device: str = "cuda"
    dtype: torch.dtype = torch.bfloat16
    control_dim: int = 6
    image_size: int = 256


class TensorCache:
    """Bounded FIFO of detached tensors; ``get_recent(n)`` stacks the newest ``n`` on dim 1."""

    def __init__(self, max_size: int = 256, device: str = "cpu"):
        self.cache: deque = deque(maxlen=max_size)
        self.device = device

    def append(self, tensor: torch.Tensor) -> None:
        self.cache.append(tensor.detach().to(self.device, non_blocking=True))

    def get_recent(self, n: int) -> Optional[torch.Tensor]:
        if len(self.cache) < n:
            return None
        return torch.stack(list(self.cache)[-n:], 1)

    def clear(self) -> None:
        self.cache.clear()


class DriveDiTSystem(nn.Module):
    def __init__(self, config: DriveDiTConfig):
        super().__init__()
        from ..config.presets import ModelConfig
        from ..inference.rollout import MemoryBank
        from ..models.vae3d import VAE3DConfig, VAE3Dv2
        from ..models.world_dit import WorldDiT

        self.config = c = config
        self.vae = VAE3Dv2(VAE3DConfig(in_channels=3, latent_dim=c.latent_channels,
                                       hidden_dims=[32, 64, 64, 64], num_res_blocks=1,
                                       use_attention=False, temporal_compression=1, spatial_compression=8,
                                       use_perceptual_loss=False))
        lat = max(2, c.image_size // 8)
        self.world_model = WorldDiT(ModelConfig(name="system", n_layers=c.n_layers, d_model=c.model_dim,
                                                n_heads=c.n_heads, mlp_hidden=4 * c.model_dim,
                                                latent_channels=c.latent_channels, latent_h=lat, latent_w=lat,
                                                action_dim=c.control_dim))
        self.memory_bank = MemoryBank(c.model_dim, max_spatial_memory=c.max_memory_frames)
        self.tensor_cache = TensorCache(c.max_memory_frames)

    @torch.no_grad()
    def encode(self, frames: torch.Tensor) -> torch.Tensor:
        """``[B, T, 3, H, W]`` in [0, 1] -> latents ``[B, T', C, h, w]`` (posterior mean)."""
        mean, _ = self.vae.encode(frames.permute(0, 2, 1, 3, 4) * 2 - 1)
        z = mean.permute(0, 2, 1, 3, 4)
        h, w = self.world_model.cfg.latent_h, self.world_model.cfg.latent_w
        z = z[..., :h, :w]                      # the encoder's grid can exceed H/8 by one
        return torch.nn.functional.pad(z, (0, w - z.shape[-1], 0, h - z.shape[-2]))

    @torch.no_grad()
    def decode(self, latents: torch.Tensor, hw) -> torch.Tensor:
        x = self.vae.decode(latents.permute(0, 2, 1, 3, 4),
                            output_shape=(latents.shape[1],) + tuple(hw))
        return ((x.permute(0, 2, 1, 3, 4) + 1) / 2).clamp(0, 1)

    def forward(self, frames: torch.Tensor, controls: torch.Tensor, depth_maps: Optional[torch.Tensor] = None,
                mode: str = "train", horizon: int = 4) -> Dict[str, torch.Tensor]:
        if mode == "train":
            return self._train_forward(frames, controls)
        return self._inference_forward(frames, controls, horizon)

    def _train_forward(self, frames, controls):
        from ..training.flow_matching import flow_matching_loss, interpolate, sample_t

        z1 = self.encode(frames)
        B, T = z1.shape[:2]
        ctx = min(self.config.context_length, T - 1)
        t = sample_t(B, "logit_normal", z1.device).view(B, 1).expand(B, T).clone()
        t[:, :ctx] = 1.0                                            # context frames stay clean
        z0 = torch.randn_like(z1)
        zt = interpolate(z0, z1, t)
        v = self.world_model(zt, t, controls[:, :T])
        loss = flow_matching_loss(v[:, ctx:], z0[:, ctx:], z1[:, ctx:])
        return {"loss": loss, "latents": z1, "velocity": v}

    @torch.no_grad()
    def _inference_forward(self, frames, controls, horizon):
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        z = self.encode(frames)
        B, Fc = z.shape[:2]
        total = Fc + horizon
        acts = controls if controls.shape[1] >= total else torch.cat(
            [controls, controls[:, -1:].expand(-1, total - controls.shape[1], -1)], 1)
        ro = StreamingRollout(self.world_model, RolloutConfig(total_frames=total, chunk_frames=1,
                                                              flow_steps=self.config.flow_matching_steps,
                                                              window_frames=max(Fc, 2)),
                              dtype=z.dtype)
        res = ro.run(z, acts[:, :total], total)
        gen = res.frames[:, Fc:]
        for f in range(gen.shape[1]):
            self.tensor_cache.append(gen[:, f])
        return {"latents": gen, "frames": self.decode(gen.float(), frames.shape[-2:]),
                "chunk_ms": torch.tensor(res.chunk_ms)}
