"""The reference's top-level system sketch (``core/base.py``: ``DriveDiTConfig``,
``TensorCache``, the encoders, ``MemoryBank``, ``CausalDiT`` and ``DriveDiTSystem``, whose
attention classes and forward methods are ``pass``) made to work from this framework's
parts. The encoders, memory bank and causal DiT are working modules with the reference's
constructors (a ``DriveDiTConfig``). ``DriveDiTSystem`` is built from the causal VAE3D turns RGB frames into latents,
the latent world model predicts the next frames by flow matching under the controls, and
the VAE decodes them.

``DriveDiTSystem.forward(frames, controls, mode="train")`` returns the flow-matching loss
on the clip's latents (context frames clean, the rest noised per frame);
``mode="inference"`` rolls out ``horizon`` frames after the given ones and decodes them.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from collections import deque
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn


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


class BaseEncoder(nn.Module, ABC):
    """An encoder into the model's token space (core/base.py:63-74)."""

    @abstractmethod
    def encode(self, x: torch.Tensor) -> torch.Tensor:
        ...

    @abstractmethod
    def get_token_dim(self) -> int:
        ...


class VAEEncoder(BaseEncoder):
    """Frames ``[B, T, 3, H, W]`` (in [0, 1]) -> latent tokens ``[B, T, h * w, model_dim]``
    and back. The reference (core/base.py:76-139) downloads a pretrained WAN-VAE; here the
    image VAE is this framework's causal VAE run frame by frame (no temporal compression,
    16x spatial), random-initialised unless weights are loaded into ``self.vae``. Latents
    are scaled by ``scaling_factor`` before the token projection, and :meth:`decode`
    inverts the projection with ``latent_unproj`` and decodes (the reference leaves its
    decode unwritten)."""

    downscale_factor = 16
    scaling_factor = 0.18215

    def __init__(self, config: DriveDiTConfig, vae: Optional[nn.Module] = None):
        super().__init__()
        from ..models.vae3d import VAE3DConfig, VAE3Dv2

        self.config = config
        self.vae = vae if vae is not None else VAE3Dv2(VAE3DConfig(
            in_channels=3, latent_dim=config.latent_channels, hidden_dims=[32, 64, 64, 64, 64],
            num_res_blocks=1, use_attention=False, temporal_compression=1,
            spatial_compression=self.downscale_factor, use_perceptual_loss=False))
        self.latent_proj = nn.Linear(config.latent_channels, config.model_dim)
        self.latent_unproj = nn.Linear(config.model_dim, config.latent_channels)

    def latents(self, frames: torch.Tensor) -> torch.Tensor:
        """``[B, T, 3, H, W]`` -> scaled posterior means ``[B, T, C, H/16, W/16]``."""
        B, T = frames.shape[:2]
        x = frames.reshape(B * T, 1, *frames.shape[2:]).transpose(1, 2) * 2 - 1  # [BT, 3, 1, H, W]
        mean, _ = self.vae.encode(x)
        h, w = frames.shape[-2] // self.downscale_factor, frames.shape[-1] // self.downscale_factor
        z = mean[:, :, 0, :h, :w]
        return (z * self.scaling_factor).reshape(B, T, *z.shape[1:])

    def encode(self, frames: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            z = self.latents(frames)
        return self.latent_proj(z.flatten(3).transpose(2, 3))  # [B, T, h*w, model_dim]

    def decode(self, tokens: torch.Tensor, hw: Tuple[int, int]) -> torch.Tensor:
        """Tokens ``[B, T, h * w, model_dim]`` -> frames ``[B, T, 3, H, W]`` in [0, 1]."""
        B, T, N, _ = tokens.shape
        h, w = hw[0] // self.downscale_factor, hw[1] // self.downscale_factor
        z = self.latent_unproj(tokens).transpose(2, 3).reshape(B * T, -1, 1, h, w) / self.scaling_factor
        x = self.vae.decode(z, output_shape=(1,) + tuple(hw))
        return ((x[:, :, 0] + 1) / 2).clamp(0, 1).reshape(B, T, *x.shape[1:2], *x.shape[-2:])

    def get_token_dim(self) -> int:
        return self.config.model_dim


class DepthEncoder(BaseEncoder):
    """Depth maps ``[B, T, 1, H, W]`` -> tokens ``[B, T, s * s, model_dim]`` (s =
    ``latent_spatial_size``): a three-convolution head (two stride-2) and adaptive
    pooling to the latent grid (core/base.py:141-180; same layer stack, so its weights
    load)."""

    def __init__(self, config: DriveDiTConfig):
        super().__init__()
        self.config = config
        s = config.latent_spatial_size
        self.depth_encoder = nn.Sequential(
            nn.Conv2d(1, 64, 3, padding=1), nn.ReLU(),
            nn.Conv2d(64, 128, 3, stride=2, padding=1), nn.ReLU(),
            nn.Conv2d(128, config.model_dim, 3, stride=2, padding=1),
            nn.AdaptiveAvgPool2d((s, s)))

    def encode(self, depth_maps: torch.Tensor) -> torch.Tensor:
        B, T = depth_maps.shape[:2]
        f = self.depth_encoder(depth_maps.flatten(0, 1))           # [BT, D, s, s]
        return f.flatten(2).transpose(1, 2).reshape(B, T, -1, f.shape[1])

    def get_token_dim(self) -> int:
        return self.config.model_dim


class ControlEncoder(BaseEncoder):
    """Controls ``[B, 6]`` (steer, accel, brake, goal x, goal y, speed) -> one token
    ``[B, 1, model_dim]`` by a two-layer SiLU MLP (core/base.py:248-272)."""

    def __init__(self, config: DriveDiTConfig):
        super().__init__()
        self.config = config
        d = config.model_dim
        self.control_mlp = nn.Sequential(nn.Linear(6, 2 * d), nn.SiLU(), nn.Linear(2 * d, d))

    def encode(self, controls: torch.Tensor) -> torch.Tensor:
        return self.control_mlp(controls)[:, None]

    def get_token_dim(self) -> int:
        return self.config.model_dim


class MemoryBank:
    """Spatial and object memory for the causal DiT's cross-attention (core/base.py:
    182-246): each frame passes a small convolutional feature extractor (``sam_encoder``,
    the stand-in the reference also uses for SAM2) into a FIFO of the last
    ``max_memory_frames`` frames; object tokens come from :meth:`add_objects` (the
    reference leaves object tracking unwritten). Until a FIFO holds its full count the
    matching tokens are one zero token."""

    def __init__(self, config: DriveDiTConfig):
        self.config = config
        self.spatial_memory = TensorCache(config.max_memory_frames, config.device)
        self.object_memory = TensorCache(config.max_memory_objects, config.device)
        self.sam_encoder = nn.Sequential(
            nn.Conv2d(3, 64, 3, padding=1), nn.ReLU(), nn.AdaptiveAvgPool2d((8, 8)), nn.Flatten(),
            nn.Linear(64 * 64, config.model_dim)).to(config.device)

    def update(self, frame: torch.Tensor, frame_idx: int = 0) -> None:
        """``frame [B, 3, H, W]``: its feature vector joins the spatial memory."""
        with torch.no_grad():
            self.spatial_memory.append(self.sam_encoder(frame.to(self.config.device)))

    def add_objects(self, object_tokens: torch.Tensor) -> None:
        """``[B, model_dim]`` tokens of tracked objects (one per call)."""
        self.object_memory.append(object_tokens)

    def _tokens(self, cache: TensorCache, n: int) -> torch.Tensor:
        t = cache.get_recent(n)
        if t is None:
            return torch.zeros(1, 1, self.config.model_dim, device=self.config.device,
                               dtype=self.config.dtype)
        return t

    def get_memory_tokens(self) -> Tuple[torch.Tensor, torch.Tensor]:
        return (self._tokens(self.spatial_memory, self.config.max_memory_frames),
                self._tokens(self.object_memory, self.config.max_memory_objects))

    def clear(self) -> None:
        self.spatial_memory.clear()
        self.object_memory.clear()


class CausalTransformerLayer(nn.Module):
    """Pre-LayerNorm layer: causal self-attention (with a key/value cache for
    generation), cross-attention to the memory tokens when there are any, SiLU FFN
    (core/base.py:346-400; same sub-module names)."""

    def __init__(self, config: DriveDiTConfig):
        super().__init__()
        from ..layers.attention import CrossAttention, MultiHeadAttention

        d, h = config.model_dim, config.n_heads
        self.config = config
        self.self_attn = MultiHeadAttention(d, h, causal=True)
        self.self_attn_norm = nn.LayerNorm(d)
        self.cross_attn = CrossAttention(d, h)
        self.cross_attn_norm = nn.LayerNorm(d)
        self.ffn = nn.Sequential(nn.Linear(d, 4 * d), nn.SiLU(), nn.Linear(4 * d, d))
        self.ffn_norm = nn.LayerNorm(d)

    def forward(self, x: torch.Tensor, memory_tokens: Tuple[torch.Tensor, torch.Tensor],
                past_kv: Optional[Dict[str, torch.Tensor]] = None,
                use_cache: bool = False) -> Tuple[torch.Tensor, Optional[Dict[str, torch.Tensor]]]:
        cache_in = (past_kv if past_kv is not None else {}) if use_cache else past_kv
        a, cache = self.self_attn(self.self_attn_norm(x), cache_in)
        x = x + a
        spatial, objects = memory_tokens
        if spatial.numel() > 0:
            mem = torch.cat([spatial, objects], 1).to(x.dtype)
            if mem.shape[0] != x.shape[0]:
                mem = mem.expand(x.shape[0], -1, -1)
            x = x + self.cross_attn(self.cross_attn_norm(x), mem)
        x = x + self.ffn(self.ffn_norm(x))
        return x, (cache if use_cache else None)


class CausalDiT(nn.Module):
    """Autoregressive causal transformer over combined tokens ``[B, L, model_dim]``; the
    last token's output is projected to the next frame's latent ``[B, C, s, s]``
    (core/base.py:274-343). With ``use_cache`` every layer keeps its keys and values
    (``self.kv_cache``) and later calls pass only the new tokens; :meth:`reset_cache`
    starts a new sequence."""

    def __init__(self, config: DriveDiTConfig):
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([CausalTransformerLayer(config) for _ in range(config.n_layers)])
        self.output_proj = nn.Linear(config.model_dim,
                                     config.latent_channels * config.latent_spatial_size ** 2)
        self.kv_cache: Optional[Dict[str, Dict[str, torch.Tensor]]] = None

    def forward(self, tokens: torch.Tensor, memory_tokens: Tuple[torch.Tensor, torch.Tensor],
                use_cache: bool = False):
        x = tokens
        new_cache = {} if use_cache else None
        for i, layer in enumerate(self.layers):
            past = self.kv_cache.get(f"layer_{i}") if (use_cache and self.kv_cache) else None
            x, c = layer(x, memory_tokens, past_kv=past, use_cache=use_cache)
            if use_cache:
                new_cache[f"layer_{i}"] = c
        s = self.config.latent_spatial_size
        nxt = self.output_proj(x[:, -1]).reshape(x.shape[0], self.config.latent_channels, s, s)
        if use_cache:
            self.kv_cache = new_cache
        return nxt, new_cache

    def reset_cache(self) -> None:
        self.kv_cache = None


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
