"""VAE / DiT / model sub-configs and the small / medium / large presets (the reference's
``config/model_config.py:12-246`` interface; same field names and defaults so saved JSON
configs load unchanged).

:meth:`ModelConfig.to_world_config` maps a student config onto this framework's
world-model :class:`~drivedit_b200.config.presets.Config`.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

from .base import BaseConfig


@dataclass
class VAEConfig(BaseConfig):
    in_channels: int = 3
    latent_dim: int = 8
    hidden_dims: Optional[List[int]] = None
    num_res_blocks: int = 2
    use_attention: bool = True
    beta: float = 1.0
    mixed_precision: bool = True
    gradient_checkpointing: bool = False

    def __post_init__(self):
        if self.hidden_dims is None:
            self.hidden_dims = [128, 256, 512, 512]
        super().__post_init__()

    def validate(self):
        if self.in_channels <= 0 or self.latent_dim <= 0:
            raise ValueError("in_channels and latent_dim must be positive")
        if self.num_res_blocks < 0:
            raise ValueError("num_res_blocks must be non-negative")
        if not 0.0 <= self.beta <= 10.0:
            raise ValueError("beta should be in [0, 10]")
        if not self.hidden_dims:
            raise ValueError("hidden_dims cannot be empty")


@dataclass
class DiTConfig(BaseConfig):
    latent_dim: int = 8
    d_model: int = 1024
    n_layers: int = 24
    n_heads: int = 16
    d_ff: Optional[int] = None
    mlp_type: str = "swiglu"
    use_rope: bool = True
    use_flash_attention: bool = False
    causal: bool = True
    max_seq_len: int = 2048
    context_length: int = 8
    use_memory: bool = True
    memory_size: int = 1024
    cond_dim: Optional[int] = None
    time_embed_dim: int = 256
    dropout: float = 0.0
    bias: bool = False
    mixed_precision: bool = True
    gradient_checkpointing: bool = False
    num_diffusion_steps: int = 1000

    def __post_init__(self):
        if self.d_ff is None:
            if self.mlp_type in ("swiglu", "geglu"):
                self.d_ff = (int(8 * self.d_model / 3) + 7) // 8 * 8
            else:
                self.d_ff = 4 * self.d_model
        super().__post_init__()

    def validate(self):
        if self.d_model <= 0 or self.n_layers <= 0 or self.n_heads <= 0 or self.latent_dim <= 0:
            raise ValueError("dimensions must be positive")
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        if self.max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if not 0.0 <= self.dropout <= 1.0:
            raise ValueError("dropout must be in [0, 1]")
        if self.mlp_type not in ("standard", "swiglu", "geglu"):
            raise ValueError(f"Invalid mlp_type: {self.mlp_type}")


@dataclass
class ModelConfig(BaseConfig):
    vae: Optional[VAEConfig] = None
    student: Optional[DiTConfig] = None
    teacher: Optional[DiTConfig] = None
    device: str = "cuda"
    seed: int = 42
    image_size: Tuple[int, int] = (512, 512)
    sequence_length: int = 32
    control_dim: int = 4
    flow_steps: int = 4
    sigma_min: float = 0.002
    sigma_max: float = 80.0

    def __post_init__(self):
        if self.vae is None:
            self.vae = VAEConfig()
        if self.student is None:
            self.student = DiTConfig(causal=True)
        if self.teacher is None:
            self.teacher = DiTConfig(causal=False)
        self.student.latent_dim = self.vae.latent_dim
        self.teacher.latent_dim = self.vae.latent_dim
        super().__post_init__()

    def validate(self):
        if self.image_size[0] <= 0 or self.image_size[1] <= 0:
            raise ValueError("Invalid image_size")
        if self.sequence_length <= 0 or self.flow_steps <= 0 or self.control_dim < 0:
            raise ValueError("sequence_length / flow_steps must be positive")
        if not 0 < self.sigma_min < self.sigma_max:
            raise ValueError("Invalid sigma values")
        self.vae.validate()
        self.student.validate()
        self.teacher.validate()

    def to_world_config(self, attention: str = "dense"):
        """The student as this framework's latent world model (VAE 8x spatial, patch 2)."""
        from .presets import Config, ModelConfig as WorldModelConfig, TrainConfig

        s = self.student
        h, w = self.image_size
        m = WorldModelConfig(name="student", n_layers=s.n_layers, d_model=s.d_model,
                             n_heads=s.n_heads, mlp_hidden=s.d_ff, latent_channels=self.vae.latent_dim,
                             latent_h=max(2, h // 8), latent_w=max(2, w // 8),
                             action_dim=self.control_dim, attention=attention,
                             causal="frame" if s.causal else "none")
        return Config(model=m, train=TrainConfig(frames=self.sequence_length, seed=self.seed))


def _preset(latent, hidden, res, d, layers, heads, seq, img, seq_len, ckpt=False) -> ModelConfig:
    return ModelConfig(
        vae=VAEConfig(latent_dim=latent, hidden_dims=hidden, num_res_blocks=res),
        student=DiTConfig(latent_dim=latent, d_model=d, n_layers=layers, n_heads=heads, max_seq_len=seq,
                          gradient_checkpointing=ckpt),
        teacher=DiTConfig(latent_dim=latent, d_model=d, n_layers=layers, n_heads=heads, max_seq_len=seq,
                          causal=False, gradient_checkpointing=ckpt),
        image_size=img, sequence_length=seq_len)


def get_small_config() -> ModelConfig:
    return _preset(4, [64, 128, 256], 1, 256, 6, 8, 128, (128, 128), 16)


def get_medium_config() -> ModelConfig:
    return _preset(8, [128, 256, 512], 2, 512, 12, 8, 512, (256, 256), 32)


def get_large_config() -> ModelConfig:
    return _preset(8, [128, 256, 512, 512], 2, 1024, 24, 16, 2048, (512, 512), 64, ckpt=True)
