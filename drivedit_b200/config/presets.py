"""Typed configuration tree and named presets.

One dataclass tree replaces the reference's scattered configs (``config/config.py``,
``config/model_config.py``, per-module dataclasses; three copies of ``REPAConfig``).
Every config serialises to/from JSON (:func:`to_dict` / :func:`from_dict`) and accepts
``key=value`` overrides with dotted paths (:func:`apply_overrides`), e.g.
``model.n_layers=4 train.batch_per_gpu=2``.

Workload presets (latent-video world models; d_head = 64 everywhere):

==================  =====================================================================
``tiny``            4 layers, d=256, 4 heads, SwiGLU 1024, dense frame-causal attention;
                    batch 2 of 4 frames x 16ch x 16x16 latents (64 tokens/frame), 2-D
                    actions; fp32 on CPU
``dit_b``           12 layers, d=768, 12 heads, SwiGLU 3072, SLA (64x64 blocks, top 12.5 %);
                    batch 8/GPU of 16 frames x 16ch x 32x64 (512 tokens/frame), 3-D actions
``moe_dit_l``       24 layers, d=1024, 16 heads, SLA, MoE 64 routed experts (hidden 512),
                    top-6, 2 shared, aux loss; batch 4/GPU of 16 frames
``rollout_dit_b``   the causal ``dit_b`` student streaming 120 frames in chunks of 4 with
                    4 flow steps per chunk and a 32-frame rolling KV window
``moe_2b_repa``     28 layers, d=1536, 24 heads, SLA, MoE 64 experts (hidden 1024), top-6,
                    2 shared; REPA at layer 8 against a frozen ViT-L (24 x 1024, 16x16
                    patches) on 256x512 RGB; batch 2/GPU of 32 frames
==================  =====================================================================
"""
from __future__ import annotations

import copy
import dataclasses
import json
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional


@dataclass
class SLAParams:
    block_size: int = 64
    topk_frac: float = 0.125
    always_diag: bool = True


@dataclass
class MoEParams:
    num_experts: int = 64
    top_k: int = 6
    expert_dim: int = 512
    num_shared: int = 2
    aux_loss_weight: float = 0.01
    bias_update_speed: float = 0.001


@dataclass
class REPAParams:
    layer: int = 8
    weight: float = 0.5
    teacher_layers: int = 24
    teacher_dim: int = 1024
    teacher_heads: int = 16
    teacher_patch: int = 16
    image_h: int = 256
    image_w: int = 512
    proj_hidden: Optional[int] = None  # None: (d_model + teacher_dim) // 2
    feature_layer: int = -1  # teacher layer whose output is aligned to (-1 = last)


@dataclass
class ModelConfig:
    name: str = "tiny"
    n_layers: int = 4
    d_model: int = 256
    n_heads: int = 4
    mlp_hidden: int = 1024
    latent_channels: int = 16
    patch: int = 2
    latent_h: int = 16
    latent_w: int = 16
    action_dim: int = 2
    attention: str = "dense"        # "dense" | "sla"
    causal: str = "frame"           # "frame" | "token" | "none"
    sla: SLAParams = field(default_factory=SLAParams)
    moe: Optional[MoEParams] = None
    rope_base: float = 10000.0
    rope_temporal_factor: float = 1.0
    rope_split: Optional[List[int]] = None
    max_frames: int = 256
    adaln_zero: bool = False
    time_scale: float = 1000.0
    norm_eps: float = 1e-6
    repa: Optional[REPAParams] = None

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_heads

    @property
    def grid_h(self) -> int:
        return self.latent_h // self.patch

    @property
    def grid_w(self) -> int:
        return self.latent_w // self.patch

    @property
    def tokens_per_frame(self) -> int:
        return self.grid_h * self.grid_w

    @property
    def patch_dim(self) -> int:
        return self.latent_channels * self.patch * self.patch


@dataclass
class TrainConfig:
    batch_per_gpu: int = 2
    frames: int = 4
    lr: float = 1e-4
    betas: List[float] = field(default_factory=lambda: [0.9, 0.95])
    weight_decay: float = 0.01
    eps: float = 1e-8
    grad_clip: float = 1.0
    seed: int = 0
    dtype: str = "fp32"             # "fp32" (CPU) | "bf16" (GPU compute)
    t_sampling: str = "logit_normal"  # "logit_normal" | "uniform"
    parallel: str = "dp"            # "dp" | "fsdp" | "fsdp_ep"
    fused_collectives: bool = True
    # FULL_SHARD for the block GEMM weights: each forward GEMM all-gathers its weight's
    # peer-owned pieces itself (fused transport); the optimizer keeps them rank-local
    shard_weights: bool = False
    # fixed-order MoE permutation: bit-reproducible expert gradients (drivedit_b200.ops.debug)
    deterministic: bool = False
    # activation checkpointing (the reference's gradient_checkpointing): each block keeps
    # only its input and recomputes its forward in the backward
    checkpoint_blocks: bool = False
    # reduce each block's gradient bucket during the backward (fused sharded transport);
    # opt-in: at 2 GPUs it measured no faster than reducing after the backward
    overlap_grad_reduce: bool = False


@dataclass
class RolloutConfig:
    total_frames: int = 120
    chunk_frames: int = 4
    flow_steps: int = 4
    window_frames: int = 32
    context_frames: int = 4
    batch: int = 1
    tp: int = 1


@dataclass
class Config:
    model: ModelConfig = field(default_factory=ModelConfig)
    train: TrainConfig = field(default_factory=TrainConfig)
    rollout: RolloutConfig = field(default_factory=RolloutConfig)


def _tiny() -> Config:
    return Config(
        model=ModelConfig(name="tiny", n_layers=4, d_model=256, n_heads=4, mlp_hidden=1024,
                          latent_h=16, latent_w=16, action_dim=2, attention="dense"),
        train=TrainConfig(batch_per_gpu=2, frames=4, dtype="fp32"),
    )


def _dit_b() -> Config:
    return Config(
        model=ModelConfig(name="dit_b", n_layers=12, d_model=768, n_heads=12, mlp_hidden=3072,
                          latent_h=32, latent_w=64, action_dim=3, attention="sla"),
        train=TrainConfig(batch_per_gpu=8, frames=16, dtype="bf16", parallel="fsdp"),
    )


def _moe_dit_l() -> Config:
    return Config(
        model=ModelConfig(name="moe_dit_l", n_layers=24, d_model=1024, n_heads=16,
                          mlp_hidden=0, latent_h=32, latent_w=64, action_dim=3,
                          attention="sla", moe=MoEParams(64, 6, 512, 2, 0.01)),
        train=TrainConfig(batch_per_gpu=4, frames=16, dtype="bf16", parallel="fsdp_ep"),
    )


def _rollout_dit_b() -> Config:
    c = _dit_b()
    c.model.name = "rollout_dit_b"
    c.model.attention = "dense"
    c.rollout = RolloutConfig(total_frames=120, chunk_frames=4, flow_steps=4, window_frames=32,
                              context_frames=4, batch=1)
    return c


def _moe_2b_repa() -> Config:
    return Config(
        model=ModelConfig(name="moe_2b_repa", n_layers=28, d_model=1536, n_heads=24,
                          mlp_hidden=0, latent_h=32, latent_w=64, action_dim=3,
                          attention="sla", moe=MoEParams(64, 6, 1024, 2, 0.01),
                          repa=REPAParams()),
        train=TrainConfig(batch_per_gpu=2, frames=32, dtype="bf16", parallel="fsdp_ep"),
    )


PRESETS = {
    "tiny": _tiny,
    "dit_b": _dit_b,
    "moe_dit_l": _moe_dit_l,
    "rollout_dit_b": _rollout_dit_b,
    "moe_2b_repa": _moe_2b_repa,
}


def get_config(name: str, overrides: Optional[List[str]] = None) -> Config:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    cfg = PRESETS[name]()
    if overrides:
        apply_overrides(cfg, overrides)
    return cfg


def _coerce(old: Any, s: str):
    if isinstance(old, bool):
        return s.lower() in ("1", "true", "yes", "on")
    if isinstance(old, int):
        return int(s)
    if isinstance(old, float):
        return float(s)
    if isinstance(old, list) or s.startswith("["):
        return json.loads(s)
    if old is None:
        try:
            return json.loads(s)
        except json.JSONDecodeError:
            return s
    return s


def apply_overrides(cfg: Any, overrides: List[str]) -> Any:
    for item in overrides:
        key, _, val = item.partition("=")
        obj = cfg
        parts = key.split(".")
        for p in parts[:-1]:
            obj = getattr(obj, p)
        if not hasattr(obj, parts[-1]):
            raise KeyError(f"unknown config key {key!r}")
        setattr(obj, parts[-1], _coerce(getattr(obj, parts[-1]), val))
    return cfg


def to_dict(cfg: Any) -> Dict[str, Any]:
    return dataclasses.asdict(cfg)


def from_dict(d: Dict[str, Any]) -> Config:
    d = copy.deepcopy(d)
    m = d.get("model", {})
    for key, cls in (("sla", SLAParams), ("moe", MoEParams), ("repa", REPAParams)):
        if isinstance(m.get(key), dict):
            m[key] = cls(**m[key])
    return Config(model=ModelConfig(**m), train=TrainConfig(**d.get("train", {})),
                  rollout=RolloutConfig(**d.get("rollout", {})))


def to_json(cfg: Config) -> str:
    return json.dumps(to_dict(cfg), indent=2)
