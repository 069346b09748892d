"""The reference's single-object configuration (``config/config.py:12-466``):
``ComponentType`` toggles, per-component sub-configs, ``DriveDiTConfig`` and the
``minimal / research / production / video_only / flow_matching`` presets with
``CONFIG_REGISTRY`` / ``get_config`` / ``list_configs``.

Field names and defaults follow the reference so its JSON configs load unchanged. The
reference's world model reads fields that its config never defines (``moe_num_experts``,
``moe_top_k``, ``moe_capacity_factor``, ``repa_feature_layers``, ``repa_alignment_dim``,
``cjepa_*``, ``rich_cond_*``; ``models/world_model.py:500-666``); here they are properties
derived from the sub-configs, so every component can actually be built.

:meth:`DriveDiTConfig.to_world_config` maps the config onto this framework's latent
world-model preset tree (:mod:`drivedit_b200.config.presets`).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional

from .base import BaseConfig


class ComponentType(Enum):
    CONTROL = "control"
    DEPTH = "depth"
    MEMORY = "memory"
    JEPA = "jepa"
    FLOW_MATCHING = "flow_matching"
    SLA = "sla"
    MOE = "moe"
    REPA = "repa"
    CAUSAL_JEPA = "causal_jepa"
    RICH_CONDITIONING = "rich_conditioning"
    CLOSED_LOOP_EVAL = "closed_loop_eval"


@dataclass
class SLAConfig(BaseConfig):
    block_size: int = 64
    critical_threshold: float = 0.5
    negligible_threshold: float = 0.01
    use_flash_attention: bool = True


@dataclass
class MoEConfig(BaseConfig):
    num_experts: int = 8
    top_k: int = 2
    expert_dim: Optional[int] = None
    num_shared_experts: int = 2
    jitter_noise: float = 0.0
    bias_update_speed: float = 0.001


@dataclass
class REPAConfig(BaseConfig):
    backbone: str = "vjepa2.1"
    alignment_layers: List[int] = field(default_factory=lambda: [6, 12, 18, 24])
    loss_weight: float = 0.1
    haste_enabled: bool = True
    haste_stop_ratio: float = 0.4
    warmup_steps: int = 2000


@dataclass
class CausalJEPAConfig(BaseConfig):
    max_objects: int = 32
    slot_dim: int = 256
    trajectory_length: int = 8
    mask_ratio: float = 0.75
    counterfactual_enabled: bool = True
    num_counterfactuals: int = 4


@dataclass
class ClosedLoopEvalConfig(BaseConfig):
    num_planning_iterations: int = 10
    physics_check_enabled: bool = True
    task_types: List[str] = field(default_factory=lambda: ["lane_keeping", "collision_avoidance",
                                                            "navigation"])
    rollout_horizon: int = 30


def _default_components() -> List[ComponentType]:
    return [ComponentType.CONTROL, ComponentType.MEMORY, ComponentType.FLOW_MATCHING]


@dataclass
class DriveDiTConfig(BaseConfig):
    # architecture
    model_dim: int = 512
    num_layers: int = 12
    num_heads: int = 8
    mlp_ratio: int = 4
    # inputs / outputs
    image_size: int = 256
    patch_size: int = 16
    in_channels: int = 3
    sequence_length: int = 16
    vae_latent_dim: int = 8
    enabled_components: List[ComponentType] = field(default_factory=_default_components)
    # optimisation
    batch_size: int = 8
    learning_rate: float = 1e-4
    weight_decay: float = 0.01
    max_steps: int = 100000
    warmup_steps: int = 1000
    # curriculum and self-forcing
    enable_curriculum: bool = True
    initial_sequence_length: int = 4
    final_sequence_length: int = 32
    curriculum_warmup_steps: int = 10000
    initial_self_forcing_ratio: float = 0.0
    final_self_forcing_ratio: float = 0.8
    self_forcing_warmup_steps: int = 5000
    self_forcing_schedule: str = "cosine"
    max_self_forcing_ratio: float = 0.8
    # flow matching
    enable_flow_matching: bool = True
    flow_matching_weight: float = 1.0
    num_flow_steps: int = 4
    # control
    control_input_dim: int = 6
    control_hidden_dim: int = 256
    control_num_layers: int = 2
    control_dropout: float = 0.1
    # depth
    depth_max_depth: float = 100.0
    depth_channels: int = 1
    # memory
    memory_dim: int = 512
    object_memory_size: int = 64
    spatial_memory_size: int = 256
    memory_update_rate: float = 0.1
    # JEPA
    jepa_target_length: int = 4
    jepa_prediction_head_dim: int = 512
    jepa_temperature: float = 0.1
    # stability
    gradient_clip_norm: float = 1.0
    mixed_precision: bool = True
    checkpoint_every: int = 1000
    # distributed
    distributed: bool = False
    local_rank: int = 0
    world_size: int = 1
    # memory management
    max_memory_gb: float = 16.0
    memory_cleanup_threshold: float = 0.8
    # data pipeline
    video_chunk_duration: int = 300
    video_overlap_duration: int = 30
    use_scene_detection: bool = True
    min_quality_score: float = 0.7
    # loss weights
    reconstruction_weight: float = 1.0
    temporal_consistency_weight: float = 0.2
    jepa_weight: float = 0.1
    perceptual_weight: float = 0.1
    l1_weight: float = 0.1
    # v2 components
    sla_config: SLAConfig = field(default_factory=SLAConfig)
    moe_config: MoEConfig = field(default_factory=MoEConfig)
    repa_config: REPAConfig = field(default_factory=REPAConfig)
    causal_jepa_config: CausalJEPAConfig = field(default_factory=CausalJEPAConfig)
    closed_loop_eval_config: ClosedLoopEvalConfig = field(default_factory=ClosedLoopEvalConfig)

    def validate(self):
        if self.model_dim % self.num_heads:
            raise ValueError("model_dim must be divisible by num_heads")
        if self.image_size % self.patch_size:
            raise ValueError("image_size must be a multiple of patch_size")
        # JSON round trips hand back strings; keep the component list typed
        self.enabled_components = [c if isinstance(c, ComponentType) else ComponentType(c)
                                   for c in self.enabled_components]

    # ---------------------------------------------------------------- components
    def get_enabled_components(self) -> List[ComponentType]:
        return self.enabled_components

    def is_component_enabled(self, component: ComponentType) -> bool:
        return component in self.enabled_components

    def enable_component(self, component: ComponentType):
        if component not in self.enabled_components:
            self.enabled_components.append(component)

    def disable_component(self, component: ComponentType):
        if component in self.enabled_components:
            self.enabled_components.remove(component)

    # ---------------------------------------------------------------- views
    def get_model_config(self) -> Dict[str, Any]:
        keys = ("model_dim", "num_layers", "num_heads", "mlp_ratio", "image_size", "patch_size",
                "in_channels", "sequence_length", "vae_latent_dim", "enabled_components")
        return {k: getattr(self, k) for k in keys}

    def get_training_config(self) -> Dict[str, Any]:
        keys = ("batch_size", "learning_rate", "weight_decay", "max_steps", "warmup_steps",
                "enable_curriculum", "curriculum_warmup_steps", "initial_self_forcing_ratio",
                "final_self_forcing_ratio", "self_forcing_warmup_steps", "enable_flow_matching",
                "flow_matching_weight", "gradient_clip_norm", "mixed_precision")
        return {k: getattr(self, k) for k in keys}

    def get_data_config(self) -> Dict[str, Any]:
        keys = ("batch_size", "sequence_length", "image_size", "video_chunk_duration",
                "video_overlap_duration", "use_scene_detection", "min_quality_score")
        return {k: getattr(self, k) for k in keys}

    # ---------------------------------------------------------------- derived fields
    @property
    def moe_num_experts(self) -> int:
        return self.moe_config.num_experts

    @property
    def moe_top_k(self) -> int:
        return self.moe_config.top_k

    @property
    def moe_capacity_factor(self) -> float:
        return 1.0   # dropless routing: every token reaches its k experts

    @property
    def repa_feature_layers(self) -> List[int]:
        return [l for l in self.repa_config.alignment_layers if l < self.num_layers] or [self.num_layers // 2]

    @property
    def repa_alignment_dim(self) -> int:
        return 256

    @property
    def cjepa_slot_dim(self) -> int:
        return self.causal_jepa_config.slot_dim

    @property
    def cjepa_num_slots(self) -> int:
        return self.causal_jepa_config.max_objects

    @property
    def cjepa_num_iterations(self) -> int:
        return 3

    @property
    def cjepa_prediction_horizon(self) -> int:
        return self.causal_jepa_config.trajectory_length

    @property
    def cjepa_temperature(self) -> float:
        return 0.1

    @property
    def rich_cond_dim(self) -> int:
        return self.model_dim

    @property
    def rich_cond_num_cameras(self) -> int:
        return 1

    @property
    def rich_cond_max_waypoints(self) -> int:
        return 20

    @property
    def rich_cond_max_objects(self) -> int:
        return 32

    @property
    def rich_cond_cfg_dropout(self) -> float:
        return 0.1

    def to_world_config(self):
        """This config as a latent world-model preset of this framework: the DiT works on
        VAE latents (8x spatial compression, patch 2) instead of 16x16 pixel patches."""
        from .presets import Config, ModelConfig, MoEParams, SLAParams, TrainConfig

        moe = None
        if self.is_component_enabled(ComponentType.MOE):
            c = self.moe_config
            from ..layers.moe import default_expert_dim

            moe = MoEParams(c.num_experts, c.top_k, c.expert_dim or default_expert_dim(self.model_dim, c.top_k),
                            c.num_shared_experts, 0.01, c.bias_update_speed)
        lat = max(2, self.image_size // 8)
        m = ModelConfig(name="drivedit", n_layers=self.num_layers, d_model=self.model_dim,
                        n_heads=self.num_heads, mlp_hidden=self.model_dim * self.mlp_ratio,
                        latent_channels=self.vae_latent_dim, latent_h=lat, latent_w=lat,
                        action_dim=self.control_input_dim,
                        attention="sla" if self.is_component_enabled(ComponentType.SLA) else "dense",
                        sla=SLAParams(block_size=self.sla_config.block_size), moe=moe)
        t = TrainConfig(batch_per_gpu=self.batch_size, frames=self.sequence_length, lr=self.learning_rate,
                        weight_decay=self.weight_decay, grad_clip=self.gradient_clip_norm,
                        dtype="bf16" if self.mixed_precision else "fp32")
        return Config(model=m, train=t)


def get_minimal_config() -> DriveDiTConfig:
    return DriveDiTConfig(model_dim=256, num_layers=6, num_heads=4, sequence_length=8, image_size=128,
                          batch_size=4, max_steps=10000, enabled_components=[ComponentType.CONTROL],
                          enable_curriculum=True, initial_sequence_length=2, final_sequence_length=8,
                          curriculum_warmup_steps=1000, enable_flow_matching=True, num_flow_steps=2,
                          max_memory_gb=4.0)


def get_research_config() -> DriveDiTConfig:
    C = ComponentType
    return DriveDiTConfig(model_dim=768, num_layers=24, num_heads=12, sequence_length=32, image_size=256,
                          batch_size=8, max_steps=200000, learning_rate=5e-5,
                          enabled_components=[C.CONTROL, C.DEPTH, C.MEMORY, C.JEPA, C.FLOW_MATCHING,
                                              C.SLA, C.REPA, C.CAUSAL_JEPA, C.CLOSED_LOOP_EVAL],
                          enable_curriculum=True, initial_sequence_length=4, final_sequence_length=32,
                          curriculum_warmup_steps=20000, initial_self_forcing_ratio=0.0,
                          final_self_forcing_ratio=0.9, self_forcing_warmup_steps=10000,
                          enable_flow_matching=True, num_flow_steps=4, flow_matching_weight=1.0,
                          max_memory_gb=32.0)


def get_production_config() -> DriveDiTConfig:
    C = ComponentType
    return DriveDiTConfig(model_dim=1024, num_layers=32, num_heads=16, sequence_length=64, image_size=512,
                          batch_size=16, max_steps=1000000, learning_rate=1e-4,
                          enabled_components=[C.CONTROL, C.MEMORY, C.FLOW_MATCHING],
                          enable_curriculum=True, initial_sequence_length=8, final_sequence_length=64,
                          curriculum_warmup_steps=50000, initial_self_forcing_ratio=0.1,
                          final_self_forcing_ratio=0.95, self_forcing_warmup_steps=25000,
                          enable_flow_matching=True, num_flow_steps=4, distributed=True,
                          max_memory_gb=128.0, video_chunk_duration=600, min_quality_score=0.8)


def get_video_only_config() -> DriveDiTConfig:
    C = ComponentType
    return DriveDiTConfig(model_dim=512, num_layers=16, num_heads=8, sequence_length=24,
                          enabled_components=[C.MEMORY, C.JEPA, C.FLOW_MATCHING], batch_size=6,
                          max_steps=150000, temporal_consistency_weight=0.5, jepa_weight=0.3,
                          enable_flow_matching=True, flow_matching_weight=2.0)


def get_flow_matching_config() -> DriveDiTConfig:
    return DriveDiTConfig(model_dim=512, num_layers=12, num_heads=8,
                          enabled_components=[ComponentType.FLOW_MATCHING], enable_flow_matching=True,
                          flow_matching_weight=5.0, num_flow_steps=8, enable_curriculum=True,
                          initial_sequence_length=2, final_sequence_length=12, batch_size=8,
                          learning_rate=2e-4, max_steps=50000)


CONFIG_REGISTRY = {
    "minimal": get_minimal_config,
    "research": get_research_config,
    "production": get_production_config,
    "video_only": get_video_only_config,
    "flow_matching": get_flow_matching_config,
}


def get_config(config_name: str) -> DriveDiTConfig:
    if config_name not in CONFIG_REGISTRY:
        raise ValueError(f"Unknown config: {config_name}. Available: {list(CONFIG_REGISTRY)}")
    return CONFIG_REGISTRY[config_name]()


def list_configs() -> List[str]:
    return list(CONFIG_REGISTRY)
