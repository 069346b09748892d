from .presets import (Config, ModelConfig, MoEParams, PRESETS, REPAParams, RolloutConfig,
                      SLAParams, TrainConfig, apply_overrides, from_dict, get_config, to_dict,
                      to_json)

from .base import (BaseConfig, create_config_from_args, get_config_diff, load_config, merge_configs,
                   save_config)
from .unified import (CONFIG_REGISTRY, CausalJEPAConfig, ClosedLoopEvalConfig, ComponentType,
                      DriveDiTConfig, MoEConfig, REPAConfig, SLAConfig, get_flow_matching_config,
                      get_minimal_config, get_production_config, get_research_config,
                      get_video_only_config, list_configs)

# ``get_config(name, overrides)`` returns this framework's workload presets; the reference's
# ``get_config(name) -> DriveDiTConfig`` is ``drivedit_b200.config.unified.get_config``.
__all__ = ["BaseConfig", "CONFIG_REGISTRY", "CausalJEPAConfig", "ClosedLoopEvalConfig", "ComponentType",
           "DriveDiTConfig", "MoEConfig", "REPAConfig", "SLAConfig", "create_config_from_args",
           "get_config_diff", "get_flow_matching_config", "get_minimal_config", "get_production_config",
           "get_research_config", "get_video_only_config", "list_configs", "load_config", "merge_configs",
           "save_config",
"Config", "ModelConfig", "MoEParams", "PRESETS", "REPAParams", "RolloutConfig",
           "SLAParams", "TrainConfig", "apply_overrides", "from_dict", "get_config",
           "to_dict", "to_json"]
