from .presets import (Config, ModelConfig, MoEParams, PRESETS, REPAParams, RolloutConfig,
                      SLAParams, TrainConfig, apply_overrides, from_dict, get_config, to_dict,
                      to_json)

__all__ = ["Config", "ModelConfig", "MoEParams", "PRESETS", "REPAParams", "RolloutConfig",
           "SLAParams", "TrainConfig", "apply_overrides", "from_dict", "get_config",
           "to_dict", "to_json"]
