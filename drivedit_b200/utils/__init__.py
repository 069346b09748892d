"""General helpers: tensors, models / checkpoints, math."""
from .model_utils import count_parameters, load_checkpoint, save_checkpoint, set_seed

__all__ = ["count_parameters", "load_checkpoint", "save_checkpoint", "set_seed"]
