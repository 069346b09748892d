"""Earlier-generation API (the reference's ``core/``): components and the system facade.
The V-JEPA backbone and C-JEPA live in :mod:`drivedit_b200.models.vjepa` and
:mod:`drivedit_b200.models.causal_jepa`."""
from ..models.causal_jepa import CausalJEPAPredictor  # noqa: F401
from ..models.vjepa import VJEPABackbone, VJEPAConfig, create_vjepa_backbone  # noqa: F401
from .base import DriveDiTConfig, DriveDiTSystem, TensorCache  # noqa: F401
from .components import (AdaptiveLayerNorm, CausalVideoTransformer, FlowMatchingPredictor,  # noqa: F401
                         MultiHeadAttention, RoPE3D, SAM2InspiredTracker, TransformerBlock)
