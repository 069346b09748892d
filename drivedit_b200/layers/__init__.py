"""PyTorch layer library (CPU path and numerical oracle for the sm_100a kernels)."""
from .attention import (AttentionBackend, BidirectionalMultiHeadAttention, CausalMultiHeadAttention,
                        CrossAttention, KVCache, MultiHeadAttention, attention_reference,
                        create_block_causal_mask, create_causal_mask, frame_causal_mask,
                        get_attention_backend, get_available_backends, mha,
                        set_attention_backend)
from .helpers import (FusedMLP, PositionalEncoding, ScaledDotProductAttention,
                      apply_rotary_pos_emb, fused_add_norm, gelu_tanh, silu)
from .mlp import GeGLU, MLP, ConditionalMLP, SwiGLU, create_mlp, pack_swiglu, unpack_swiglu
from .moe import ExpertFFN, MoEFFN, MoEOutput, Router, aux_load_balance_loss
from .norms import AdaLN, AdaLNZero, LayerNorm, RMSNorm
from .rope import RoPE3D, RoPELayer, apply_rope, rope_angles_3d, rope_apply, rope_table
from .rope_v2 import (RoPEConfig, RoPEFrequencyCache, RoPELayerV2, apply_rope_3d_efficient,
                      compute_resolution_aware_rope_freqs, compute_rope_3d_freqs,
                      interpolate_rope_freqs)
from .sla import (CausalSparseLinearAttention, SLAConfig, SparseLinearAttention,
                  create_sla_layer, sla_reference, sla_route)
