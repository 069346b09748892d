"""Component-toggled world model over RGB frames (the reference's ``models/world_model.py``
orchestrator: ``WorldModel(config: DriveDiTConfig)`` with the control / depth / memory /
JEPA / flow-matching heads, the v2 MoE / SLA / REPA / C-JEPA / rich-conditioning parts and
the ``train / inference / self_forcing / sla / rich_cond / cjepa`` forward modes).

Differences from the reference, each a fix of something it does not do:

* context tokens (controls, depth, retrieved memory) come *before* the frame tokens; the
  reference appends them after the frame tokens (``:976-990``), where its token-causal mask
  hides them from every frame token;
* the memory system is used (its retrieval is a context token); the reference builds it and
  never calls it;
* ``inference`` decodes incrementally with per-layer KV caches (each new frame costs one
  frame of tokens); the reference re-runs the whole window per step (``:1023-1061``);
* ``switch_attention_mode("sla")`` / ``forward_with_sla`` really compute sparse-linear
  attention (block top-k softmax + linear branch, :mod:`drivedit_b200.layers.sla`) with the
  blocks' own projections; the reference only flips a flag (``:1173-1200``);
* rich conditioning modulates every block through AdaLN; the reference computes it and
  drops it (``:1255-1262``);
* fields the reference reads but never defines come from :class:`DriveDiTConfig`
  properties, so the MoE / REPA / C-JEPA / rich-conditioning parts all build.

The latent-video training and serving hot path is :class:`~drivedit_b200.models.world_dit.WorldDiT`
with the fused sm_100a engine; this module is the reference-compatible research API.
"""
from __future__ import annotations

import logging
import math
import warnings
from typing import Any, Dict, List, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config.unified import ComponentType, DriveDiTConfig
from .blocks import DiTBlock, MoEDiTBlock

logger = logging.getLogger(__name__)

_AVAILABLE = {c: True for c in ComponentType}


def check_component_availability(component: ComponentType) -> bool:
    """Every component is implemented in this framework."""
    return _AVAILABLE.get(component, False)


class PatchEmbed(nn.Module):
    """``[B, C, H, W]`` -> ``[B, (H/p)(W/p), D]`` non-overlapping patch projection."""

    def __init__(self, img_size: int = 224, patch_size: int = 16, in_chans: int = 3, embed_dim: int = 768):
        super().__init__()
        self.img_size, self.patch_size = img_size, patch_size
        self.num_patches = (img_size // patch_size) ** 2
        self.proj = nn.Conv2d(in_chans, embed_dim, kernel_size=patch_size, stride=patch_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.proj(x).flatten(2).transpose(1, 2)


class ControlEncoder(nn.Module):
    """MLP over control vectors (ReLU + dropout between layers)."""

    def __init__(self, input_dim: int, hidden_dim: int, output_dim: int, num_layers: int = 2,
                 dropout: float = 0.1):
        super().__init__()
        layers: List[nn.Module] = []
        for i in range(num_layers):
            last = i == num_layers - 1
            layers.append(nn.Linear(input_dim if i == 0 else hidden_dim, output_dim if last else hidden_dim))
            if not last:
                layers += [nn.ReLU(), nn.Dropout(dropout)]
        self.encoder = nn.Sequential(*layers)

    def forward(self, controls: torch.Tensor) -> torch.Tensor:
        return self.encoder(controls)


class DepthEncoder(nn.Module):
    """Depth map (clamped to ``[0, max_depth]`` and normalised) -> 16x16 = 256 tokens."""

    def __init__(self, input_dim: int, output_dim: int, max_depth: float = 100.0):
        super().__init__()
        self.max_depth = max_depth
        self.encoder = nn.Sequential(
            nn.Conv2d(input_dim, 64, 3, padding=1), nn.ReLU(),
            nn.Conv2d(64, 128, 3, stride=2, padding=1), nn.ReLU(),
            nn.Conv2d(128, output_dim, 3, stride=2, padding=1),
            nn.AdaptiveAvgPool2d((16, 16)), nn.Flatten(2))

    def forward(self, depth: torch.Tensor) -> torch.Tensor:
        return self.encoder(torch.clamp(depth / self.max_depth, 0, 1)).transpose(-2, -1)


class MemorySystem(nn.Module):
    """Learned object / spatial memory banks read by cross-attention from a pooled query."""

    def __init__(self, dim: int, max_objects: int = 64, max_spatial: int = 256, num_heads: int = 8):
        super().__init__()
        from ..layers.attention import CrossAttention

        self.dim, self.max_objects, self.max_spatial = dim, max_objects, max_spatial
        self.object_memory = nn.Parameter(torch.randn(max_objects, dim) * 0.02)
        self.spatial_memory = nn.Parameter(torch.randn(max_spatial, dim) * 0.02)
        self.object_update = nn.Linear(dim, dim)
        self.spatial_update = nn.Linear(dim, dim)
        heads = num_heads if dim % num_heads == 0 else 1
        self.memory_retrieval = CrossAttention(dim, heads)
        nn.init.normal_(self.memory_retrieval.proj.weight, std=0.02)

    def get_memory_tokens(self, batch_size: int) -> torch.Tensor:
        m = torch.cat([self.object_memory, self.spatial_memory], 0)
        return m.unsqueeze(0).expand(batch_size, -1, -1)

    def forward(self, hidden_states: torch.Tensor, step: int = 0) -> torch.Tensor:
        """``[B, T, D]`` -> retrieved memory broadcast to ``[B, T, D]``."""
        B, T, _ = hidden_states.shape
        q = hidden_states.mean(1, keepdim=True)
        r = self.memory_retrieval(q, self.get_memory_tokens(B))
        return r.expand(B, T, -1)


class JEPAPredictor(nn.Module):
    """Predicts ``target_length`` future representations from the mean of the last 4 tokens."""

    def __init__(self, input_dim: int, target_length: int, prediction_head_dim: int):
        super().__init__()
        self.target_length = target_length
        self.predictor = nn.Sequential(nn.Linear(input_dim, prediction_head_dim), nn.ReLU(),
                                       nn.Linear(prediction_head_dim, input_dim * target_length))

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        B, _, D = hidden_states.shape
        return self.predictor(hidden_states[:, -4:].mean(1)).view(B, self.target_length, D)


class FlowMatchingPredictor(nn.Module):
    """Time-conditioned velocity MLP over pooled states with Euler sampling (the reference's
    ignores ``t``; here ``t`` enters through sinusoidal features)."""

    def __init__(self, dim: int, num_steps: int = 4):
        super().__init__()
        self.dim, self.num_steps = dim, num_steps
        self.time_proj = nn.Linear(64, dim)
        self.flow_net = nn.Sequential(nn.Linear(dim, dim * 2), nn.SiLU(), nn.Linear(dim * 2, dim), nn.SiLU(),
                                      nn.Linear(dim, dim), nn.Tanh())

    def forward(self, z: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        half = torch.exp(-math.log(10000.0) * torch.arange(32, device=z.device) / 32)
        ang = t.float()[:, None] * 1000.0 * half[None]
        te = self.time_proj(torch.cat([ang.sin(), ang.cos()], -1)).to(z.dtype)
        return self.flow_net(z + te)

    @torch.no_grad()
    def sample(self, z_init: torch.Tensor, num_steps: Optional[int] = None) -> torch.Tensor:
        n = num_steps or self.num_steps
        z = z_init.clone()
        for i in range(n):
            t = torch.full((z.shape[0],), i / n, device=z.device)
            z = z + self.forward(z, t) / n
        return z


class SelfForcingScheduler:
    """Self-forcing ratio by step: linear, cosine or exponential approach to the final ratio."""

    def __init__(self, config: DriveDiTConfig):
        self.config = config
        self.step = 0

    def update(self, step: int):
        self.step = step

    def get_ratio(self) -> float:
        c = self.config
        p = min(1.0, self.step / max(c.self_forcing_warmup_steps, 1))
        a, b = c.initial_self_forcing_ratio, c.final_self_forcing_ratio
        if c.self_forcing_schedule == "linear":
            return a + p * (b - a)
        if c.self_forcing_schedule == "cosine":
            return a + 0.5 * (1 - math.cos(math.pi * p)) * (b - a)
        return b + (a - b) * 0.999 ** self.step


class REPAAlignmentHead(nn.Module):
    """Linear -> LayerNorm (-> GELU) stack projecting hidden states for REPA alignment."""

    def __init__(self, model_dim: int, alignment_dim: int = 256, num_layers: int = 2):
        super().__init__()
        layers: List[nn.Module] = []
        for i in range(num_layers):
            layers += [nn.Linear(model_dim if i == 0 else alignment_dim, alignment_dim), nn.LayerNorm(alignment_dim)]
            if i < num_layers - 1:
                layers.append(nn.GELU())
        self.projection = nn.Sequential(*layers)

    def forward(self, features: torch.Tensor) -> torch.Tensor:
        return self.projection(features)


class WorldModel(nn.Module):
    def __init__(self, config: DriveDiTConfig):
        super().__init__()
        self.config = config
        self.enabled_components = config.get_enabled_components()
        self._active_components: List[ComponentType] = []
        self._unavailable_components: List[ComponentType] = []
        C = ComponentType
        self.tokens_per_frame = (config.image_size // config.patch_size) ** 2
        self.max_seq_len = self.tokens_per_frame * config.final_sequence_length + 512
        self._attention_mode = "sla" if C.SLA in self.enabled_components else "standard"
        rich = C.RICH_CONDITIONING in self.enabled_components
        cond_dim = config.rich_cond_dim if rich else None
        self.use_moe = C.MOE in self.enabled_components
        d, H = config.model_dim, config.num_heads
        if self.use_moe:
            m = config.moe_config
            self.backbone = nn.ModuleList([
                MoEDiTBlock(d, H, num_experts=m.num_experts, top_k=m.top_k, expert_dim=m.expert_dim,
                            num_shared_experts=m.num_shared_experts, causal=True, max_seq_len=self.max_seq_len,
                            cond_dim=cond_dim, jitter_noise=m.jitter_noise,
                            bias_update_speed=m.bias_update_speed, aux_loss_weight=1.0)
                for _ in range(config.num_layers)])
            self._active_components.append(C.MOE)
        else:
            self.backbone = nn.ModuleList([
                DiTBlock(d, H, d_ff=d * config.mlp_ratio, causal=True, max_seq_len=self.max_seq_len,
                         cond_dim=cond_dim)
                for _ in range(config.num_layers)])
        self.patch_embed = PatchEmbed(config.image_size, config.patch_size, config.in_channels, d)
        self.control_encoder = self.depth_encoder = self.memory_system = None
        self.flow_predictor = self.jepa_predictor = None
        if C.CONTROL in self.enabled_components:
            self.control_encoder = ControlEncoder(config.control_input_dim, config.control_hidden_dim, d,
                                                  config.control_num_layers, config.control_dropout)
            self._active_components.append(C.CONTROL)
        if C.DEPTH in self.enabled_components:
            self.depth_encoder = DepthEncoder(config.depth_channels, d, config.depth_max_depth)
            self._active_components.append(C.DEPTH)
        if C.MEMORY in self.enabled_components:
            self.memory_system = MemorySystem(config.memory_dim, config.object_memory_size,
                                              config.spatial_memory_size)
            self.memory_proj = nn.Linear(config.memory_dim, d) if config.memory_dim != d else nn.Identity()
            self._active_components.append(C.MEMORY)
        if C.FLOW_MATCHING in self.enabled_components:
            self.flow_predictor = FlowMatchingPredictor(d, config.num_flow_steps)
            self._active_components.append(C.FLOW_MATCHING)
        if C.JEPA in self.enabled_components:
            self.jepa_predictor = JEPAPredictor(d, config.jepa_target_length, config.jepa_prediction_head_dim)
            self._active_components.append(C.JEPA)
        if C.SLA in self.enabled_components:
            self._active_components.append(C.SLA)
        self.cjepa_predictor = None
        if C.CAUSAL_JEPA in self.enabled_components:
            from .causal_jepa import CausalJEPAConfig, CausalJEPAPredictor

            cj = config.causal_jepa_config
            self.cjepa_predictor = CausalJEPAPredictor(CausalJEPAConfig(
                input_dim=d, slot_dim=config.cjepa_slot_dim, max_objects=config.cjepa_num_slots,
                num_slot_iterations=config.cjepa_num_iterations,
                prediction_horizon=config.cjepa_prediction_horizon, mask_ratio=cj.mask_ratio,
                enable_counterfactual=cj.counterfactual_enabled, num_counterfactuals=cj.num_counterfactuals))
            self._active_components.append(C.CAUSAL_JEPA)
        self.rich_conditioning = None
        if rich:
            from .conditioning import create_conditioning_module

            self.rich_conditioning = create_conditioning_module(
                model_dim=d, cond_dim=config.rich_cond_dim, num_cameras=config.rich_cond_num_cameras,
                max_waypoints=config.rich_cond_max_waypoints, max_objects=config.rich_cond_max_objects,
                cfg_dropout_prob=config.rich_cond_cfg_dropout)
            self._active_components.append(C.RICH_CONDITIONING)
        self.repa_heads = None
        if C.REPA in self.enabled_components:
            self.repa_heads = nn.ModuleDict({str(l): REPAAlignmentHead(d, config.repa_alignment_dim)
                                             for l in config.repa_feature_layers})
            self._active_components.append(C.REPA)
        if C.CLOSED_LOOP_EVAL in self.enabled_components:
            self._active_components.append(C.CLOSED_LOOP_EVAL)
        self.frame_head = nn.Linear(d, config.vae_latent_dim)
        self.self_forcing_scheduler = SelfForcingScheduler(config)
        self.past_kvs: Optional[List[Dict[str, torch.Tensor]]] = None
        self._intermediate_features: Dict[int, torch.Tensor] = {}
        logger.info("WorldModel: active %s", [c.value for c in self._active_components])

    # ------------------------------------------------------------------ status
    def get_active_components(self) -> List[ComponentType]:
        return list(self._active_components)

    def get_unavailable_components(self) -> List[ComponentType]:
        return list(self._unavailable_components)

    def is_component_active(self, component: ComponentType) -> bool:
        return component in self._active_components

    def get_component_status(self) -> Dict[str, Any]:
        return {"active": [c.value for c in self._active_components],
                "unavailable": [c.value for c in self._unavailable_components],
                "requested": [c.value for c in self.enabled_components],
                "use_moe": self.use_moe, "attention_mode": self._attention_mode,
                "availability": {c.value: check_component_availability(c) for c in ComponentType}}

    def switch_attention_mode(self, mode: str) -> None:
        if mode not in ("standard", "sla", "flash"):
            raise ValueError(f"Invalid attention mode: {mode}. Valid: ['standard', 'sla', 'flash']")
        self._attention_mode = mode

    def get_attention_mode(self) -> str:
        return self._attention_mode

    # ------------------------------------------------------------------ features
    def get_object_slots(self, hidden_states: torch.Tensor, return_attention: bool = False):
        if self.cjepa_predictor is None:
            raise RuntimeError("C-JEPA predictor not initialized: enable CAUSAL_JEPA")
        so = self.cjepa_predictor.slot_encoder(hidden_states)
        return (so["slots"], so.get("attention")) if return_attention else so["slots"]

    def get_intermediate_features(self, layer_indices: Optional[List[int]] = None) -> Dict[int, torch.Tensor]:
        if layer_indices is None:
            return dict(self._intermediate_features)
        return {i: self._intermediate_features[i] for i in layer_indices if i in self._intermediate_features}

    def get_repa_projections(self, features: Optional[Dict[int, torch.Tensor]] = None) -> Dict[int, torch.Tensor]:
        if self.repa_heads is None:
            raise RuntimeError("REPA heads not initialized: enable REPA")
        features = self._intermediate_features if features is None else features
        return {int(k): h(features[int(k)]) for k, h in self.repa_heads.items() if int(k) in features}

    # ------------------------------------------------------------------ forward
    def forward(self, frames: torch.Tensor, controls: Optional[torch.Tensor] = None,
                depth: Optional[torch.Tensor] = None, mode: str = "train", **kw) -> Dict[str, torch.Tensor]:
        if mode == "train":
            return self._forward_train(frames, controls, depth, **kw)
        if mode == "inference":
            return self._forward_inference(frames, controls, depth, **kw)
        if mode == "self_forcing":
            return self._forward_self_forcing(frames, controls, depth, **kw)
        if mode == "sla":
            return self.forward_with_sla(frames, controls, depth, **kw)
        if mode == "rich_cond":
            return self.forward_with_rich_conditioning(frames, **kw)
        if mode == "cjepa":
            return self.forward_cjepa(frames, controls, depth, **kw)
        raise ValueError(f"Unknown mode: {mode}")

    def _sla_attention(self, blk, h: torch.Tensor, kv_cache, start_pos: int):
        """The block's attention computed as sparse-linear attention (same projections)."""
        from ..layers.sla import SLAConfig, sla_reference

        a = blk.attn
        B, T, D = h.shape
        q, k, v = a.qkv(h).view(B, T, 3, a.n_heads, a.d_head).unbind(2)
        q, k = a._rope(q, start_pos), a._rope(k, start_pos)
        new = None
        if isinstance(kv_cache, dict):
            if kv_cache.get("k") is not None:
                k = torch.cat([kv_cache["k"], k], 1)
                v = torch.cat([kv_cache["v"], v], 1)
            new = {"k": k.detach(), "v": v.detach()}
        sc = self.config.sla_config
        cfg = SLAConfig(block_size=min(sc.block_size, T), causal=True,
                        critical_threshold=sc.critical_threshold,
                        negligible_threshold=sc.negligible_threshold)
        if k.shape[1] != T:     # cached decode: a query block against the whole key set
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
        else:
            o = sla_reference(q, k, v, cfg)
        return a.proj(o.reshape(B, T, D)), new

    def _forward_backbone(self, tokens: torch.Tensor, capture_intermediate: bool = False,
                          kv_cache: Optional[List[Dict[str, torch.Tensor]]] = None, start_pos: int = 0,
                          cond: Optional[torch.Tensor] = None):
        x = tokens
        new_cache: List[Dict[str, torch.Tensor]] = []
        if capture_intermediate:
            self._intermediate_features = {}
        capture = {int(i) for i in self.repa_heads.keys()} if (capture_intermediate and self.repa_heads) else set()
        sla = self._attention_mode == "sla"
        for i, blk in enumerate(self.backbone):
            cache = kv_cache[i] if kv_cache is not None and i < len(kv_cache) else ({} if kv_cache is not None else None)
            if sla:
                h = blk._norm(blk.norm_attn, x, cond)
                a, nc = self._sla_attention(blk, h, cache, start_pos)
                x = x + a
                hm = blk._norm(blk.norm_mlp, x, cond)
                if isinstance(blk, MoEDiTBlock):
                    out = blk.moe_ffn(hm)
                    blk._last_aux_loss = out.aux_loss
                    x = x + out.output
                else:
                    x = x + blk.mlp(hm)
            else:
                x, nc = blk(x, kv_cache=cache, cond=cond, start_pos=start_pos)
            if nc is not None:
                new_cache.append(nc)
            if i in capture:
                self._intermediate_features[i] = x
        return x, (new_cache or None)

    def _context_tokens(self, B: int, T: int, controls, depth, frame_tokens) -> Optional[torch.Tensor]:
        ctx = []
        if self.control_encoder is not None and controls is not None:
            c = self.control_encoder(controls.to(frame_tokens.dtype))
            ctx.append(c.unsqueeze(1) if c.dim() == 2 else c)
        if self.depth_encoder is not None and depth is not None:
            dt = self.depth_encoder(depth.reshape(-1, *depth.shape[-3:]).to(frame_tokens.dtype))
            ctx.append(dt.reshape(B, -1, dt.shape[-1]))
        if self.memory_system is not None:
            mem = self.memory_system(frame_tokens)[:, :1]
            ctx.append(self.memory_proj(mem))
        return torch.cat(ctx, 1) if ctx else None

    def _embed(self, frames: torch.Tensor) -> torch.Tensor:
        B, T = frames.shape[:2]
        tok = self.patch_embed(frames.reshape(-1, *frames.shape[2:]))
        return tok.reshape(B, T * tok.shape[1], tok.shape[2])

    def _forward_train(self, frames: torch.Tensor, controls: Optional[torch.Tensor] = None,
                       depth: Optional[torch.Tensor] = None, capture_intermediate: bool = False,
                       cond: Optional[torch.Tensor] = None, return_cache: bool = False, **kw):
        B, T = frames.shape[:2]
        ft = self._embed(frames)
        ctx = self._context_tokens(B, T, controls, depth, ft)
        n_ctx = 0 if ctx is None else ctx.shape[1]
        tokens = ft if ctx is None else torch.cat([ctx, ft], 1)
        capture = capture_intermediate or self.repa_heads is not None
        h, cache = self._forward_backbone(tokens, capture, kv_cache=[] if return_cache else None, cond=cond)
        fh = h[:, n_ctx:]
        out: Dict[str, torch.Tensor] = {"predictions": self._decode_frame_tokens(self.frame_head(fh), B, T),
                                        "hidden_states": fh}
        if self.jepa_predictor is not None:
            out["jepa_predictions"] = self.jepa_predictor(fh)
        if self.flow_predictor is not None:
            t = torch.rand(B, device=frames.device)
            out["flow_predictions"] = self.flow_predictor(fh.mean(1), t)
        if self.cjepa_predictor is not None:
            cj = self.cjepa_predictor(fh.reshape(B, T, -1, fh.shape[-1]))
            out["cjepa_slots"] = cj["slots"]
            out["cjepa_predictions"] = cj["predicted_slots"]
        if self.repa_heads is not None and self._intermediate_features:
            out["repa_projections"] = self.get_repa_projections(
                {i: f[:, n_ctx:] for i, f in self._intermediate_features.items()})
        if return_cache:
            out["_cache"] = cache
            out["_length"] = tokens.shape[1]
        return out

    @torch.no_grad()
    def _forward_inference(self, frames: torch.Tensor, controls: Optional[torch.Tensor] = None,
                           depth: Optional[torch.Tensor] = None, num_steps: int = 1,
                           use_kv_cache: bool = True, **kw) -> Dict[str, torch.Tensor]:
        """Generates ``num_steps`` frames; each step feeds the last prediction back. With the
        cache, a step runs one frame of tokens against the cached keys / values."""
        B = frames.shape[0]
        self.reset_cache()
        out = self._forward_train(frames, controls, depth, return_cache=use_kv_cache)
        gen = [out["predictions"][:, -1:]]
        cache, length = out.get("_cache"), out.get("_length", 0)
        window = frames
        for _ in range(num_steps - 1):
            nxt = gen[-1]
            if use_kv_cache and cache is not None and length + self.tokens_per_frame <= self.max_seq_len:
                tok = self._embed(nxt)
                h, cache = self._forward_backbone(tok, kv_cache=cache, start_pos=length)
                length += tok.shape[1]
                gen.append(self._decode_frame_tokens(self.frame_head(h), B, 1))
                self.past_kvs = cache
            else:   # window full (or no cache): slide and re-encode
                window = torch.cat([window[:, 1:], nxt], 1)
                o = self._forward_train(window, controls, depth, return_cache=use_kv_cache)
                cache, length = o.get("_cache"), o.get("_length", 0)
                gen.append(o["predictions"][:, -1:])
        return {"generated_frames": torch.cat(gen, 1), "final_states": out["hidden_states"]}

    def _forward_self_forcing(self, frames: torch.Tensor, controls: Optional[torch.Tensor] = None,
                              depth: Optional[torch.Tensor] = None, self_forcing_ratio: Optional[float] = None,
                              **kw) -> Dict[str, torch.Tensor]:
        """First half of the clip is context; each later frame's input is the ground truth
        with probability ``1 - ratio`` and the model's previous prediction otherwise."""
        T = frames.shape[1]
        ratio = self.self_forcing_scheduler.get_ratio() if self_forcing_ratio is None else self_forcing_ratio
        L = max(1, T // 2)
        ctx, tgt = frames[:, :L], frames[:, L:]
        sl = lambda x, n: None if x is None else (x[:, :n] if x.dim() >= 3 else x)
        ctx_out = self._forward_train(ctx, sl(controls, L), sl(depth, L), capture_intermediate=True)
        preds, slots = [], []
        cur = ctx[:, -1:]
        for t in range(tgt.shape[1]):
            inp = tgt[:, t:t + 1] if torch.rand(1).item() > ratio else cur
            seq = torch.cat([ctx, inp], 1)
            o = self._forward_train(seq, sl(controls, seq.shape[1]), sl(depth, seq.shape[1]))
            cur = o["predictions"][:, -1:]
            preds.append(cur)
            if "cjepa_slots" in o:
                slots.append(o["cjepa_slots"])
        res = {"predictions": torch.cat(preds, 1) if preds else ctx[:, :0], "targets": tgt,
               "self_forcing_ratio": ratio, "context_length": L, "hidden_states": ctx_out["hidden_states"]}
        if slots:
            res["cjepa_slots"] = torch.stack(slots, 1)
        return res

    def forward_with_sla(self, frames, controls=None, depth=None, **kw):
        prev = self._attention_mode
        self._attention_mode = "sla"
        try:
            out = self._forward_train(frames, controls, depth, **kw)
            out["attention_mode"] = "sla"
            return out
        finally:
            self._attention_mode = prev

    def forward_with_rich_conditioning(self, frames: torch.Tensor, camera_data=None, road_data=None,
                                       bbox_data=None, ego_data=None, temporal_data=None,
                                       cfg_scale: float = 1.0, **kw) -> Dict[str, torch.Tensor]:
        if self.rich_conditioning is None:
            warnings.warn("rich conditioning is not enabled; running the plain forward")
            return self._forward_train(frames, **kw)
        co = self.rich_conditioning(camera_data=camera_data, road_data=road_data, bbox_data=bbox_data,
                                    ego_data=ego_data, temporal_data=temporal_data, cfg_scale=cfg_scale,
                                    return_cross_attention_contexts=True)
        out = self._forward_train(frames, cond=co["conditioning"].to(frames.dtype), capture_intermediate=True, **kw)
        out["conditioning"] = co["conditioning"]
        out["adaln_params"] = co["adaln_params"]
        for k in ("road_context", "object_tokens"):
            if k in co:
                out[k] = co[k]
        return out

    def forward_cjepa(self, frames, controls=None, depth=None, return_all_slots: bool = False, **kw):
        if self.cjepa_predictor is None:
            raise RuntimeError("C-JEPA predictor not initialized: enable CAUSAL_JEPA")
        out = self._forward_train(frames, controls, depth, capture_intermediate=True)
        B, T = frames.shape[:2]
        fh = out["hidden_states"]
        cj = self.cjepa_predictor(fh.reshape(B, T, -1, fh.shape[-1]))
        out.update({"cjepa_slots": cj["slots"], "cjepa_predictions": cj["predicted_slots"],
                    "cjepa_outputs": cj})
        return out

    def _decode_frame_tokens(self, frame_tokens: torch.Tensor, B: int, T: int) -> torch.Tensor:
        """Per-patch latents -> frames in [0, 1]: bilinear upsampling of the latent grid, the
        latent channels summed into each of the 3 colour channels, sigmoid."""
        n = self.config.image_size // self.config.patch_size
        C = self.config.vae_latent_dim
        x = frame_tokens.reshape(B, T, n, n, C).permute(0, 1, 4, 2, 3).reshape(B * T, C, n, n)
        x = F.interpolate(x, size=(self.config.image_size,) * 2, mode="bilinear", align_corners=False)
        if C != 3:
            x = x.sum(1, keepdim=True).expand(-1, 3, -1, -1)
        return torch.sigmoid(x).reshape(B, T, 3, self.config.image_size, self.config.image_size)

    # ------------------------------------------------------------------ misc
    def reset_cache(self) -> None:
        self.past_kvs = None
        self._intermediate_features = {}

    def update_self_forcing_step(self, step: int) -> None:
        self.self_forcing_scheduler.update(step)

    def get_num_parameters(self, trainable_only: bool = False) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad or not trainable_only)

    def get_moe_aux_loss(self) -> Optional[torch.Tensor]:
        if not self.use_moe:
            return None
        losses = [b.get_aux_loss() for b in self.backbone if b.get_aux_loss() is not None]
        return sum(losses) / len(losses) if losses else None


def create_world_model(config: DriveDiTConfig) -> WorldModel:
    return WorldModel(config)
