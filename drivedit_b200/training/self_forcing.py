"""Self-Forcing++ training of the causal world model.

API of the reference ``training/self_forcing_plus.py``: ``RollingKVCache`` (:29-145),
``SelfForcingPlusConfig`` (:153-197), ``CurriculumScheduler`` (smooth-step sequence
length, self-forcing ratio schedules, staged loss weights, :204-303),
``FutureAnchorEncoder`` (:310-403), ``ExtendedControlEncoder`` (6-D control
normalisation, encoder, inverse-dynamics head, :410-598), ``ControlConditioner`` (FiLM,
:601-653), ``EMAModel`` (:660-731), ``UncertaintyWeighting`` (Kendall et al., :734-812),
``PerLayerGradientClipper`` (pattern / adaptive thresholds, :815-944) and
``SelfForcingPlusTrainer`` (:947-1264) with ``get_default_config`` /
``get_minimal_config``.

Where the reference's rollout is a placeholder (the "model output" is its input frame,
:1178-1181), this trainer calls the world model:

1. context: the first ``context_frames`` frames are ground truth; each later chunk of
   ``chunk_frames`` frames is, with probability ``sf_ratio``, replaced by the model's own
   rollout (no grad; KV-cached, ``flow_steps`` Euler steps, exactly the inference
   path) conditioned on the mixed history;
2. loss: one training forward over ``[mixed clean context (t = 1), noisy ground-truth
   chunk (t ~ logit-normal)]`` with frame-causal attention, so the chunk sees its history
   the way it does at inference (clean keys/values); losses on the chunk: flow matching
   (velocity MSE), reconstruction (one-step clean estimate), temporal (frame-difference
   consistency) and control (inverse dynamics from consecutive frame states);
3. curriculum weights -> uncertainty weighting -> backward -> per-layer clipping -> AdamW
   -> EMA.

Host synchronisation is avoided in the step: gradient norms, clip coefficients, adaptive
thresholds, uncertainty weights and the EMA live on the device; the returned statistics
are device tensors (``float()`` them when logging).
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .flow_matching import interpolate, sample_t


# ----------------------------------------------------------------------------- KV cache
class RollingKVCache:
    """Per-layer K/V history with truncation (keep the newest ``truncate_to`` entries
    once ``max_length`` is exceeded) and periodic gradient detachment."""

    def __init__(self, max_length: int = 512, truncate_to: int = 256, detach_interval: int = 8,
                 num_layers: int = 12, device=None):
        self.max_length, self.truncate_to = max_length, truncate_to
        self.detach_interval, self.num_layers = detach_interval, num_layers
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.cache: Dict[int, Dict[str, torch.Tensor]] = {}
        self.step_count = 0
        self.total_length = 0

    def reset(self):
        self.cache = {}
        self.step_count = 0
        self.total_length = 0

    def update(self, layer_idx: int, new_k: torch.Tensor, new_v: torch.Tensor):
        """``new_k/new_v [B, T_new, H, D]`` -> full (cached + new) K, V."""
        self.step_count += 1
        det = self.step_count % self.detach_interval == 0
        if layer_idx not in self.cache:
            k, v = (new_k.detach(), new_v.detach()) if det else (new_k, new_v)
        else:
            ck, cv = self.cache[layer_idx]["k"], self.cache[layer_idx]["v"]
            if det:
                ck, cv, new_k, new_v = ck.detach(), cv.detach(), new_k.detach(), new_v.detach()
            k, v = torch.cat([ck, new_k], 1), torch.cat([cv, new_v], 1)
            if k.shape[1] > self.max_length:
                cut = k.shape[1] - self.truncate_to
                k, v = k[:, cut:].detach(), v[:, cut:].detach()
        self.cache[layer_idx] = {"k": k, "v": v}
        self.total_length = k.shape[1]
        return k, v

    def get_cache(self, layer_idx: int) -> Optional[Dict[str, torch.Tensor]]:
        return self.cache.get(layer_idx)

    def get_length(self) -> int:
        return self.total_length

    def get_memory_usage(self) -> float:
        return sum(t.element_size() * t.numel() for c in self.cache.values()
                   for t in c.values()) / 1024 ** 3


# ----------------------------------------------------------------------------- config + curriculum
@dataclass
class SelfForcingPlusConfig:
    model_dim: int = 512
    num_heads: int = 8
    num_layers: int = 12
    initial_sequence_length: int = 8
    final_sequence_length: int = 64
    max_sequence_length: int = 128
    context_frames: int = 4
    kv_cache_max_length: int = 512
    kv_cache_truncate_to: int = 256
    kv_cache_detach_interval: int = 8
    curriculum_warmup_steps: int = 10000
    sequence_curriculum_steps: int = 20000
    initial_self_forcing_ratio: float = 0.0
    final_self_forcing_ratio: float = 1.0
    self_forcing_warmup_steps: int = 15000
    self_forcing_schedule: str = "cosine"
    enable_future_anchors: bool = True
    future_anchor_horizons: List[float] = field(default_factory=lambda: [2.0, 4.0, 6.0])
    future_anchor_dim: int = 64
    fps: float = 10.0
    control_dim: int = 6
    control_hidden_dim: int = 256
    batch_size: int = 8
    learning_rate: float = 1e-4
    weight_decay: float = 0.01
    mixed_precision: bool = True
    max_memory_gb: float = 16.0
    # rollout used to self-generate context chunks
    chunk_frames: int = 4
    flow_steps: int = 4
    window_frames: int = 32
    grad_clip: float = 1.0
    ema_decay: float = 0.9999


class CurriculumScheduler:
    def __init__(self, config: SelfForcingPlusConfig):
        self.config = config
        self.current_step = 0

    def update(self, step: int):
        self.current_step = step

    @staticmethod
    def _smooth_step(x: float) -> float:
        x = max(0.0, min(1.0, x))
        return x * x * (3 - 2 * x)

    def get_sequence_length(self) -> int:
        c = self.config
        if self.current_step >= c.sequence_curriculum_steps:
            return c.final_sequence_length
        p = self._smooth_step(self.current_step / c.sequence_curriculum_steps)
        n = int(c.initial_sequence_length + p * (c.final_sequence_length - c.initial_sequence_length))
        return max(c.initial_sequence_length, min(n, c.final_sequence_length))

    def get_self_forcing_ratio(self) -> float:
        c = self.config
        if self.current_step >= c.self_forcing_warmup_steps:
            return c.final_self_forcing_ratio
        p = self.current_step / c.self_forcing_warmup_steps
        if c.self_forcing_schedule == "cosine":
            r = 0.5 * (1 - math.cos(math.pi * p))
        elif c.self_forcing_schedule == "exponential":
            r = 1 - math.exp(-3 * p)
        else:
            r = p
        return c.initial_self_forcing_ratio + r * (c.final_self_forcing_ratio - c.initial_self_forcing_ratio)

    def get_curriculum_weights(self) -> Dict[str, float]:
        p = min(1.0, self.current_step / self.config.curriculum_warmup_steps)
        return {"reconstruction": 1.0, "temporal_consistency": p, "temporal": p,
                "flow_matching": max(0.1, p),
                "future_anchor": (p - 0.3) / 0.7 if p > 0.3 else 0.0,
                "control_prediction": p, "control": p, "kv_regularization": 0.01}

    def get_stats(self) -> Dict[str, Any]:
        return {"step": self.current_step, "sequence_length": self.get_sequence_length(),
                "self_forcing_ratio": self.get_self_forcing_ratio(),
                "curriculum_weights": self.get_curriculum_weights()}


# ----------------------------------------------------------------------------- conditioning encoders
class FutureAnchorEncoder(nn.Module):
    """Goal states at several horizons (seconds) relative to the current state
    ``[x, y, heading, speed, heading_rate]`` -> one ``[B, model_dim]`` embedding."""

    def __init__(self, config: SelfForcingPlusConfig):
        super().__init__()
        self.config = config
        self.horizons = list(config.future_anchor_horizons)
        self.anchor_dim = config.future_anchor_dim
        self.anchor_input_dim = 5
        self.horizon_encoders = nn.ModuleList([
            nn.Sequential(nn.Linear(5, self.anchor_dim), nn.SiLU(),
                          nn.Linear(self.anchor_dim, self.anchor_dim), nn.LayerNorm(self.anchor_dim))
            for _ in self.horizons])
        self.fusion = nn.Sequential(nn.Linear(len(self.horizons) * self.anchor_dim, config.model_dim),
                                    nn.SiLU(), nn.Linear(config.model_dim, config.model_dim),
                                    nn.LayerNorm(config.model_dim))

    def get_anchor_indices(self, current_time: int, max_time: int) -> List[int]:
        return [min(current_time + int(h * self.config.fps), max_time - 1) for h in self.horizons]

    def forward(self, future_states: torch.Tensor, current_time: int = 0) -> torch.Tensor:
        B, T, _ = future_states.shape
        cur = future_states[:, min(current_time, T - 1)]
        feats = [enc(future_states[:, idx] - cur) for enc, idx in
                 zip(self.horizon_encoders, self.get_anchor_indices(current_time, T))]
        return self.fusion(torch.cat(feats, -1))


class ExtendedControlEncoder(nn.Module):
    DEFAULT_RANGES = {"steering": (-1.0, 1.0), "acceleration": (-5.0, 5.0), "goal_x": (-50.0, 50.0),
                      "goal_y": (-50.0, 50.0), "speed": (0.0, 40.0), "heading_rate": (-1.0, 1.0)}
    KEYS = ("steering", "acceleration", "goal_x", "goal_y", "speed", "heading_rate")

    def __init__(self, config: SelfForcingPlusConfig, custom_ranges: Optional[Dict[str, Tuple[float, float]]] = None):
        super().__init__()
        self.config = config
        self.control_dim, self.hidden_dim, self.model_dim = config.control_dim, config.control_hidden_dim, config.model_dim
        self.ranges = {**self.DEFAULT_RANGES, **(custom_ranges or {})}
        self.register_buffer("norm_min", torch.tensor([self.ranges[k][0] for k in self.KEYS]))
        self.register_buffer("norm_max", torch.tensor([self.ranges[k][1] for k in self.KEYS]))
        h, d = self.hidden_dim, self.model_dim
        self.encoder = nn.Sequential(nn.Linear(self.control_dim, h), nn.SiLU(), nn.Linear(h, h), nn.SiLU(),
                                     nn.Linear(h, d), nn.LayerNorm(d))
        self.temporal_encoder = nn.Sequential(nn.Linear(d, d), nn.SiLU(), nn.Linear(d, d))
        self.control_predictor = nn.Sequential(nn.Linear(2 * d, h), nn.SiLU(), nn.Linear(h, h), nn.SiLU(),
                                               nn.Linear(h, self.control_dim))

    def normalize(self, controls: torch.Tensor) -> torch.Tensor:
        lo, hi = self.norm_min.to(controls.dtype), self.norm_max.to(controls.dtype)
        c = torch.maximum(torch.minimum(controls, hi), lo)
        return 2 * (c - lo) / (hi - lo + 1e-8) - 1

    def denormalize(self, normalized: torch.Tensor) -> torch.Tensor:
        lo, hi = self.norm_min.to(normalized.dtype), self.norm_max.to(normalized.dtype)
        return (normalized + 1) / 2 * (hi - lo) + lo

    def forward(self, controls: torch.Tensor, normalize: bool = True) -> torch.Tensor:
        if normalize:
            controls = self.normalize(controls)
        e = self.encoder(controls)
        return e + self.temporal_encoder(e) if controls.dim() == 3 else e

    def predict_control(self, current_state: torch.Tensor, next_state: torch.Tensor) -> torch.Tensor:
        return self.control_predictor(torch.cat([current_state, next_state], -1)).clamp(-1, 1)

    def get_control_loss(self, predicted, target, normalize_target: bool = True):
        if normalize_target:
            target = self.normalize(target)
        return (predicted - target).pow(2).mean()


class ControlConditioner(nn.Module):
    """FiLM: ``gamma(c) * hidden + beta(c)``."""

    def __init__(self, config: SelfForcingPlusConfig):
        super().__init__()
        d = config.model_dim
        self.config = config
        self.gamma_net = nn.Sequential(nn.Linear(d, d), nn.SiLU(), nn.Linear(d, d))
        self.beta_net = nn.Sequential(nn.Linear(d, d), nn.SiLU(), nn.Linear(d, d))

    def forward(self, hidden: torch.Tensor, control_embedding: torch.Tensor) -> torch.Tensor:
        if control_embedding.dim() == 2 and hidden.dim() == 3:
            control_embedding = control_embedding[:, None].expand(-1, hidden.shape[1], -1)
        return self.gamma_net(control_embedding) * hidden + self.beta_net(control_embedding)


# ----------------------------------------------------------------------------- stability tools
class EMAModel:
    """Exponential moving average of the trainable parameters. With ``group`` (a
    :class:`~drivedit_b200.parallel.flat.FlatParamGroup`) the shadow is one flat fp32
    buffer updated by a single lerp per step; otherwise one tensor per name."""

    def __init__(self, model: nn.Module, decay: float = 0.9999, device=None, group=None):
        self.decay = decay
        self.device = device
        self.group = group
        self.backup: Dict[str, torch.Tensor] = {}
        if group is not None:
            self.flat = group.master.detach().clone()
            self.shadow = {n: self.flat[o:o + k].view_as(p) for n, p, (o, k) in
                           zip(group.names, group.params, (group.offsets[n] for n in group.names))}
        else:
            self.flat = None
            self.shadow = {n: p.detach().clone().to(device) if device else p.detach().clone()
                           for n, p in model.named_parameters() if p.requires_grad}

    @torch.no_grad()
    def update(self, model: nn.Module):
        if self.flat is not None:
            self.flat.lerp_(self.group.master, 1 - self.decay)
            return
        for n, p in model.named_parameters():
            if n in self.shadow:
                self.shadow[n].lerp_(p.detach().to(self.shadow[n].device), 1 - self.decay)

    @torch.no_grad()
    def apply_shadow(self, model: nn.Module):
        for n, p in model.named_parameters():
            if n in self.shadow:
                self.backup[n] = p.detach().clone()
                p.data.copy_(self.shadow[n].to(p.device))
        if self.group is not None:
            self.group.refresh_compute()

    @torch.no_grad()
    def restore(self, model: nn.Module):
        for n, p in model.named_parameters():
            if n in self.backup:
                p.data.copy_(self.backup[n])
        self.backup = {}
        if self.group is not None:
            self.group.refresh_compute()

    def state_dict(self) -> Dict[str, Any]:
        return {"shadow": {n: t.clone() for n, t in self.shadow.items()}, "decay": self.decay}

    def load_state_dict(self, state_dict: Dict[str, Any]):
        for n, t in state_dict["shadow"].items():
            if n in self.shadow:
                self.shadow[n].copy_(t)
            else:
                self.shadow[n] = t.clone()
        self.decay = state_dict.get("decay", self.decay)


class UncertaintyWeighting(nn.Module):
    """Homoscedastic-uncertainty task weighting (Kendall, Gal & Cipolla, CVPR 2018).

    Each task i has a learnable ``s_i = log sigma_i^2``. For regression-type losses the
    Gaussian likelihood gives ``L = sum_i L_i / (2 sigma_i^2) + log sigma_i
    = sum_i 0.5 (exp(-s_i) L_i + s_i)``: a noisier task gets less weight, and the
    ``s_i`` term stops every sigma from growing without bound. The losses present in a
    call are stacked and weighted in one vector expression; absent ones contribute
    nothing (their ``s_i`` receive no gradient)."""

    def __init__(self, loss_names: List[str], initial_log_var: float = 0.0):
        super().__init__()
        self.loss_names = list(loss_names)
        self.num_losses = len(self.loss_names)
        self._index = {n: i for i, n in enumerate(self.loss_names)}
        self.log_vars = nn.Parameter(torch.full((self.num_losses,), float(initial_log_var)))

    def forward(self, losses: Dict[str, torch.Tensor]):
        names = [n for n in self.loss_names if n in losses]
        if not names:
            return torch.zeros((), device=self.log_vars.device), {}
        idx = torch.tensor([self._index[n] for n in names], device=self.log_vars.device)
        s = self.log_vars.index_select(0, idx)
        vals = torch.stack([losses[n].reshape(()).to(s.dtype) for n in names])
        precision = torch.exp(-s)
        total = 0.5 * (precision * vals + s).sum()
        return total, dict(zip(names, precision.detach().unbind(0)))

    def get_weights(self) -> Dict[str, float]:
        """Current precision ``exp(-s_i)`` per task."""
        return dict(zip(self.loss_names, self.log_vars.detach().neg().exp().tolist()))

    def get_uncertainties(self) -> Dict[str, float]:
        """Current ``sigma_i = exp(s_i / 2)`` per task."""
        return dict(zip(self.loss_names, self.log_vars.detach().mul(0.5).exp().tolist()))


class PerLayerGradientClipper:
    """Per-parameter gradient-norm clipping with name-pattern thresholds and optional
    adaptive thresholds (EMA of the 95th percentile of the last 100 norms). All norms,
    thresholds and coefficients stay on the device (two foreach kernels per call)."""

    def __init__(self, model: nn.Module, default_max_norm: float = 1.0,
                 layer_configs: Optional[Dict[str, float]] = None, adaptive: bool = False,
                 adaptive_factor: float = 0.99, history: int = 100):
        self.model = model
        self.default_max_norm = default_max_norm
        self.layer_configs = layer_configs or {}
        self.adaptive, self.adaptive_factor = adaptive, adaptive_factor
        self.names = [n for n, p in model.named_parameters() if p.requires_grad]
        self.params = [p for _, p in model.named_parameters() if p.requires_grad]
        self.layer_max_norms = self._compute_layer_norms()
        dev = self.params[0].device if self.params else torch.device("cpu")
        self._max = torch.tensor([self.layer_max_norms[n] for n in self.names], device=dev)
        self._hist = torch.zeros(history, len(self.names), device=dev)
        self._hcount = 0
        self._thresh = self._max.clone()
        self._last: Optional[torch.Tensor] = None

    def _compute_layer_norms(self) -> Dict[str, float]:
        out = {}
        for n in self.names:
            m = self.default_max_norm
            for pat, v in self.layer_configs.items():
                if pat in n:
                    m = v
                    break
            out[n] = m
        return out

    @torch.no_grad()
    def clip_gradients(self) -> Dict[str, torch.Tensor]:
        idx = [i for i, p in enumerate(self.params) if p.grad is not None]
        if not idx:
            return {}
        grads = [self.params[i].grad for i in idx]
        norms = torch.stack(torch._foreach_norm(grads)).float()
        sel = torch.tensor(idx, device=norms.device)
        full = torch.zeros(len(self.params), device=norms.device)
        full[sel] = norms
        self._last = full
        limit = (self._thresh if self.adaptive else self._max)[sel]
        coef = torch.clamp(limit / (norms + 1e-8), max=1.0)
        torch._foreach_mul_(grads, [c for c in coef.to(grads[0].dtype).unbind()])
        if self.adaptive:
            self._hist[self._hcount % self._hist.shape[0]] = full
            self._hcount += 1
            n = min(self._hcount, self._hist.shape[0])
            if n >= 10:
                srt = self._hist[:n].sort(0).values
                p95 = srt[int(0.95 * n)]
                self._thresh = self.adaptive_factor * self._thresh + (1 - self.adaptive_factor) * p95
        return {self.names[i]: norms[j] for j, i in enumerate(idx)}

    @torch.no_grad()
    def get_total_grad_norm(self) -> torch.Tensor:
        grads = [p.grad for p in self.params if p.grad is not None]
        if not grads:
            return torch.zeros(())
        return torch.stack(torch._foreach_norm(grads)).float().norm()

    def get_gradient_stats(self) -> Dict[str, Any]:
        norms = self._last if self._last is not None else torch.zeros(len(self.names))
        vals = norms.tolist()
        return {"total_norm": float(self.get_total_grad_norm()),
                "layer_norms": dict(zip(self.names, vals)),
                "clipped_layers": [n for n, v in zip(self.names, vals) if v > self.layer_max_norms[n]]}


# ----------------------------------------------------------------------------- trainer
class SelfForcingPlusTrainer:
    """Self-Forcing++ on a :class:`~drivedit_b200.models.world_dit.WorldDiT`.

    ``batch``: ``frames [B, T, C, H, W]`` clean latents, ``controls [B, T, 6]`` raw 6-D
    controls, optional ``ego_states [B, T, 5]``. The normalised controls (first
    ``action_dim`` of them) are the model's per-frame actions; the control embedding
    (+ future-anchor embedding) is added to its per-frame conditioning."""

    LOSS_NAMES = ["reconstruction", "temporal", "flow_matching", "control", "future_anchor"]

    def __init__(self, model: nn.Module, config: SelfForcingPlusConfig, device=None,
                 lr: Optional[float] = None, seed: int = 0):
        from ..parallel.flat import FlatParamGroup
        from .optim import FlatAdamW

        self.model = model
        self.config = config
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        d = model.cfg.d_model
        if config.model_dim != d:
            config.model_dim = d
        self.kv_cache = RollingKVCache(config.kv_cache_max_length, config.kv_cache_truncate_to,
                                       config.kv_cache_detach_interval, config.num_layers, self.device)
        self.curriculum = CurriculumScheduler(config)
        self.future_anchor_encoder = FutureAnchorEncoder(config) if config.enable_future_anchors else None
        self.control_encoder = ExtendedControlEncoder(config)
        self.control_conditioner = ControlConditioner(config)
        C = model.cfg.latent_channels
        self.state_encoder = nn.Linear(C, d)  # pooled latent frame -> state for inverse dynamics
        self.uncertainty_weighter = UncertaintyWeighting(self.LOSS_NAMES)
        self.aux = nn.ModuleDict({"control_encoder": self.control_encoder,
                                  "control_conditioner": self.control_conditioner,
                                  "state_encoder": self.state_encoder,
                                  "uncertainty_weighter": self.uncertainty_weighter})
        if self.future_anchor_encoder is not None:
            self.aux["future_anchor_encoder"] = self.future_anchor_encoder
        self.model.to(self.device)
        self.aux.to(self.device)
        named = list(model.flat_layout(model.named_parameters())) + [("aux." + n, p) for n, p in self.aux.named_parameters()]
        nd = set(model.no_decay_names()) | {"aux." + n for n, p in self.aux.named_parameters()
                                            if p.dim() < 2}
        self.group = FlatParamGroup(named, self.device, no_decay=nd)
        self.opt = FlatAdamW(self.group, lr or config.learning_rate, (0.9, 0.95), 1e-8,
                             config.weight_decay, 0.0)
        if self.device.type == "cuda":
            model.enable_fused(group=self.group)
        self.ema = EMAModel(model, config.ema_decay, group=self.group)
        self.gradient_clipper = PerLayerGradientClipper(model, config.grad_clip,
                                                        {"attn": 0.5, "out_proj": 1.5}, adaptive=True)
        self.compute_dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        self.gen = torch.Generator(device=self.device).manual_seed(seed + 11)
        self.rng = random.Random(seed)
        self.global_step = 0
        self.training_stats: Dict[str, Any] = {"total_loss": [], "losses": {}, "curriculum_stats": []}

    # ------------------------------------------------------------------ pieces
    def _actions(self, ctrl_norm: torch.Tensor) -> torch.Tensor:
        A = self.model.cfg.action_dim
        if ctrl_norm.shape[-1] >= A:
            return ctrl_norm[..., :A]
        return F.pad(ctrl_norm, (0, A - ctrl_norm.shape[-1]))

    def _state(self, frames: torch.Tensor) -> torch.Tensor:
        """``[B, F, C, H, W]`` -> ``[B, F, d]`` (spatially pooled channels, projected)."""
        return self.state_encoder(frames.float().mean((-2, -1)))

    @torch.no_grad()
    def _mixed_context(self, frames, actions, extra, s0: int, sf_ratio: float):
        """Frames ``[0, s0)``: ground truth for the context and for chunks kept as GT, the
        model's own KV-cached rollout for chunks drawn with probability ``sf_ratio``."""
        cfg = self.config
        ctx = cfg.context_frames
        z = frames[:, :s0].to(self.compute_dtype)
        if sf_ratio <= 0 or s0 <= ctx:
            return z, 0
        starts = list(range(ctx, s0, cfg.chunk_frames))
        use_sg = {f: self.rng.random() < sf_ratio for f in starts}
        if not any(use_sg.values()):
            return z, 0
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        rc = RolloutConfig(total_frames=s0, chunk_frames=cfg.chunk_frames, flow_steps=cfg.flow_steps,
                           window_frames=cfg.window_frames, context_frames=ctx, batch=frames.shape[0])
        r = StreamingRollout(self.model, rc, self.compute_dtype)
        res = r.run(z[:, :ctx], actions[:, :s0], total_frames=s0, generator=self.gen,
                    extra_cond=extra[:, :s0],
                    replace=lambda f0, n: None if use_sg.get(f0, False) else z[:, f0:f0 + n])
        return res.frames[:, :s0], sum(use_sg.values())

    # ------------------------------------------------------------------ step
    def train_step(self, batch: Dict[str, torch.Tensor], optimizer=None) -> Dict[str, Any]:
        cfg = self.config
        self.model.train()
        self.group.zero_grad()
        seq = self.curriculum.get_sequence_length()
        sf_ratio = self.curriculum.get_self_forcing_ratio()
        cw = self.curriculum.get_curriculum_weights()
        frames = batch["frames"][:, :seq].to(self.device, non_blocking=True)
        controls = batch["controls"][:, :seq].to(self.device, non_blocking=True).float()
        B, T = frames.shape[:2]
        c = cfg.chunk_frames
        ctx = cfg.context_frames
        assert T >= ctx + c, "sequence shorter than context + one chunk"
        n_chunks = (T - ctx) // c
        s0 = ctx + c * self.rng.randrange(n_chunks)        # loss chunk [s0, s0 + c)
        L = s0 + c

        ctrl_norm = self.control_encoder.normalize(controls)
        actions = self._actions(ctrl_norm)
        extra = self.control_encoder(controls)              # [B, T, d]
        if self.future_anchor_encoder is not None and "ego_states" in batch:
            ego = batch["ego_states"][:, :seq].to(self.device).float()
            extra = extra + self.future_anchor_encoder(ego, current_time=s0)[:, None]

        z, n_sg = self._mixed_context(frames, actions, extra.detach(), s0, sf_ratio)
        gt = frames[:, s0:L].float()
        tf = sample_t(B, "logit_normal", self.device, self.gen)             # [B]
        noise = torch.randn(gt.shape, device=self.device, generator=self.gen)
        x_chunk = interpolate(noise, gt, tf)
        x_in = torch.cat([z.to(self.compute_dtype), x_chunk.to(self.compute_dtype)], 1)
        t_frames = torch.ones(B, L, device=self.device)
        t_frames[:, s0:] = tf[:, None]
        v = self.model(x_in, t_frames, actions[:, :L], extra_cond=extra[:, :L])
        v = v[:, s0:].float()
        losses: Dict[str, torch.Tensor] = {}
        losses["flow_matching"] = (v - (gt - noise)).pow(2).mean()
        tt = tf.view(B, 1, 1, 1, 1)
        x1_hat = x_chunk + (1 - tt) * v
        losses["reconstruction"] = (x1_hat - gt).pow(2).mean()
        prev_hat = torch.cat([z[:, s0 - 1:s0].float(), x1_hat[:, :-1]], 1)
        prev_gt = frames[:, s0 - 1:L - 1].float()
        losses["temporal"] = ((x1_hat - prev_hat) - (gt - prev_gt)).abs().mean()
        st_prev = self._state(frames[:, s0 - 1:L - 1])
        st_next = self._state(x1_hat)
        pred_ctrl = self.control_encoder.predict_control(st_prev, st_next)
        losses["control"] = (pred_ctrl - ctrl_norm[:, s0:L]).pow(2).mean()

        weighted = {k: l * cw.get(k, 1.0) for k, l in losses.items()}
        total, uw = self.uncertainty_weighter(weighted)
        total.backward()
        grad_norms = self.gradient_clipper.clip_gradients()
        if optimizer is not None:
            optimizer.step()
        else:
            self.opt.step()
        self.ema.update(self.model)
        self.global_step += 1
        self.curriculum.update(self.global_step)
        out: Dict[str, Any] = {"total_loss": total.detach(), "sf_ratio": sf_ratio, "seq_length": T,
                               "self_generated_chunks": n_sg, "loss_chunk_start": s0,
                               "grad_norm": self.gradient_clipper.get_total_grad_norm()}
        for k, l in losses.items():
            out[f"loss_{k}"] = l.detach()
        for k, w in uw.items():
            out[f"weight_{k}"] = w
        return out

    # ------------------------------------------------------------------ misc API
    def update_curriculum(self, step: int):
        self.curriculum.update(step)
        self.global_step = step

    def get_curriculum_stats(self) -> Dict[str, Any]:
        return self.curriculum.get_stats()

    def use_ema_for_eval(self) -> None:
        self.ema.apply_shadow(self.model)

    def restore_training_weights(self) -> None:
        self.ema.restore(self.model)

    def state_dict(self) -> Dict[str, Any]:
        return {"global_step": self.global_step, "curriculum_step": self.curriculum.current_step,
                "ema": self.ema.state_dict(), "uncertainty_weighter": self.uncertainty_weighter.state_dict(),
                "aux": self.aux.state_dict(), "optim": self.opt.state_dict(),
                "training_stats": self.training_stats}

    def load_state_dict(self, sd: Dict[str, Any]):
        self.global_step = sd.get("global_step", 0)
        self.curriculum.update(sd.get("curriculum_step", 0))
        if "ema" in sd:
            self.ema.load_state_dict(sd["ema"])
        if "uncertainty_weighter" in sd:
            self.uncertainty_weighter.load_state_dict(sd["uncertainty_weighter"])
        if "aux" in sd:
            self.aux.load_state_dict(sd["aux"])
        if "optim" in sd:
            self.opt.load_state_dict(sd["optim"])
        self.training_stats = sd.get("training_stats", self.training_stats)


def get_default_config() -> SelfForcingPlusConfig:
    return SelfForcingPlusConfig()


def get_minimal_config() -> SelfForcingPlusConfig:
    return SelfForcingPlusConfig(initial_sequence_length=4, final_sequence_length=16,
                                 kv_cache_max_length=128, kv_cache_truncate_to=64,
                                 curriculum_warmup_steps=1000, sequence_curriculum_steps=2000,
                                 self_forcing_warmup_steps=2000)


# first-generation self-forcing trainer (frame -> frame models), kept under the same module
from .self_forcing_v1 import SelfForcingTrainer, create_dummy_dataloader, create_simple_model  # noqa: E402,F401
