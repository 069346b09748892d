"""Unified trainer: flow matching + optional REPA (with the HASTE plateau controller),
C-JEPA object prediction, MoE monitoring, sequence-length curriculum, callbacks,
validation (incl. closed loop), checkpoint / resume and JSONL metrics.

API of the reference ``training/unified_trainer.py``: ``TrainingCallback`` /
``CallbackEvent`` / ``OnREPADisabledCallback`` / ``OnExpertImbalanceCallback``
(:43-137), ``REPAConfig`` / ``CJEPAConfig`` / ``MoEConfig`` / ``ValidationConfig`` /
``TrainingConfig`` (:144-284), ``CurriculumScheduler`` (cosine ramps, :291-329),
``HASTEController`` (windowed loss-plateau early stop, :332-420), ``REPAProjector``
(BatchNorm MLP, :427-471), ``REPABackbone`` (:474-522), ``SlotAttention`` /
``CJEPAPredictor`` (:529-704), ``MoEMonitor`` (usage, balance E*sum frac^2, router
z-loss, imbalance callbacks, :711-859), ``UnifiedTrainer`` (:866-1823: train_step,
train_epoch, losses, checkpoints, evaluate) and the factories (:1830-1902).

The reference's trainer cannot be constructed (it calls a method its own config class
lacks); this one runs the framework's ``WorldDiT`` (fused kernels on CUDA): the flow
matching step is the same as :class:`~drivedit_b200.training.trainer.WorldModelTrainer`
and the optional objectives hang off the same forward (layer features for REPA and
C-JEPA, per-layer expert counts for the MoE monitor). Per-step statistics stay on the
device; the host reads them every ``log_every`` steps.
"""
from __future__ import annotations

import logging
import math
import time
from dataclasses import asdict, dataclass, field
from enum import Enum
from typing import Any, Callable, Dict, Iterable, List, Optional, Protocol

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..models.causal_jepa import SlotAttention as _SlotAttention
from .flow_matching import interpolate, sample_t

log = logging.getLogger(__name__)


# ----------------------------------------------------------------------------- callbacks
class TrainingCallback(Protocol):
    def on_train_step_end(self, trainer: "UnifiedTrainer", step: int, losses: Dict[str, float],
                          metrics: Dict[str, Any]) -> None: ...

    def on_epoch_end(self, trainer: "UnifiedTrainer", epoch: int, metrics: Dict[str, Any]) -> None: ...


class CallbackEvent(Enum):
    REPA_DISABLED = "repa_disabled"
    EXPERT_IMBALANCE = "expert_imbalance"
    CURRICULUM_MILESTONE = "curriculum_milestone"
    VALIDATION_IMPROVEMENT = "validation_improvement"


@dataclass
class OnREPADisabledCallback:
    on_disabled: Optional[Callable[[int, float, float], None]] = None

    def __call__(self, step: int, final_loss: float, threshold: float) -> None:
        if self.on_disabled is not None:
            self.on_disabled(step, final_loss, threshold)
        log.info("REPA disabled at step %d: loss=%.6f threshold=%.6f", step, final_loss, threshold)


@dataclass
class OnExpertImbalanceCallback:
    imbalance_threshold: float = 0.3
    on_imbalance: Optional[Callable[[int, Dict[str, float]], None]] = None

    def __call__(self, step: int, expert_loads: Dict[str, float]) -> bool:
        if not expert_loads:
            return False
        loads = list(expert_loads.values())
        if max(loads) - min(loads) > self.imbalance_threshold:
            if self.on_imbalance is not None:
                self.on_imbalance(step, expert_loads)
            log.warning("expert imbalance at step %d: max=%.3f min=%.3f", step, max(loads), min(loads))
            return True
        return False


# ----------------------------------------------------------------------------- configs
@dataclass
class REPAConfig:
    enabled: bool = False
    backbone_type: str = "vjepa_2.1"
    alignment_dim: int = 768
    loss_weight: float = 0.5
    temperature: float = 0.07
    projection_hidden_dim: int = 2048
    projection_output_dim: int = 256
    haste_enabled: bool = True
    haste_warmup_steps: int = 5000
    haste_window_size: int = 1000
    haste_threshold: float = 0.01
    haste_patience: int = 3
    feature_layer: int = 2


@dataclass
class CJEPAConfig:
    enabled: bool = False
    num_object_queries: int = 64
    object_dim: int = 256
    loss_weight: float = 0.3
    contrastive_temperature: float = 0.1
    prediction_horizon: int = 4
    use_slot_attention: bool = True
    slot_attention_iters: int = 3
    mask_ratio: float = 0.75
    mask_strategy: str = "object"
    feature_layer: int = 2


@dataclass
class MoEConfig:
    enabled: bool = False
    num_experts: int = 8
    top_k: int = 2
    load_balance_weight: float = 0.01
    router_z_loss_weight: float = 0.001
    capacity_factor: float = 1.25
    log_expert_utilization: bool = True
    utilization_log_frequency: int = 100
    use_auxiliary_loss: bool = True
    use_entropy_regularization: bool = True


@dataclass
class ValidationConfig:
    enabled: bool = True
    frequency: int = 1000
    num_batches: int = 10
    closed_loop_enabled: bool = False
    closed_loop_horizon: int = 30
    compute_physics_metrics: bool = False
    compute_driving_metrics: bool = False


@dataclass
class TrainingConfig:
    batch_size: int = 8
    learning_rate: float = 1e-4
    weight_decay: float = 0.01
    max_steps: int = 100000
    warmup_steps: int = 1000
    enable_curriculum: bool = True
    initial_sequence_length: int = 4
    final_sequence_length: int = 32
    curriculum_warmup_steps: int = 10000
    initial_self_forcing_ratio: float = 0.0
    final_self_forcing_ratio: float = 0.8
    self_forcing_warmup_steps: int = 5000
    enable_flow_matching: bool = True
    flow_matching_weight: float = 1.0
    num_flow_steps: int = 4
    gradient_clip_norm: float = 1.0
    mixed_precision: bool = True
    checkpoint_every: int = 1000
    distributed: bool = False
    local_rank: int = 0
    world_size: int = 1
    max_memory_gb: float = 16.0
    memory_cleanup_threshold: float = 0.8
    repa: REPAConfig = field(default_factory=REPAConfig)
    cjepa: CJEPAConfig = field(default_factory=CJEPAConfig)
    moe: MoEConfig = field(default_factory=MoEConfig)
    validation: ValidationConfig = field(default_factory=ValidationConfig)
    loss_weights: Dict[str, float] = field(default_factory=lambda: {
        "reconstruction": 1.0, "flow_matching": 1.0, "temporal_consistency": 0.2, "jepa": 0.1,
        "repa": 0.5, "cjepa": 0.3, "moe_balance": 0.01})
    # this framework's additions, after the reference's fields
    # (training/unified_trainer.py TrainingConfig) so positional construction matches
    checkpoint_dir: Optional[str] = None
    log_dir: Optional[str] = None
    log_every: int = 100
    seed: int = 0

    def is_component_enabled(self, name: str) -> bool:
        sub = getattr(self, name, None)
        return bool(getattr(sub, "enabled", False))


# ----------------------------------------------------------------------------- schedulers
class CurriculumScheduler:
    def __init__(self, config: TrainingConfig):
        self.config, self.step = config, 0

    def update(self, step: int) -> None:
        self.step = step

    @staticmethod
    def _smooth_schedule(p: float) -> float:
        return 0.5 * (1 - math.cos(math.pi * p))

    def get_sequence_length(self) -> int:
        c = self.config
        if not c.enable_curriculum:
            return c.final_sequence_length
        p = self._smooth_schedule(min(1.0, self.step / c.curriculum_warmup_steps))
        return int(c.initial_sequence_length + p * (c.final_sequence_length - c.initial_sequence_length))

    def get_self_forcing_ratio(self) -> float:
        c = self.config
        p = self._smooth_schedule(min(1.0, self.step / c.self_forcing_warmup_steps))
        return c.initial_self_forcing_ratio + p * (c.final_self_forcing_ratio - c.initial_self_forcing_ratio)


class HASTEController:
    """Disables REPA once its windowed mean loss stops changing by more than
    ``haste_threshold`` over ``haste_patience`` consecutive windows."""

    def __init__(self, config: REPAConfig):
        self.config = config
        self.loss_history: List[float] = []
        self.is_active = config.enabled and config.haste_enabled
        self.repa_disabled = False
        self.disable_step: Optional[int] = None
        self.callbacks: List[OnREPADisabledCallback] = []

    def add_callback(self, cb: OnREPADisabledCallback) -> None:
        self.callbacks.append(cb)

    def update(self, step: int, repa_loss: float) -> bool:
        if not self.is_active or self.repa_disabled:
            return not self.repa_disabled
        if step < self.config.haste_warmup_steps:
            return True
        w, pat = self.config.haste_window_size, self.config.haste_patience
        self.loss_history.append(float(repa_loss))
        self.loss_history = self.loss_history[-w * (pat + 1):]
        if len(self.loss_history) >= w * 2 and self._check_plateau():
            self.repa_disabled, self.disable_step = True, step
            final = sum(self.loss_history[-w:]) / w
            for cb in self.callbacks:
                cb(step, final, self.config.haste_threshold)
            return False
        return True

    def _check_plateau(self) -> bool:
        w, pat, thr = self.config.haste_window_size, self.config.haste_patience, self.config.haste_threshold
        if len(self.loss_history) < w * (pat + 1):
            return False
        h = self.loss_history
        means = [sum(h[len(h) - (i + 1) * w: len(h) - i * w]) / w for i in range(pat + 1)]
        return all(abs(means[i + 1] - means[i]) <= thr for i in range(pat))

    def should_compute_repa(self) -> bool:
        return self.config.enabled and not self.repa_disabled


# ----------------------------------------------------------------------------- heads
class REPAProjector(nn.Module):
    def __init__(self, input_dim: int, hidden_dim: int = 2048, output_dim: int = 256):
        super().__init__()
        self.projector = nn.Sequential(nn.Linear(input_dim, hidden_dim), nn.BatchNorm1d(hidden_dim), nn.ReLU(),
                                       nn.Linear(hidden_dim, hidden_dim), nn.BatchNorm1d(hidden_dim), nn.ReLU(),
                                       nn.Linear(hidden_dim, output_dim))

    def forward(self, x):
        shp = x.shape
        y = self.projector(x.reshape(-1, shp[-1]).float())
        return y.view(*shp[:-1], -1)


class REPABackbone(nn.Module):
    """Frozen image encoder for REPA targets: the framework's ViT teacher when
    ``backbone_type`` names a V-JEPA / ViT, else a small frozen conv encoder."""

    def __init__(self, config: REPAConfig, image_hw=(64, 64), patch: int = 16):
        super().__init__()
        self.config = config
        if "vjepa" in config.backbone_type or "vit" in config.backbone_type:
            from ..models.vjepa import VJEPABackbone, VJEPAConfig

            heads = max(1, config.alignment_dim // 64)
            self.vit = VJEPABackbone(VJEPAConfig(embed_dim=config.alignment_dim, num_layers=2, num_heads=heads,
                                                 patch_size=patch, tubelet_size=1, num_frames=1,
                                                 image_size=tuple(image_hw), extract_layers=[1]))
            self.encoder = None
        else:
            self.vit = None
            self.encoder = nn.Sequential(nn.Conv2d(3, 64, 7, 2, 3), nn.BatchNorm2d(64), nn.ReLU(),
                                         nn.Conv2d(64, 128, 3, 2, 1), nn.BatchNorm2d(128), nn.ReLU(),
                                         nn.Conv2d(128, config.alignment_dim, 3, 2, 1), nn.AdaptiveAvgPool2d(1),
                                         nn.Flatten())
            for p in self.encoder.parameters():
                p.requires_grad = False

    @torch.no_grad()
    def forward(self, frames: torch.Tensor) -> torch.Tensor:
        """``[B, T, 3, H, W]`` in [0, 1] -> per-frame features ``[B, T, D]``."""
        B, T = frames.shape[:2]
        x = frames.reshape(B * T, *frames.shape[2:])
        if self.vit is not None:
            f = self.vit(x[:, :, None], max_layer=1)["intermediate"]["layer_1"].float().mean(1)
        else:
            self.encoder.eval()
            f = self.encoder(x.float())
        return f.view(B, T, -1)


class SlotAttention(_SlotAttention):
    """Slot attention over token features (shared with the C-JEPA model)."""


class CJEPAPredictor(nn.Module):
    """Object-slot prediction on the DiT's hidden states: slots of the context frames
    predict the slots of the next ``prediction_horizon`` frames; InfoNCE between
    predicted and actual (stop-gradient) slots."""

    def __init__(self, config: CJEPAConfig, model_dim: int):
        input_dim = model_dim
        super().__init__()
        self.config = config
        self.slots = SlotAttention(config.num_object_queries, config.object_dim, input_dim,
                                   config.slot_attention_iters, 2 * config.object_dim)
        self.predictor = nn.GRU(config.object_dim, config.object_dim, batch_first=True)
        self.head = nn.Linear(config.object_dim, config.object_dim)

    def forward(self, hidden: torch.Tensor, frames: int) -> Dict[str, torch.Tensor]:
        B, T, D = hidden.shape
        tpf = T // frames
        tok = hidden.float().view(B * frames, tpf, D)
        slots, _ = self.slots(tok)
        slots = slots.view(B, frames, self.config.num_object_queries, -1)
        h = min(self.config.prediction_horizon, frames - 1)
        ctx = slots[:, :frames - h].permute(0, 2, 1, 3).reshape(B * slots.shape[2], frames - h, -1)
        out, _ = self.predictor(ctx)
        pred = self.head(out[:, -1:].expand(-1, h, -1))                       # [B*K, h, S]
        tgt = slots[:, frames - h:].permute(0, 2, 1, 3).reshape(B * slots.shape[2], h, -1).detach()
        a = F.normalize(pred.reshape(-1, pred.shape[-1]), dim=-1)
        b = F.normalize(tgt.reshape(-1, tgt.shape[-1]), dim=-1)
        logits = a @ b.t() / self.config.contrastive_temperature
        loss = F.cross_entropy(logits, torch.arange(a.shape[0], device=a.device))
        return {"loss": loss, "slots": slots, "predicted": pred}


class MoEMonitor:
    def __init__(self, config: MoEConfig):
        self.config = config
        self.expert_counts: Dict[str, List[torch.Tensor]] = {}
        self.callbacks: List[OnExpertImbalanceCallback] = []

    def add_callback(self, cb: OnExpertImbalanceCallback) -> None:
        self.callbacks.append(cb)

    def update(self, router_logits: torch.Tensor, layer_name: str = "default") -> Dict[str, torch.Tensor]:
        if not self.config.enabled:
            return {}
        E = router_logits.shape[-1]
        idx = router_logits.float().topk(self.config.top_k, -1).indices.reshape(-1)
        usage = torch.bincount(idx, minlength=E).float() / max(router_logits[..., 0].numel(), 1)
        return self.record_usage(usage, layer_name)

    def record_usage(self, usage: torch.Tensor, layer_name: str) -> Dict[str, torch.Tensor]:
        h = self.expert_counts.setdefault(layer_name, [])
        h.append(usage.detach())
        del h[:-100]
        return {f"{layer_name}_expert_usage_std": usage.std(), f"{layer_name}_expert_usage_max": usage.max(),
                f"{layer_name}_expert_usage_min": usage.min()}

    def compute_load_balance_loss(self, router_logits: torch.Tensor) -> torch.Tensor:
        if not self.config.use_auxiliary_loss:
            return router_logits.new_zeros(())
        frac = F.softmax(router_logits.float(), -1).reshape(-1, router_logits.shape[-1]).mean(0)
        return self.config.num_experts * (frac * frac).sum() * self.config.load_balance_weight

    def compute_router_z_loss(self, router_logits: torch.Tensor) -> torch.Tensor:
        return torch.logsumexp(router_logits.float(), -1).pow(2).mean() * self.config.router_z_loss_weight

    def get_expert_utilization(self) -> Dict[str, float]:
        out = {}
        for name, h in self.expert_counts.items():
            if h:
                avg = torch.stack(h[-10:]).mean(0).tolist()
                out.update({f"{name}_expert_{i}": v for i, v in enumerate(avg)})
        return out

    def check_imbalance(self, step: int) -> bool:
        util = self.get_expert_utilization()
        return any(cb(step, util) for cb in self.callbacks)


# ----------------------------------------------------------------------------- trainer
class UnifiedTrainer:
    def __init__(self, model: nn.Module, config: TrainingConfig, device=None, train_loader=None,
                 val_loader=None, callbacks: Optional[List[Any]] = None):
        from ..parallel.flat import FlatParamGroup
        from .distributed import CheckpointManager
        from .optim import FlatAdamW

        self.model, self.config = model, config
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.train_loader, self.val_loader = train_loader, val_loader
        self.callbacks = list(callbacks or [])
        self.model.to(self.device)
        d = model.cfg.d_model
        self.heads = nn.ModuleDict()
        self.repa_backbone = None
        if config.repa.enabled:
            self.heads["repa"] = REPAProjector(d, config.repa.projection_hidden_dim, config.repa.alignment_dim)
            self.repa_backbone = REPABackbone(config.repa).to(self.device)
        if config.cjepa.enabled:
            self.heads["cjepa"] = CJEPAPredictor(config.cjepa, d)
        self.heads.to(self.device)
        named = list(model.flat_layout(model.named_parameters())) + [("heads." + n, p) for n, p in self.heads.named_parameters()]
        nd = set(model.no_decay_names()) | {"heads." + n for n, p in self.heads.named_parameters() if p.dim() < 2}
        self.group = FlatParamGroup(named, self.device, no_decay=nd)
        self.optimizer = FlatAdamW(self.group, config.learning_rate, (0.9, 0.95), 1e-8, config.weight_decay,
                                   config.gradient_clip_norm)
        if self.device.type == "cuda":
            model.enable_fused(group=self.group)
        self.curriculum = CurriculumScheduler(config)
        self.haste = HASTEController(config.repa)
        self.moe_monitor = MoEMonitor(config.moe)
        for cb in self.callbacks:
            if isinstance(cb, OnREPADisabledCallback):
                self.haste.add_callback(cb)
            if isinstance(cb, OnExpertImbalanceCallback):
                self.moe_monitor.add_callback(cb)
        self.ckpt = CheckpointManager(config.checkpoint_dir) if config.checkpoint_dir else None
        self.metrics = None
        if config.log_dir:
            from ..utils.observability import MetricsLogger

            self.metrics = MetricsLogger(config.log_dir, config={"training": asdict(config)})
        self.gen = torch.Generator(device=self.device).manual_seed(config.seed + 1)
        self.global_step = 0
        self.epoch = 0
        self.best_val = float("inf")
        self._pending: List[Dict[str, torch.Tensor]] = []
        self.compute_dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32

    def _lr(self) -> float:
        c = self.config
        s = self.global_step
        if s < c.warmup_steps:
            return c.learning_rate * (s + 1) / c.warmup_steps
        p = min(1.0, (s - c.warmup_steps) / max(1, c.max_steps - c.warmup_steps))
        return c.learning_rate * 0.5 * (1 + math.cos(math.pi * p))

    # ------------------------------------------------------------------ losses
    def _forward_pass(self, batch: Dict[str, torch.Tensor]):
        c = self.config
        lat = batch["latents"].to(self.device, non_blocking=True)
        F_ = min(self.curriculum.get_sequence_length(), lat.shape[1])
        lat = lat[:, :F_]
        act = batch["actions"].to(self.device, non_blocking=True)[:, :F_]
        B = lat.shape[0]
        x0 = torch.randn(lat.shape, device=self.device, generator=self.gen)
        t = sample_t(B, "logit_normal", self.device, self.gen)
        x_t = interpolate(x0, lat.float(), t).to(self.compute_dtype)
        layer = None
        if c.repa.enabled and self.haste.should_compute_repa():
            layer = c.repa.feature_layer
        if c.cjepa.enabled:
            layer = c.cjepa.feature_layer if layer is None else layer
        if layer is not None:
            v, aux, feats = self.model(x_t, t, act, return_aux=True, return_features=layer)
            feats = feats.reshape(B, -1, feats.shape[-1])
        else:
            v, aux = self.model(x_t, t, act, return_aux=True)
            feats = None
        return {"velocity": v, "target": lat.float() - x0, "aux": aux, "features": feats, "frames": F_,
                "rgb": batch.get("rgb")}

    def _compute_losses(self, out) -> Dict[str, torch.Tensor]:
        c, w = self.config, self.config.loss_weights
        L = {"flow_matching": (out["velocity"].float() - out["target"]).pow(2).mean() * c.flow_matching_weight,
             "moe_aux": out["aux"]}
        if out["features"] is not None and "repa" in self.heads and self.haste.should_compute_repa() \
                and out["rgb"] is not None:
            from .repa import alignment_loss

            tgt = self.repa_backbone(out["rgb"].to(self.device)[:, :out["frames"]])        # [B, F, D]
            proj = self.heads["repa"](out["features"])                                      # [B, T, D]
            L["repa"] = alignment_loss(proj, tgt, "cosine") * w.get("repa", 0.5)
        if out["features"] is not None and "cjepa" in self.heads and out["frames"] > 1:
            L["cjepa"] = self.heads["cjepa"](out["features"], out["frames"])["loss"] * w.get("cjepa", 0.3)
        return L

    def _moe_usage(self) -> Dict[str, torch.Tensor]:
        stats = {}
        if not self.config.moe.enabled:
            return stats
        for i, blk in enumerate(getattr(self.model, "blocks", [])):
            moe = getattr(blk, "moe", None)
            cnt = getattr(moe, "last_counts", None) if moe is not None else None
            if cnt is not None:
                stats.update(self.moe_monitor.record_usage(cnt.float() / cnt.sum().clamp_min(1), f"layer{i}"))
        return stats

    # ------------------------------------------------------------------ steps
    def train_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        self.model.train()
        self.heads.train()
        self.group.zero_grad()
        out = self._forward_pass(batch)
        L = self._compute_losses(out)
        total = torch.stack([v.float() for v in L.values()]).sum()
        total.backward()
        self.optimizer.lr = self._lr()
        self.optimizer.step()
        self.global_step += 1
        self.curriculum.update(self.global_step)
        stats = {k: v.detach() for k, v in L.items()}
        stats["total"] = total.detach()
        stats.update(self._moe_usage())
        if "repa" in stats and self.haste.is_active:
            self._pending.append({"repa": stats["repa"]})
        if self.global_step % self.config.log_every == 0:
            self._flush(stats)
        if self.ckpt is not None and self.global_step % self.config.checkpoint_every == 0:
            self.save_checkpoint()
        return stats

    def _flush(self, stats):
        host = {k: float(v) for k, v in stats.items()}
        for rec in self._pending:
            self.haste.update(self.global_step, float(rec["repa"]))
        self._pending.clear()
        if self.config.moe.enabled:
            self.moe_monitor.check_imbalance(self.global_step)
        if self.metrics is not None:
            self.metrics.log(self.global_step, {**host, "lr": self.optimizer.lr,
                                                "seq_len": self.curriculum.get_sequence_length()})
        for cb in self.callbacks:
            if hasattr(cb, "on_train_step_end"):
                cb.on_train_step_end(self, self.global_step, host, {})

    def train_epoch(self, dataloader: Optional[Iterable] = None) -> Dict[str, float]:
        dl = dataloader or self.train_loader
        acc: Dict[str, torch.Tensor] = {}
        n = 0
        t0 = time.perf_counter()
        for batch in dl:
            s = self.train_step(batch)
            for k, v in s.items():
                acc[k] = acc.get(k, 0) + v
            n += 1
            if self.global_step >= self.config.max_steps:
                break
        self.epoch += 1
        res = {k: float(v) / max(n, 1) for k, v in acc.items()}
        res["epoch_time_s"] = time.perf_counter() - t0
        for cb in self.callbacks:
            if hasattr(cb, "on_epoch_end"):
                cb.on_epoch_end(self, self.epoch, res)
        return res

    @torch.no_grad()
    def evaluate(self, dataloader: Optional[Iterable] = None, num_batches: Optional[int] = None) -> Dict[str, float]:
        dl = dataloader or self.val_loader
        if dl is None:
            return {}
        self.model.eval()
        tot, n = 0.0, 0
        for i, batch in enumerate(dl):
            if num_batches is not None and i >= num_batches:
                break
            out = self._forward_pass(batch)
            tot += float((out["velocity"].float() - out["target"]).pow(2).mean())
            n += 1
        res = {"val_flow_matching": tot / max(n, 1)}
        if res["val_flow_matching"] < self.best_val:
            self.best_val = res["val_flow_matching"]
            res["improved"] = 1.0
        return res

    # ------------------------------------------------------------------ checkpoints
    def state_dict(self) -> Dict[str, Any]:
        return {"model": self.model.state_dict(), "heads": self.heads.state_dict(),
                "optim": self.optimizer.state_dict(), "step": self.global_step, "epoch": self.epoch,
                "haste": {"disabled": self.haste.repa_disabled, "disable_step": self.haste.disable_step},
                "best_val": self.best_val}

    def load_state_dict(self, sd: Dict[str, Any]) -> None:
        self.model.load_state_dict(sd["model"])
        self.heads.load_state_dict(sd["heads"])
        self.group.refresh_compute()
        self.optimizer.load_state_dict(sd["optim"])
        self.global_step, self.epoch = sd["step"], sd["epoch"]
        self.curriculum.update(self.global_step)
        self.haste.repa_disabled = sd["haste"]["disabled"]
        self.haste.disable_step = sd["haste"]["disable_step"]
        self.best_val = sd.get("best_val", float("inf"))

    def save_checkpoint(self, is_best: bool = False) -> Optional[str]:
        if self.ckpt is None:
            return None

        class _Wrap:
            def __init__(s, sd):
                s.sd = sd

            def state_dict(s):
                return s.sd

        sd = self.state_dict()
        return self.ckpt.save_checkpoint(_Wrap(sd), None, None, self.epoch, self.global_step, 0.0,
                                         is_best=is_best, config=asdict(self.config))

    def load_checkpoint(self, path: Optional[str] = None) -> bool:
        if self.ckpt is None:
            return False

        holder = {}

        class _Sink:
            def load_state_dict(s, sd, strict=True):
                holder["sd"] = sd

        info = self.ckpt.load_checkpoint(_Sink(), checkpoint_path=path)
        if not info:
            return False
        self.load_state_dict(holder["sd"])
        return True


def create_training_config(preset: str = "default", **overrides) -> TrainingConfig:
    cfg = TrainingConfig()
    if preset == "full":
        cfg.repa.enabled = cfg.cjepa.enabled = cfg.moe.enabled = True
    elif preset == "minimal":
        cfg.enable_curriculum = False
        cfg.validation.enabled = False
    for k, v in overrides.items():
        obj, attr = cfg, k
        if "." in k:
            head, attr = k.split(".", 1)
            obj = getattr(cfg, head)
        setattr(obj, attr, v)
    return cfg


def create_unified_trainer(model_config, training_config: Optional[TrainingConfig] = None,
                           device=None, **kw) -> UnifiedTrainer:
    """A trainer over a new :class:`~drivedit_b200.models.world_model.WorldModel` built
    from ``model_config`` (a ``DriveDiTConfig``), as the reference's factory
    (training/unified_trainer.py:1830-1851); an ``nn.Module`` as the first argument is
    trained as it is."""
    if isinstance(model_config, nn.Module):
        model = model_config
    else:
        from ..models.world_model import WorldModel

        model = WorldModel(model_config)
    return UnifiedTrainer(model, training_config or TrainingConfig(), device, **kw)
