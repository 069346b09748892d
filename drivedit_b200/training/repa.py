"""REPA representation alignment with the HASTE stage-wise schedule.

Same surface as the reference ``training/repa_loss.py``: ``REPAConfig`` (:26-59),
``ProjectionMLP`` (fc-GELU-dropout-fc-LayerNorm, :62-95), ``HASTEScheduler`` (warm-up ->
active -> terminated, :98-166), ``REPALoss`` (project DiT hidden states, pool the longer
sequence to the shorter with adaptive average pooling, normalise, cosine / mse /
smooth-l1 alignment, per-layer weights, HASTE x base x relative weight, :169-351),
``REPAIntegration`` (:354-387) and ``create_repa_loss`` (:390-417).

Differences by design: the loss history keeps detached device tensors (no per-step host
synchronisation; floats are produced on demand by ``get_loss_stats``), and on CUDA the
projection's two GEMMs and its LayerNorm run on the hand-written kernels.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class REPAConfig:
    dit_hidden_dim: int = 512
    vjepa_feature_dim: int = 1024
    projection_hidden_dim: Optional[int] = None
    dit_layers_to_align: List[int] = field(default_factory=lambda: [6, 8, 10])
    vjepa_layers_to_use: List[int] = field(default_factory=lambda: [18, 20, 22])
    enable_haste: bool = True
    haste_termination_ratio: float = 0.4
    haste_warmup_ratio: float = 0.05
    haste_schedule: str = "cosine"
    base_repa_weight: float = 1.0
    per_layer_weights: Optional[List[float]] = None
    repa_relative_weight: float = 0.1
    alignment_type: str = "cosine"
    normalize_features: bool = True
    total_training_steps: int = 100000

    def __post_init__(self):
        if self.projection_hidden_dim is None:
            self.projection_hidden_dim = (self.dit_hidden_dim + self.vjepa_feature_dim) // 2
        if self.per_layer_weights is None:
            self.per_layer_weights = [1.0] * len(self.dit_layers_to_align)


def _kernels_ok(x: torch.Tensor, *dims: int) -> bool:
    if not x.is_cuda:
        return False
    from ..ops._ext import available

    return available() and all(d % 64 == 0 for d in dims)


class ProjectionMLP(nn.Module):
    def __init__(self, input_dim: int, hidden_dim: int, output_dim: int, use_layer_norm: bool = True,
                 dropout: float = 0.1):
        super().__init__()
        self.fc1 = nn.Linear(input_dim, hidden_dim)
        self.act = nn.GELU()
        self.dropout = nn.Dropout(dropout)
        self.fc2 = nn.Linear(hidden_dim, output_dim)
        self.use_layer_norm = use_layer_norm
        if use_layer_norm:
            self.norm = nn.LayerNorm(output_dim)
        for fc in (self.fc1, self.fc2):
            nn.init.normal_(fc.weight, std=0.02)
            nn.init.zeros_(fc.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dims = (self.fc1.in_features, self.fc1.out_features, self.fc2.out_features)
        if _kernels_ok(x, *dims) and (not self.use_layer_norm or self.fc2.out_features % 256 == 0):
            from ..ops.fused import layer_norm
            from ..ops.linear import linear

            shp = x.shape
            h = x.reshape(-1, shp[-1]).to(torch.bfloat16).contiguous()
            h = linear(h, self.fc1.weight.to(torch.bfloat16), self.fc1.bias.float(),
                       self.fc1.weight, self.fc1.bias)
            h = self.dropout(F.gelu(h))
            h = linear(h.contiguous(), self.fc2.weight.to(torch.bfloat16), self.fc2.bias.float(),
                       self.fc2.weight, self.fc2.bias)
            if self.use_layer_norm:
                h = layer_norm(h, self.norm.weight, self.norm.bias, self.norm.eps)
            return h.view(*shp[:-1], -1)
        x = self.fc2(self.dropout(self.act(self.fc1(x))))
        return self.norm(x) if self.use_layer_norm else x


class HASTEScheduler:
    """REPA weight under HASTE's stage-wise termination (Wang et al. 2025, "REPA Works
    Until It Doesn't"): representation alignment helps early training and is switched
    off later. The weight ramps in over the first ``haste_warmup_ratio`` of training
    (``haste_schedule``: linear, cosine, or step = off until the ramp ends), holds at 1,
    and is 0 from ``haste_termination_ratio`` of training on. Built on the shared
    piecewise schedule; ``enable_haste=False`` keeps the weight at 1 throughout."""

    PHASES = ("warmup", "active", "terminated")

    def __init__(self, config: REPAConfig):
        from ..utils.schedules import PiecewiseSchedule, Segment

        self.config = config
        self.current_step = 0
        total = config.total_training_steps
        self.warmup_end = int(total * config.haste_warmup_ratio)
        self.termination_start = max(self.warmup_end, int(total * config.haste_termination_ratio))
        shape = config.haste_schedule if config.haste_schedule in ("linear", "cosine") else "step"
        segs = []
        if self.warmup_end > 0:
            segs.append(Segment(self.warmup_end, 0.0, 1.0, shape, "warmup"))
        if self.termination_start > self.warmup_end:
            segs.append(Segment(self.termination_start - self.warmup_end, 1.0, 1.0, "constant",
                                "active"))
        segs.append(Segment(None, 0.0, 0.0, "constant", "terminated"))
        self.schedule = PiecewiseSchedule(segs)

    def get_weight(self, step: Optional[int] = None) -> float:
        if step is not None:
            self.current_step = step
        if not self.config.enable_haste:
            return 1.0
        return self.schedule(self.current_step)

    def update(self, step: int):
        self.current_step = step

    def is_active(self) -> bool:
        return self.get_weight() > 0.0

    def get_phase(self) -> str:
        return self.schedule.phase(self.current_step)

    def get_progress_info(self) -> Dict[str, Any]:
        return {"current_step": self.current_step, "warmup_end": self.warmup_end,
                "termination_start": self.termination_start,
                "total_steps": self.config.total_training_steps,
                "current_weight": self.get_weight(), "current_phase": self.get_phase(),
                "is_active": self.is_active()}


def _pool_to(x: torch.Tensor, n: int) -> torch.Tensor:
    """Adaptive average pooling over the sequence dim ``[B, L, D] -> [B, n, D]``."""
    if x.shape[1] == n:
        return x
    L = x.shape[1]
    if L % n == 0:  # equal windows: a reshape-mean (what adaptive pooling computes here)
        return x.view(x.shape[0], n, L // n, x.shape[2]).mean(2)
    return F.adaptive_avg_pool1d(x.transpose(1, 2), n).transpose(1, 2)


def alignment_loss(dit: torch.Tensor, teacher: torch.Tensor, alignment_type: str = "cosine",
                   normalize: bool = True) -> torch.Tensor:
    n = min(dit.shape[1], teacher.shape[1])
    dit, teacher = _pool_to(dit.float(), n), _pool_to(teacher.float(), n)
    if normalize:
        dit, teacher = F.normalize(dit, dim=-1), F.normalize(teacher, dim=-1)
    if alignment_type == "cosine":
        return (1 - (dit * teacher).sum(-1)).mean()
    if alignment_type == "mse":
        return F.mse_loss(dit, teacher)
    if alignment_type == "smooth_l1":
        return F.smooth_l1_loss(dit, teacher)
    raise ValueError(f"Unknown alignment type: {alignment_type}")


class REPALoss(nn.Module):
    def __init__(self, config: REPAConfig):
        super().__init__()
        self.config = config
        self.projections = nn.ModuleDict()
        for dl, vl in zip(config.dit_layers_to_align, config.vjepa_layers_to_use):
            self.projections[f"proj_{dl}_to_{vl}"] = ProjectionMLP(
                config.dit_hidden_dim, config.projection_hidden_dim, config.vjepa_feature_dim)
        self.haste_scheduler = HASTEScheduler(config)
        self.loss_history: Dict[str, Any] = {
            "total": [], "per_layer": {f"layer_{l}": [] for l in config.dit_layers_to_align}}

    def _compute_alignment_loss(self, dit_features, vjepa_features, alignment_type="cosine"):
        return alignment_loss(dit_features, vjepa_features, alignment_type,
                              self.config.normalize_features)

    def forward(self, dit_features: Dict[str, torch.Tensor], vjepa_features: Dict[str, torch.Tensor],
                step: Optional[int] = None, return_per_layer: bool = True) -> Dict[str, Any]:
        if step is not None:
            self.haste_scheduler.update(step)
        w = self.haste_scheduler.get_weight()
        dev = next(iter(dit_features.values())).device
        if w == 0.0:
            return {"total_repa_loss": torch.zeros((), device=dev), "repa_weight": 0.0,
                    "haste_phase": self.haste_scheduler.get_phase(),
                    "per_layer_losses": {} if return_per_layer else None}
        per, total = {}, torch.zeros((), device=dev)
        for i, (dl, vl) in enumerate(zip(self.config.dit_layers_to_align, self.config.vjepa_layers_to_use)):
            dk, vk = f"layer_{dl}", f"layer_{vl}"
            if dk not in dit_features:
                warnings.warn(f"DiT layer {dk} not found")
                continue
            if vk not in vjepa_features:
                warnings.warn(f"V-JEPA layer {vk} not found")
                continue
            proj = self.projections[f"proj_{dl}_to_{vl}"](dit_features[dk])
            l = self._compute_alignment_loss(proj, vjepa_features[vk].detach(),
                                             self.config.alignment_type)
            per[dk] = l * self.config.per_layer_weights[i]
            total = total + per[dk]
        raw = total * w * self.config.base_repa_weight
        final = raw * self.config.repa_relative_weight
        self.loss_history["total"].append(final.detach())
        if len(self.loss_history["total"]) > 100:
            del self.loss_history["total"][:-100]
        out = {"total_repa_loss": final, "raw_repa_loss": raw, "repa_weight": w,
               "haste_phase": self.haste_scheduler.get_phase()}
        if return_per_layer:
            out["per_layer_losses"] = per
        return out

    def get_loss_stats(self) -> Dict[str, Any]:
        stats: Dict[str, Any] = {}
        h = self.loss_history["total"]
        if h:
            vals = torch.stack([t.float() for t in h]).cpu()
            stats["repa_mean"] = float(vals.mean())
            stats["repa_current"] = float(vals[-1])
        stats.update(self.haste_scheduler.get_progress_info())
        return stats


class REPAIntegration:
    def __init__(self, vjepa_backbone: nn.Module, repa_config: REPAConfig):
        self.vjepa_backbone = vjepa_backbone
        self.repa_loss = REPALoss(repa_config)
        self.config = repa_config

    def to(self, device) -> "REPAIntegration":
        self.repa_loss = self.repa_loss.to(device)
        self.vjepa_backbone = self.vjepa_backbone.to(device)
        return self

    def compute_repa_loss(self, video, dit_intermediate_features, step: int):
        with torch.no_grad():
            feats = self.vjepa_backbone(video, return_all_layers=True,
                                        max_layer=max(self.config.vjepa_layers_to_use))
        return self.repa_loss(dit_intermediate_features, feats["intermediate"], step=step)

    def is_active(self) -> bool:
        return self.repa_loss.haste_scheduler.is_active()

    def get_trainable_parameters(self):
        return self.repa_loss.projections.parameters()


def create_repa_loss(dit_hidden_dim: int, vjepa_feature_dim: int = 1024, dit_layers=None,
                     vjepa_layers=None, total_training_steps: int = 100000,
                     haste_termination_ratio: float = 0.4, **kwargs) -> REPALoss:
    cfg = REPAConfig(dit_hidden_dim=dit_hidden_dim, vjepa_feature_dim=vjepa_feature_dim,
                     dit_layers_to_align=dit_layers or [6, 8, 10],
                     vjepa_layers_to_use=vjepa_layers or [18, 20, 22],
                     total_training_steps=total_training_steps,
                     haste_termination_ratio=haste_termination_ratio,
                     **{k: v for k, v in kwargs.items() if k in REPAConfig.__dataclass_fields__})
    return REPALoss(cfg)
