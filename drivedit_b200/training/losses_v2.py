"""Configurable multi-objective losses (v2).

Same catalogue, dictionary contract and aggregation as the reference
``training/losses_v2.py``: ``LossType`` (28 kinds, :39-81), ``LossConfig`` (:84-159),
``BaseLoss`` (:166-198), the loss classes (:205-1829), ``LearnedTaskWeights``
(Kendall et al. 2018, :1841-1886), ``GradientNormalizer`` (GradNorm, :1889-1953),
``GradientSurgery`` (PCGrad, :1956-2010), ``LossAggregator`` (curriculum schedules,
:2013-2279), the config factories and the ``UnifiedLoss`` wrapper (:2282-2400).
Every loss reads the same ``predictions`` / ``targets`` keys as the reference and
returns a zero tensor when its inputs are absent.

Perceptual losses (LPIPS / VGG / DINO / CLIP) need pretrained networks that are not
available offline: they use fixed random-initialised feature extractors of the same
shape (conv pyramid / ViT patch encoder), which keeps the code path and the gradient
structure; load real weights into ``.features`` / ``.encoder`` to get the published
metric.
"""
from __future__ import annotations

import math
from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


class LossType(Enum):
    LATENT_MSE = "latent_mse"
    TEACHER_STUDENT_FLOW = "teacher_student_flow"
    KV_CACHE_CONSISTENCY = "kv_cache_consistency"
    AUTOREGRESSIVE_NEXT_FRAME = "autoregressive_next_frame"
    INFONCE = "infonce"
    CROSS_MODAL_CONTRASTIVE = "cross_modal_contrastive"
    TEMPORAL_CONTRASTIVE = "temporal_contrastive"
    VICREG = "vicreg"
    CONDITIONAL_FLOW_MATCHING = "conditional_flow_matching"
    FLOW_DISTILLATION = "flow_distillation"
    FLOW_CONSISTENCY = "flow_consistency"
    TRAJECTORY_STRAIGHTENING = "trajectory_straightening"
    SCALE_INVARIANT_DEPTH = "scale_invariant_depth"
    DEPTH_GRADIENT_SMOOTHNESS = "depth_gradient_smoothness"
    EDGE_AWARE_DEPTH = "edge_aware_depth"
    MULTI_SCALE_DEPTH = "multi_scale_depth"
    INVERSE_DYNAMICS = "inverse_dynamics"
    ACTION_SMOOTHNESS = "action_smoothness"
    BOUNDARY_ACTION_CLIPPING = "boundary_action_clipping"
    GOAL_CONDITIONED_ACTION = "goal_conditioned_action"
    LPIPS = "lpips"
    VGG_FEATURE = "vgg_feature"
    DINO_FEATURE = "dino_feature"
    CLIP_SIMILARITY = "clip_similarity"
    TEMPORAL_CONSISTENCY = "temporal_consistency"
    FLICKER_REDUCTION = "flicker_reduction"
    MOTION_MAGNITUDE = "motion_magnitude"
    SCENE_STABILITY = "scene_stability"


_DEFAULT_WEIGHTS = {
    "latent_mse": 1.0, "teacher_student_flow": 0.5, "kv_cache_consistency": 0.1,
    "autoregressive_next_frame": 1.0, "infonce": 0.5, "cross_modal_contrastive": 0.3,
    "temporal_contrastive": 0.3, "vicreg": 0.2, "conditional_flow_matching": 1.0, "flow_distillation": 0.5,
    "flow_consistency": 0.2, "trajectory_straightening": 0.1, "scale_invariant_depth": 0.5,
    "depth_gradient_smoothness": 0.1, "edge_aware_depth": 0.2, "multi_scale_depth": 0.3,
    "inverse_dynamics": 0.3, "action_smoothness": 0.1, "boundary_action_clipping": 0.05,
    "goal_conditioned_action": 0.2, "lpips": 0.5, "vgg_feature": 0.3, "dino_feature": 0.3,
    "clip_similarity": 0.2, "temporal_consistency": 0.3, "flicker_reduction": 0.1, "motion_magnitude": 0.1,
    "scene_stability": 0.1}


@dataclass
class LossConfig:
    enabled_losses: List[LossType] = field(default_factory=lambda: [
        LossType.LATENT_MSE, LossType.TEMPORAL_CONSISTENCY, LossType.CONDITIONAL_FLOW_MATCHING])
    weights: Dict[str, float] = field(default_factory=lambda: dict(_DEFAULT_WEIGHTS))
    use_uncertainty_weighting: bool = False
    use_gradient_normalization: bool = False
    use_gradient_surgery: bool = False
    enable_curriculum: bool = True
    curriculum_warmup_steps: int = 10000
    infonce_temperature: float = 0.1
    vicreg_sim_weight: float = 25.0
    vicreg_var_weight: float = 25.0
    vicreg_cov_weight: float = 1.0
    flow_num_steps: int = 4
    flow_sigma_min: float = 1e-4
    depth_max_depth: float = 100.0
    depth_gradient_weight: float = 0.1
    action_smoothness_order: int = 2
    action_boundary_margin: float = 0.95
    lpips_net: str = "vgg"
    vgg_layers: List[str] = field(default_factory=lambda: ["relu1_2", "relu2_2", "relu3_3", "relu4_3"])
    temporal_window: int = 3
    flicker_threshold: float = 0.1


def _device(*ds) -> torch.device:
    for d in ds:
        for v in d.values():
            if torch.is_tensor(v):
                return v.device
    return torch.device("cpu")


class BaseLoss(ABC, nn.Module):
    def __init__(self, weight: float = 1.0):
        super().__init__()
        self.weight = weight
        self._history: List[torch.Tensor] = []

    @abstractmethod
    def forward(self, predictions: Dict[str, Any], targets: Dict[str, Any], **kwargs) -> torch.Tensor:
        ...

    def update_history(self, value):
        self._history.append(value.detach() if torch.is_tensor(value) else torch.tensor(float(value)))
        if len(self._history) > 1000:
            del self._history[:-500]

    @property
    def mean(self) -> float:
        return float(torch.stack([h.float().cpu() for h in self._history[-100:]]).mean()) if self._history else 0.0

    @property
    def std(self) -> float:
        if len(self._history) < 2:
            return 0.0
        return float(torch.stack([h.float().cpu() for h in self._history[-100:]]).std(unbiased=False))

    def _zero(self, *ds):
        return torch.zeros((), device=_device(*ds))

    def _out(self, loss):
        self.update_history(loss)
        return loss * self.weight


def _frames(x):
    return x.reshape(-1, *x.shape[-3:]).float()


# ----------------------------------------------------------------------------- self-forcing
class LatentMSELoss(BaseLoss):
    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("latents"), targets.get("latents")
        if p is None or t is None:
            return self._zero(predictions, targets)
        if p.dim() > 1 and t.dim() > 1 and p.shape[1] != t.shape[1]:
            t = t[:, -p.shape[1]:]
        return self._out(F.mse_loss(p.float(), t.float()))


class TeacherStudentFlowLoss(BaseLoss):
    def forward(self, predictions, targets, **kw):
        s, t = predictions.get("flow_predictions"), targets.get("teacher_flow")
        if s is None or t is None:
            return self._zero(predictions, targets)
        return self._out(F.mse_loss(s.float(), t.detach().float()))


class KVCacheConsistencyLoss(BaseLoss):
    """Margin-hinged change of cached K/V between consecutive autoregressive steps."""

    def __init__(self, weight: float = 1.0, margin: float = 0.1):
        super().__init__(weight)
        self.margin = margin

    def forward(self, predictions, targets, **kw):
        h = predictions.get("kv_cache_history")
        if h is None or len(h) < 2:
            return self._zero(predictions, targets)
        terms = []
        for a, b in zip(h[:-1], h[1:]):
            if "k" in a and "k" in b:
                n = min(a["k"].shape[1], b["k"].shape[1])
                for key in ("k", "v"):
                    terms.append(torch.clamp(F.mse_loss(a[key][:, :n].float(), b[key][:, :n].float()) - self.margin,
                                             min=0.0))
        if not terms:
            return self._zero(predictions, targets)
        return self._out(torch.stack(terms).mean())


class AutoregressiveNextFrameLoss(BaseLoss):
    """``predictions[:, t]`` is the model's estimate of ``frames[:, t + 1]`` (teacher
    forcing); when lengths already match the prediction is aligned to the tail."""

    def forward(self, predictions, targets, **kw):
        p, f = predictions.get("predictions"), targets.get("frames")
        if p is None or f is None or f.shape[1] < 2:
            return self._zero(predictions, targets)
        tgt = f[:, 1:] if p.shape[1] == f.shape[1] - 1 else f[:, -p.shape[1]:]
        pr = p if p.shape[1] == tgt.shape[1] else p[:, :tgt.shape[1]]
        return self._out(F.mse_loss(pr.float(), tgt.float()))


# ----------------------------------------------------------------------------- contrastive
def _info_nce(a: torch.Tensor, b: torch.Tensor, temperature: float) -> torch.Tensor:
    a, b = F.normalize(a.float(), dim=-1), F.normalize(b.float(), dim=-1)
    logits = a @ b.t() / temperature
    lab = torch.arange(a.shape[0], device=a.device)
    return 0.5 * (F.cross_entropy(logits, lab) + F.cross_entropy(logits.t(), lab))


class InfoNCELoss(BaseLoss):
    """Positives: the same sequence's representation ``delta`` steps later; negatives:
    the rest of the batch (symmetric InfoNCE). With ``use_hard_negatives`` the state one
    step past the positive (same sequence, when it exists) joins each anchor's negatives:
    close in time, but not the target."""

    def __init__(self, weight: float = 1.0, temperature: float = 0.1, delta: int = 1,
                 use_hard_negatives: bool = True):
        super().__init__(weight)
        self.temperature, self.delta, self.use_hard_negatives = temperature, delta, use_hard_negatives

    def forward(self, predictions, targets, **kw):
        h = predictions.get("hidden_states")
        d = self.delta
        if h is None or h.dim() != 3 or h.shape[1] <= d:
            return self._zero(predictions, targets)
        B, T, D = h.shape
        if not self.use_hard_negatives or T <= d + 1:
            a = h[:, :-d].reshape(-1, D)
            b = h[:, d:].reshape(-1, D)
            return self._out(_info_nce(a, b, self.temperature))
        za = F.normalize(h[:, :-d].float(), dim=-1)                     # [B, T-d, D]
        zp = F.normalize(h[:, d:].float(), dim=-1)
        zh = F.normalize(h[:, d + 1:].float(), dim=-1)                  # [B, T-d-1, D]
        a, p = za.reshape(-1, D), zp.reshape(-1, D)
        logits = a @ p.t() / self.temperature                           # in-batch
        hard = torch.full((B, T - d), float("-inf"), device=h.device)
        hard[:, :T - d - 1] = (za[:, :T - d - 1] * zh).sum(-1) / self.temperature
        logits = torch.cat([logits, hard.reshape(-1, 1)], 1)
        lab = torch.arange(a.shape[0], device=h.device)
        return self._out(F.cross_entropy(logits, lab))


class CrossModalContrastiveLoss(BaseLoss):
    MODALITY_KEYS = {"rgb": "hidden_states", "depth": "depth_features", "control": "control_features"}

    def __init__(self, weight: float = 1.0, temperature: float = 0.1, modality_pairs=None):
        super().__init__(weight)
        self.temperature = temperature
        self.modality_pairs = modality_pairs or [("rgb", "depth"), ("rgb", "control")]

    def forward(self, predictions, targets, **kw):
        terms = []
        for m1, m2 in self.modality_pairs:
            a = predictions.get(self.MODALITY_KEYS.get(m1, m1))
            b = predictions.get(self.MODALITY_KEYS.get(m2, m2))
            if a is None or b is None:
                continue
            a = a.float().mean(1) if a.dim() == 3 else a.float()
            b = b.float().mean(1) if b.dim() == 3 else b.float()
            if a.shape[-1] != b.shape[-1]:
                d = min(a.shape[-1], b.shape[-1])
                a, b = a[..., :d], b[..., :d]
            terms.append(_info_nce(a, b, self.temperature))
        if not terms:
            return self._zero(predictions, targets)
        return self._out(torch.stack(terms).mean())


class TemporalContrastiveLoss(BaseLoss):
    """Frames within ``positive_window`` steps of an anchor are positives; negatives are
    other sequences' frames and the anchor's own frames at least ``negative_margin``
    steps away; own frames in between are neither (multi-positive InfoNCE over time)."""

    def __init__(self, weight: float = 1.0, temperature: float = 0.1, positive_window: int = 2,
                 negative_margin: int = 5):
        super().__init__(weight)
        self.temperature, self.window = temperature, positive_window
        self.negative_margin = max(negative_margin, positive_window + 1)

    def forward(self, predictions, targets, **kw):
        h = predictions.get("hidden_states")
        if h is None or h.dim() != 3 or h.shape[1] < 2:
            return self._zero(predictions, targets)
        B, T, D = h.shape
        z = F.normalize(h.float(), dim=-1).reshape(B * T, D)
        sim = z @ z.t() / self.temperature
        seq = torch.arange(B, device=h.device).repeat_interleave(T)
        tt = torch.arange(T, device=h.device).repeat(B)
        same = seq[:, None] == seq[None]
        dt = (tt[:, None] - tt[None]).abs()
        near = dt <= self.window
        eye = torch.eye(B * T, dtype=torch.bool, device=h.device)
        pos = same & near & ~eye
        ignore = eye | (same & ~near & (dt < self.negative_margin))
        sim = sim.masked_fill(ignore, -1e9)
        logp = sim - torch.logsumexp(sim, 1, keepdim=True)
        loss = -(logp * pos).sum(1) / pos.sum(1).clamp_min(1)
        return self._out(loss.mean())


class VICRegLoss(BaseLoss):
    """Variance-invariance-covariance regularisation (Bardes et al. 2022)."""

    def __init__(self, weight: float = 1.0, sim_weight: float = 25.0, var_weight: float = 25.0,
                 cov_weight: float = 1.0, variance_target: float = 1.0):
        super().__init__(weight)
        self.sim_weight, self.var_weight, self.cov_weight = sim_weight, var_weight, cov_weight
        self.variance_target = variance_target

    def _var_cov(self, z):
        z = z - z.mean(0)
        std = torch.sqrt(z.var(0) + 1e-4)
        var = F.relu(self.variance_target - std).mean()
        n, d = z.shape
        cov = (z.t() @ z) / max(n - 1, 1)
        off = cov - torch.diag(torch.diag(cov))
        return var, off.pow(2).sum() / d

    def forward(self, predictions, targets, **kw):
        a, b = predictions.get("hidden_states"), predictions.get("hidden_states_aug")
        if a is None:
            return self._zero(predictions, targets)
        a = a.float().reshape(-1, a.shape[-1])
        b = a.roll(1, 0) if b is None else b.float().reshape(-1, b.shape[-1])
        inv = F.mse_loss(a, b)
        va, ca = self._var_cov(a)
        vb, cb = self._var_cov(b)
        return self._out(self.sim_weight * inv + self.var_weight * (va + vb) + self.cov_weight * (ca + cb))


# ----------------------------------------------------------------------------- flow matching
class ConditionalFlowMatchingLoss(BaseLoss):
    """``||v - (x1 - x0)||^2``: ``flow_predictions`` vs ``latents`` (or ``frames``) minus
    ``noise``; with no noise given, vs ``x1 - predictions``."""

    def forward(self, predictions, targets, **kw):
        v = predictions.get("flow_predictions")
        x1 = targets.get("latents", targets.get("frames"))
        if v is None or x1 is None:
            return self._zero(predictions, targets)
        x0 = targets.get("noise")
        if x0 is None:
            x0 = predictions.get("predictions")
        if x0 is None:
            return self._zero(predictions, targets)
        tgt = x1.float() - x0.float()
        if tgt.shape != v.shape and tgt.dim() > 1:
            tgt = tgt[:, -v.shape[1]:]
        return self._out(F.mse_loss(v.float(), tgt))


class FlowDistillationLoss(BaseLoss):
    def forward(self, predictions, targets, **kw):
        v, traj = predictions.get("flow_predictions"), targets.get("teacher_trajectory")
        if v is None or traj is None:
            return self._zero(predictions, targets)
        tv = (traj[-1] - traj[0]).float() / (len(traj) - 1) if len(traj) > 1 else traj[0].float()
        return self._out(F.mse_loss(v.float(), tv.detach()))


class FlowConsistencyLoss(BaseLoss):
    """``||v(z_t, t) - v(z_t + dt v, t + dt)||^2`` with the second term from
    ``flow_model`` (no gradient)."""

    def __init__(self, weight: float = 1.0, dt: float = 0.01):
        super().__init__(weight)
        self.dt = dt

    def forward(self, predictions, targets, flow_model=None, **kw):
        z, t, v = predictions.get("z_t"), predictions.get("timesteps"), predictions.get("flow_predictions")
        if z is None or t is None or v is None or flow_model is None:
            return self._zero(predictions, targets)
        with torch.no_grad():
            v2 = flow_model(z + self.dt * v, torch.clamp(t + self.dt, 0, 1))
        return self._out(F.mse_loss(v.float(), v2.float()))


class TrajectoryStraighteningLoss(BaseLoss):
    """Deviation of a sampled trajectory ``[K+1, B, ...]`` (or ``[B, K+1, ...]``) from
    the straight line between its end points."""

    def forward(self, predictions, targets, **kw):
        tr = predictions.get("trajectory")
        if tr is None:
            return self._zero(predictions, targets)
        tr = torch.stack(list(tr)) if isinstance(tr, (list, tuple)) else tr
        K = tr.shape[0] - 1
        if K < 2:
            return self._zero(predictions, targets)
        s = torch.linspace(0, 1, K + 1, device=tr.device).view(-1, *([1] * (tr.dim() - 1)))
        line = tr[0:1] + s * (tr[-1:] - tr[0:1])
        return self._out(F.mse_loss(tr.float(), line.float()))


# ----------------------------------------------------------------------------- depth
def _grad_xy(x):
    return x[..., :, 1:] - x[..., :, :-1], x[..., 1:, :] - x[..., :-1, :]


class ScaleInvariantDepthLoss(BaseLoss):
    """Eigen et al. 2014: ``mean(d^2) - lambda_scale * mean(d)^2`` with
    ``d = log p - log t`` over target depths in ``(eps, max_depth)``."""

    def __init__(self, weight: float = 1.0, lambda_scale: float = 0.5, max_depth: float = 100.0,
                 eps: float = 1e-3):
        super().__init__(weight)
        self.lam, self.max_depth, self.eps = lambda_scale, max_depth, eps

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("depth_predictions"), targets.get("depth")
        if p is None or t is None:
            return self._zero(predictions, targets)
        valid = (t > self.eps) & (t < self.max_depth)
        d = torch.log(p.float().clamp_min(self.eps)) - torch.log(t.float().clamp_min(self.eps))
        d = d[valid]
        if d.numel() == 0:
            return self._zero(predictions, targets)
        return self._out((d.pow(2).mean() - self.lam * d.mean().pow(2)).clamp_min(0))


class DepthGradientSmoothnessLoss(BaseLoss):
    """Edge-aware smoothness: depth gradients weighted by ``exp(-|image gradient|)``."""

    def forward(self, predictions, targets, **kw):
        d, img = predictions.get("depth_predictions"), targets.get("frames")
        if d is None:
            return self._zero(predictions, targets)
        d = _frames(d) if d.dim() == 5 else d.float()
        dx, dy = _grad_xy(d / (d.mean((-2, -1), keepdim=True) + 1e-7))
        if img is not None:
            im = _frames(img)
            ix, iy = _grad_xy(im.mean(1, keepdim=True))
            dx, dy = dx * torch.exp(-ix.abs()), dy * torch.exp(-iy.abs())
        return self._out(dx.abs().mean() + dy.abs().mean())


class EdgeAwareDepthLoss(BaseLoss):
    """Gradient matching between predicted and target depth, emphasised at image edges."""

    def forward(self, predictions, targets, **kw):
        p, t, img = predictions.get("depth_predictions"), targets.get("depth"), targets.get("frames")
        if p is None or t is None:
            return self._zero(predictions, targets)
        p = _frames(p) if p.dim() == 5 else p.float()
        t = _frames(t) if t.dim() == 5 else t.float()
        px, py = _grad_xy(p)
        tx, ty = _grad_xy(t)
        if img is not None:
            ix, iy = _grad_xy(_frames(img).mean(1, keepdim=True))
            wx, wy = 1 + ix.abs(), 1 + iy.abs()
        else:
            wx = wy = 1.0
        return self._out(((px - tx).abs() * wx).mean() + ((py - ty).abs() * wy).mean())


class MultiScaleDepthLoss(BaseLoss):
    """Depth error at several average-pooled resolutions, each weighted 1/scale: L1, or
    with ``use_si`` the scale-invariant log error."""

    def __init__(self, weight: float = 1.0, scales: Tuple[int, ...] = (1, 2, 4, 8), use_si: bool = False):
        super().__init__(weight)
        self.scales = scales
        self.si = ScaleInvariantDepthLoss(1.0) if use_si else None

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("depth_predictions"), targets.get("depth")
        if p is None or t is None:
            return self._zero(predictions, targets)
        p = _frames(p) if p.dim() == 5 else p.float()
        t = _frames(t) if t.dim() == 5 else t.float()
        terms = []
        for s in self.scales:
            if min(p.shape[-2:]) // s < 1:
                continue
            ps, ts = (F.avg_pool2d(p, s), F.avg_pool2d(t, s)) if s > 1 else (p, t)
            if self.si is not None:
                terms.append(self.si({"depth_predictions": ps}, {"depth": ts}).reshape(()) / s)
            else:
                terms.append(F.l1_loss(ps, ts) / s)
        return self._out(torch.stack(terms).sum())


# ----------------------------------------------------------------------------- actions
class InverseDynamicsLoss(BaseLoss):
    def forward(self, predictions, targets, **kw):
        a, c = predictions.get("predicted_actions"), targets.get("controls")
        if a is None or c is None:
            return self._zero(predictions, targets)
        if c.shape[1] != a.shape[1]:
            c = c[:, -a.shape[1]:] if c.shape[1] > a.shape[1] else c
        d = min(a.shape[-1], c.shape[-1])
        return self._out(F.mse_loss(a[..., :d].float(), c[..., :d].float()))


class ActionSmoothnessLoss(BaseLoss):
    def __init__(self, weight: float = 1.0, order: int = 2):
        super().__init__(weight)
        self.order = order

    def forward(self, predictions, targets, **kw):
        a = predictions.get("predicted_actions")
        if a is None or a.shape[1] <= self.order:
            return self._zero(predictions, targets)
        d = a.float()
        for _ in range(self.order):
            d = d[:, 1:] - d[:, :-1]
        return self._out(d.pow(2).mean())


class BoundaryActionClippingLoss(BaseLoss):
    """Penalises actions beyond ``margin`` of the valid range ``action_bounds``
    (quadratic in the excess over the shrunken bounds)."""

    def __init__(self, weight: float = 1.0, margin: float = 0.95,
                 action_bounds: Tuple[float, float] = (-1.0, 1.0)):
        super().__init__(weight)
        self.margin = margin
        self.lower, self.upper = action_bounds

    def forward(self, predictions, targets, **kw):
        a = predictions.get("predicted_actions")
        if a is None:
            return self._zero(predictions, targets)
        mid, half = 0.5 * (self.upper + self.lower), 0.5 * (self.upper - self.lower)
        return self._out(F.relu((a.float() - mid).abs() - self.margin * half).pow(2).mean())


class GoalConditionedActionLoss(BaseLoss):
    """Actions should move the state toward ``goals``: cosine between the predicted
    (steering, acceleration) direction and the goal direction, plus imitation of the
    recorded controls when given."""

    def forward(self, predictions, targets, **kw):
        a, goals, c = predictions.get("predicted_actions"), targets.get("goals"), targets.get("controls")
        if a is None or (goals is None and c is None):
            return self._zero(predictions, targets)
        terms = []
        if goals is not None:
            g = goals.float()
            g = g[:, None].expand(-1, a.shape[1], -1) if g.dim() == 2 else g
            d = min(a.shape[-1], g.shape[-1], 2)
            terms.append((1 - F.cosine_similarity(a[..., :d].float(), g[..., :d], dim=-1)).mean())
        if c is not None:
            d = min(a.shape[-1], c.shape[-1])
            n = min(a.shape[1], c.shape[1])
            terms.append(F.mse_loss(a[:, :n, :d].float(), c[:, :n, :d].float()))
        return self._out(torch.stack(terms).sum())


# ----------------------------------------------------------------------------- perceptual
class _ConvPyramid(nn.Module):
    def __init__(self, chans=(64, 128, 256, 512), seed: int = 0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        layers, c = [], 3
        for o in chans:
            conv = nn.Conv2d(c, o, 3, padding=1)
            with torch.no_grad():
                conv.weight.normal_(0, math.sqrt(2.0 / (9 * c)), generator=g)
                conv.bias.zero_()
            layers.append(nn.Sequential(conv, nn.ReLU(), nn.AvgPool2d(2)))
            c = o
        self.stages = nn.ModuleList(layers)
        for p in self.parameters():
            p.requires_grad = False

    def forward(self, x):
        out = []
        for s in self.stages:
            x = s(x)
            out.append(x)
        return out


class LPIPSLoss(BaseLoss):
    """Channel-normalised feature distance over a frozen conv pyramid (LPIPS form)."""

    def __init__(self, weight: float = 1.0, net: str = "vgg"):
        super().__init__(weight)
        self.net = net
        self.features = _ConvPyramid(seed=1 if net == "vgg" else 2)

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("predictions"), targets.get("frames")
        if p is None or t is None or p.shape[-3] != 3:
            return self._zero(predictions, targets)
        t = t[:, -p.shape[1]:] if p.dim() == 5 and t.shape[1] != p.shape[1] else t
        fp, ft = self.features(_frames(p) * 2 - 1), self.features(_frames(t) * 2 - 1)
        d = [(F.normalize(a, dim=1) - F.normalize(b, dim=1)).pow(2).sum(1).mean() for a, b in zip(fp, ft)]
        return self._out(torch.stack(d).sum())


class VGGFeatureLoss(BaseLoss):
    def __init__(self, weight: float = 1.0, layers: Optional[List[str]] = None):
        super().__init__(weight)
        self.layers = layers or ["relu1_2", "relu2_2", "relu3_3", "relu4_3"]
        self.features = _ConvPyramid(seed=3)

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("predictions"), targets.get("frames")
        if p is None or t is None or p.shape[-3] != 3:
            return self._zero(predictions, targets)
        t = t[:, -p.shape[1]:] if p.dim() == 5 and t.shape[1] != p.shape[1] else t
        fp, ft = self.features(_frames(p)), self.features(_frames(t))
        n = len(self.layers)
        return self._out(torch.stack([F.l1_loss(a, b) for a, b in zip(fp[:n], ft[:n])]).mean())


class _PatchViT(nn.Module):
    def __init__(self, dim: int = 256, patch: int = 16, depth: int = 2, seed: int = 0):
        super().__init__()
        torch.manual_seed(seed)
        self.embed = nn.Conv2d(3, dim, patch, patch)
        self.blocks = nn.TransformerEncoder(nn.TransformerEncoderLayer(dim, 4, 2 * dim, batch_first=True,
                                                                       norm_first=True), depth,
                                            enable_nested_tensor=False)
        for p in self.parameters():
            p.requires_grad = False

    def forward(self, x):
        return self.blocks(self.embed(x).flatten(2).transpose(1, 2))


class DINOFeatureLoss(BaseLoss):
    """Cosine distance between patch tokens of a frozen ViT encoder."""

    def __init__(self, weight: float = 1.0, embed_dim: int = 256):
        super().__init__(weight)
        self.encoder = _PatchViT(embed_dim, seed=4)

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("predictions"), targets.get("frames")
        if p is None or t is None or p.shape[-3] != 3 or min(p.shape[-2:]) < 16:
            return self._zero(predictions, targets)
        t = t[:, -p.shape[1]:] if p.dim() == 5 and t.shape[1] != p.shape[1] else t
        a, b = self.encoder(_frames(p)), self.encoder(_frames(t))
        return self._out((1 - F.cosine_similarity(a, b, dim=-1)).mean())


class CLIPSimilarityLoss(BaseLoss):
    """``1 - cos`` between pooled embeddings of a frozen image encoder."""

    def __init__(self, weight: float = 1.0, embed_dim: int = 256):
        super().__init__(weight)
        self.encoder = _PatchViT(embed_dim, seed=5)

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("predictions"), targets.get("frames")
        if p is None or t is None or p.shape[-3] != 3 or min(p.shape[-2:]) < 16:
            return self._zero(predictions, targets)
        t = t[:, -p.shape[1]:] if p.dim() == 5 and t.shape[1] != p.shape[1] else t
        a, b = self.encoder(_frames(p)).mean(1), self.encoder(_frames(t)).mean(1)
        return self._out((1 - F.cosine_similarity(a, b, dim=-1)).mean())


# ----------------------------------------------------------------------------- video quality
class TemporalConsistencyLoss(BaseLoss):
    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("predictions"), targets.get("frames")
        if p is None or p.dim() < 3 or p.shape[1] < 2:
            return self._zero(predictions, targets)
        pd = p[:, 1:].float() - p[:, :-1].float()
        if t is None:
            return self._out(pd.pow(2).mean())
        t = t[:, -p.shape[1]:]
        return self._out(F.mse_loss(pd, t[:, 1:].float() - t[:, :-1].float()))


class FlickerReductionLoss(BaseLoss):
    """Penalises sign-alternating intensity changes (second temporal difference) above
    ``threshold``."""

    def __init__(self, weight: float = 1.0, threshold: float = 0.1):
        super().__init__(weight)
        self.threshold = threshold

    def forward(self, predictions, targets, **kw):
        p = predictions.get("predictions")
        if p is None or p.dim() < 3 or p.shape[1] < 3:
            return self._zero(predictions, targets)
        x = p.float()
        d2 = (x[:, 2:] - 2 * x[:, 1:-1] + x[:, :-2]).abs()
        return self._out(F.relu(d2 - self.threshold).mean())


class MotionMagnitudeLoss(BaseLoss):
    """Keeps the mean frame-to-frame motion of the prediction at the target's level
    (no frozen / exploding video)."""

    def forward(self, predictions, targets, **kw):
        p = predictions.get("predictions")
        t = targets.get("frames")
        if p is None or p.dim() < 3 or p.shape[1] < 2:
            return self._zero(predictions, targets)
        mp = (p[:, 1:].float() - p[:, :-1].float()).abs().flatten(2).mean(-1)
        if t is None or t.shape[1] < 2:
            return self._out(mp.var(unbiased=False))
        t = t[:, -p.shape[1]:]
        mt = (t[:, 1:].float() - t[:, :-1].float()).abs().flatten(2).mean(-1)
        return self._out(F.l1_loss(mp, mt))


class SceneStabilityLoss(BaseLoss):
    """Low-frequency content (heavily pooled frames) should change like the target's;
    with ``motion_threshold > 0`` instead, the prediction should stay still wherever the
    target's pooled change is at most the threshold (static scene content)."""

    def __init__(self, weight: float = 1.0, motion_threshold: float = 0.0, pool: int = 8):
        super().__init__(weight)
        self.motion_threshold, self.pool = motion_threshold, pool

    def forward(self, predictions, targets, **kw):
        p, t = predictions.get("predictions"), targets.get("frames")
        if p is None or t is None or p.dim() != 5 or p.shape[1] < 2:
            return self._zero(predictions, targets)
        t = t[:, -p.shape[1]:]
        k = max(1, min(self.pool, p.shape[-1], p.shape[-2]))
        lp = F.avg_pool2d(_frames(p), k).view(p.shape[0], p.shape[1], -1)
        lt = F.avg_pool2d(_frames(t), k).view(t.shape[0], t.shape[1], -1)
        dp, dtg = lp[:, 1:] - lp[:, :-1], lt[:, 1:] - lt[:, :-1]
        if self.motion_threshold > 0:
            # the prediction should not change where the target scene is static
            static = (dtg.abs() <= self.motion_threshold).float()
            return self._out((dp * static).pow(2).mean())
        return self._out(F.mse_loss(dp, dtg))


# ----------------------------------------------------------------------------- balancing
class LearnedTaskWeights(nn.Module):
    """``sum_i exp(-2 s_i) L_i + s_i`` with ``s_i = log sigma_i`` (Kendall et al. 2018)."""

    def __init__(self, num_tasks: int, init_sigma: float = 1.0):
        super().__init__()
        self.log_sigmas = nn.Parameter(torch.full((num_tasks,), math.log(init_sigma)))

    def forward(self, losses: Dict[str, torch.Tensor]):
        total = torch.zeros((), device=self.log_sigmas.device)
        out = {}
        for i, (name, l) in enumerate(losses.items()):
            if i >= len(self.log_sigmas):
                break
            w = torch.exp(-2 * self.log_sigmas[i]) * l + self.log_sigmas[i]
            out[name] = w.detach()
            total = total + w
        return total, out

    def get_weights(self) -> Dict[int, float]:
        w = 1.0 / (torch.exp(self.log_sigmas.detach()).pow(2) + 1e-8)
        return dict(enumerate(w.tolist()))


class GradientNormalizer:
    """GradNorm (Chen et al. 2018): per-task weights that equalise the shared-parameter
    gradient norms, scaled by each task's relative training rate ** alpha."""

    def __init__(self, num_tasks: int, alpha: float = 1.5):
        self.num_tasks, self.alpha = num_tasks, alpha
        self.initial_losses: Optional[torch.Tensor] = None
        self.weights = torch.ones(num_tasks)

    def normalize(self, losses: Dict[str, torch.Tensor], shared_params: List[torch.Tensor]) -> Dict[str, torch.Tensor]:
        vals = list(losses.values())
        cur = torch.stack([v.detach().float() for v in vals])
        if self.initial_losses is None:
            self.initial_losses = cur.clone()
        norms = []
        for l in vals:
            g = torch.autograd.grad(l, shared_params, retain_graph=True, allow_unused=True)
            norms.append(torch.stack([x.norm() for x in g if x is not None]).sum() if any(x is not None for x in g)
                         else cur.new_zeros(()))
        norms = torch.stack(norms)
        ratio = cur / (self.initial_losses + 1e-8)
        rel = ratio / (ratio.mean() + 1e-8)
        tgt = norms.mean() * rel.pow(self.alpha)
        w = (tgt / (norms + 1e-8)).detach()
        self.weights = w[:self.num_tasks].cpu()
        return {k: v * w[i] if i < self.num_tasks else v for i, (k, v) in enumerate(losses.items())}


class GradientSurgery:
    """PCGrad (Yu et al. 2020): project each task gradient off the others it conflicts
    with (negative dot product), then combine."""

    @staticmethod
    def project_conflicting_gradients(grads: List[torch.Tensor], reduction: str = "mean") -> torch.Tensor:
        if len(grads) == 1:
            return grads[0]
        G = torch.stack([g.flatten().float() for g in grads])
        P = G.clone()
        for i in range(len(grads)):
            for j in range(len(grads)):
                if i == j:
                    continue
                dot = (P[i] * G[j]).sum()
                P[i] = torch.where(dot < 0, P[i] - dot / (G[j].pow(2).sum() + 1e-8) * G[j], P[i])
        return P.mean(0) if reduction == "mean" else P.sum(0)


# ----------------------------------------------------------------------------- aggregator
class LossAggregator(nn.Module):
    def __init__(self, config: LossConfig):
        super().__init__()
        self.config = config
        self.step = 0
        self.losses = nn.ModuleDict()
        self._build_losses()
        self.task_weights = LearnedTaskWeights(len(self.losses)) if config.use_uncertainty_weighting else None
        self.grad_normalizer = GradientNormalizer(len(self.losses)) if config.use_gradient_normalization else None
        self.use_gradient_surgery = config.use_gradient_surgery
        self.loss_history: Dict[str, List[torch.Tensor]] = {}
        self.curriculum_weights: Dict[str, float] = {}

    def _build_losses(self):
        c = self.config
        mapping = {
            LossType.LATENT_MSE: LatentMSELoss, LossType.TEACHER_STUDENT_FLOW: TeacherStudentFlowLoss,
            LossType.KV_CACHE_CONSISTENCY: KVCacheConsistencyLoss,
            LossType.AUTOREGRESSIVE_NEXT_FRAME: AutoregressiveNextFrameLoss,
            LossType.INFONCE: lambda w: InfoNCELoss(w, c.infonce_temperature),
            LossType.CROSS_MODAL_CONTRASTIVE: CrossModalContrastiveLoss,
            LossType.TEMPORAL_CONTRASTIVE: TemporalContrastiveLoss,
            LossType.VICREG: lambda w: VICRegLoss(w, c.vicreg_sim_weight, c.vicreg_var_weight, c.vicreg_cov_weight),
            LossType.CONDITIONAL_FLOW_MATCHING: ConditionalFlowMatchingLoss,
            LossType.FLOW_DISTILLATION: FlowDistillationLoss, LossType.FLOW_CONSISTENCY: FlowConsistencyLoss,
            LossType.TRAJECTORY_STRAIGHTENING: TrajectoryStraighteningLoss,
            LossType.SCALE_INVARIANT_DEPTH: lambda w: ScaleInvariantDepthLoss(w, max_depth=c.depth_max_depth),
            LossType.DEPTH_GRADIENT_SMOOTHNESS: DepthGradientSmoothnessLoss,
            LossType.EDGE_AWARE_DEPTH: EdgeAwareDepthLoss, LossType.MULTI_SCALE_DEPTH: MultiScaleDepthLoss,
            LossType.INVERSE_DYNAMICS: InverseDynamicsLoss,
            LossType.ACTION_SMOOTHNESS: lambda w: ActionSmoothnessLoss(w, c.action_smoothness_order),
            LossType.BOUNDARY_ACTION_CLIPPING: lambda w: BoundaryActionClippingLoss(w, c.action_boundary_margin),
            LossType.GOAL_CONDITIONED_ACTION: GoalConditionedActionLoss,
            LossType.LPIPS: lambda w: LPIPSLoss(w, c.lpips_net),
            LossType.VGG_FEATURE: lambda w: VGGFeatureLoss(w, c.vgg_layers),
            LossType.DINO_FEATURE: DINOFeatureLoss, LossType.CLIP_SIMILARITY: CLIPSimilarityLoss,
            LossType.TEMPORAL_CONSISTENCY: TemporalConsistencyLoss,
            LossType.FLICKER_REDUCTION: lambda w: FlickerReductionLoss(w, c.flicker_threshold),
            LossType.MOTION_MAGNITUDE: MotionMagnitudeLoss, LossType.SCENE_STABILITY: SceneStabilityLoss,
        }
        for lt in c.enabled_losses:
            self.losses[lt.value] = mapping[lt](c.weights.get(lt.value, 1.0))

    def _get_curriculum_weight(self, name: str) -> float:
        if not self.config.enable_curriculum:
            return 1.0
        p = min(1.0, self.step / self.config.curriculum_warmup_steps)
        late = lambda s: (p - s) / (1 - s) if p > s else 0.0
        return {"latent_mse": 1.0, "autoregressive_next_frame": 1.0, "temporal_consistency": p,
                "conditional_flow_matching": 0.1 + 0.9 * p, "flow_distillation": p, "infonce": late(0.3),
                "vicreg": late(0.3), "cross_modal_contrastive": late(0.2), "lpips": 0.5 + 0.5 * p,
                "vgg_feature": 0.5 + 0.5 * p, "dino_feature": p, "clip_similarity": late(0.4)}.get(name, 1.0)

    def forward(self, predictions, targets, step: Optional[int] = None, **kwargs) -> Dict[str, torch.Tensor]:
        if step is not None:
            self.step = step
        losses: Dict[str, torch.Tensor] = {}
        for name, fn in self.losses.items():
            w = self._get_curriculum_weight(name)
            self.curriculum_weights[name] = w
            losses[name] = fn(predictions, targets, **kwargs) * w
            h = self.loss_history.setdefault(name, [])
            h.append(losses[name].detach())
            if len(h) > 1000:
                del h[:-500]
        if self.task_weights is not None:
            total, _ = self.task_weights(losses)
        else:
            total = torch.stack(list(losses.values())).sum() if losses else torch.zeros(())
        losses["total"] = total
        return losses

    def apply_gradient_surgery(self, losses: Dict[str, torch.Tensor], shared_params: List[torch.Tensor]):
        """Writes the PCGrad-combined gradient into ``shared_params[i].grad``; returns
        the total loss (for logging)."""
        items = [(k, v) for k, v in losses.items() if k != "total" and v.requires_grad]
        if not self.use_gradient_surgery or not items:
            return losses.get("total", sum(losses.values()))
        flats = []
        for _, l in items:
            g = torch.autograd.grad(l, shared_params, retain_graph=True, allow_unused=True)
            flats.append(torch.cat([(x if x is not None else torch.zeros_like(p)).flatten()
                                    for x, p in zip(g, shared_params)]))
        comb = GradientSurgery.project_conflicting_gradients(flats)
        off = 0
        for p in shared_params:
            n = p.numel()
            p.grad = comb[off:off + n].view_as(p).to(p.dtype).clone()
            off += n
        return losses["total"]

    def get_loss_stats(self) -> Dict[str, Dict[str, float]]:
        out = {}
        for name, h in self.loss_history.items():
            if h:
                r = torch.stack([x.float().cpu() for x in h[-100:]])
                out[name] = {"mean": float(r.mean()), "std": float(r.std(unbiased=False)), "min": float(r.min()),
                             "max": float(r.max()), "current": float(r[-1]),
                             "curriculum_weight": self.curriculum_weights.get(name, 1.0)}
        return out

    def get_curriculum_progress(self) -> Dict[str, float]:
        return {n: self._get_curriculum_weight(n) for n in self.losses}


def create_loss_aggregator(config: Optional[LossConfig] = None) -> LossAggregator:
    return LossAggregator(config or LossConfig())


def create_default_loss_config() -> LossConfig:
    return LossConfig(enabled_losses=[LossType.LATENT_MSE, LossType.AUTOREGRESSIVE_NEXT_FRAME,
                                      LossType.TEMPORAL_CONSISTENCY, LossType.CONDITIONAL_FLOW_MATCHING])


def create_full_loss_config() -> LossConfig:
    return LossConfig(enabled_losses=list(LossType), use_uncertainty_weighting=True,
                      use_gradient_normalization=True, use_gradient_surgery=True)


def create_minimal_loss_config() -> LossConfig:
    return LossConfig(enabled_losses=[LossType.LATENT_MSE, LossType.TEMPORAL_CONSISTENCY], enable_curriculum=False)


class UnifiedLoss:
    """v1-compatible interface on top of the aggregator: ``loss(predictions, targets,
    step)`` -> dict with ``total``."""

    def __init__(self, training_config=None, config: Optional[LossConfig] = None):
        self.config = training_config
        self.aggregator = LossAggregator(config or create_default_loss_config())
        self.step = 0

    def __call__(self, predictions, targets, step: Optional[int] = None):
        if step is not None:
            self.step = step
        return self.aggregator(predictions, targets, step=self.step)

    def get_loss_stats(self):
        return self.aggregator.get_loss_stats()
