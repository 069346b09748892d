"""Rectified-flow / flow-matching objective and samplers.

Convention (reference ``blocks/flow_matching.py``): ``x_t = (1 - t) x0 + t x1`` with
``x0`` noise and ``x1`` data (:457), velocity target ``x1 - x0`` (:342), Euler
integration from t = 0 to 1 (:253-276) with optional classifier-free guidance
(:228-281). Time sampling: ``uniform`` (the reference, :454) or ``logit_normal``
(``sigmoid(N(m, s))``, the world-model presets).
"""
from __future__ import annotations

from typing import Callable, Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..models.blocks import FlowMatchingBlock, FlowMatchingConfig, FlowPredictor  # noqa: F401
from ..models.blocks import FlowTimestepEmbedding as TimestepEmbedding  # noqa: F401


def sample_t(n: int, mode: str = "logit_normal", device=None, generator=None,
             mean: float = 0.0, std: float = 1.0) -> torch.Tensor:
    if mode == "uniform":
        return torch.rand(n, device=device, generator=generator)
    if mode == "logit_normal":
        return torch.sigmoid(torch.randn(n, device=device, generator=generator) * std + mean)
    raise ValueError(f"unknown t sampling {mode!r}")


def _bcast(t: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    while t.dim() < x.dim():
        t = t[..., None]
    return t


def interpolate(x0: torch.Tensor, x1: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
    tb = _bcast(t.to(x1.dtype), x1)
    return (1 - tb) * x0 + tb * x1


def velocity_target(x0: torch.Tensor, x1: torch.Tensor) -> torch.Tensor:
    return x1 - x0


def flow_matching_loss(v_pred: torch.Tensor, x0: torch.Tensor, x1: torch.Tensor) -> torch.Tensor:
    return F.mse_loss(v_pred.float(), (x1 - x0).float())


def euler_sample(velocity_fn: Callable, x0: torch.Tensor, num_steps: int = 4,
                 cfg_scale: float = 1.0, uncond_fn: Optional[Callable] = None,
                 return_trajectory: bool = False):
    """Euler integration ``x += dt * v(x, t)`` from t = 0 to 1 over ``num_steps`` equal
    steps; with ``uncond_fn`` and ``cfg_scale != 1`` the velocity is the classifier-free
    guided ``vu + cfg_scale * (v - vu)``. With ``return_trajectory`` also the stacked
    states ``[num_steps + 1, ...]``."""
    ts = torch.linspace(0.0, 1.0, num_steps + 1, device=x0.device)
    x = x0
    traj = [x0] if return_trajectory else None
    for i in range(num_steps):
        t, dt = ts[i], ts[i + 1] - ts[i]
        v = velocity_fn(x, t)
        if uncond_fn is not None and cfg_scale != 1.0:
            vu = uncond_fn(x, t)
            v = vu + cfg_scale * (v - vu)
        x = x + dt * v
        if traj is not None:
            traj.append(x)
    return (x, torch.stack(traj, 0)) if return_trajectory else x


def ddim_sample(velocity_fn: Callable, z_init: torch.Tensor, num_steps: int = 4,
                eta: float = 0.0, t_start: float = 1.0, t_end: float = 0.0,
                generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """DDIM-style sampler in the flow-matching parameterisation (the reference's
    ``RectifiedFlowSampler.ddim_sample``, blocks/flow_matching.py:283-314, runs t from
    1 to 0 by default).

    At each step the velocity gives both endpoint estimates, ``x1 = x + (1 - t) v``
    (data) and ``x0 = x - t v`` (noise), and the state moves to the next time on the
    straight path between them. With ``eta = 0`` that equals an Euler step of the ODE.
    With ``eta > 0`` the noise estimate is partly replaced by fresh Gaussian noise,
    ``x0 <- sqrt(1 - eta^2) x0 + eta * eps``, which keeps its variance (the stochastic
    DDIM family of Song et al. 2021)."""
    ts = torch.linspace(t_start, t_end, num_steps + 1, device=z_init.device, dtype=torch.float64)
    x = z_init
    for i in range(num_steps):
        t, t_next = float(ts[i]), float(ts[i + 1])
        v = velocity_fn(x, ts[i].to(z_init.dtype))
        x1_hat = x + (1.0 - t) * v
        x0_hat = x - t * v
        if eta > 0.0:
            eps = torch.randn(x.shape, device=x.device, dtype=x.dtype, generator=generator)
            x0_hat = (1.0 - eta * eta) ** 0.5 * x0_hat + eta * eps
        x = (1.0 - t_next) * x0_hat + t_next * x1_hat
    return x


def _masked_mean(err: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    """Mean of ``err [B, T, D]``; with a token mask ``[B, T]`` the sum over the kept
    tokens divided by their count (the reference's convention, not also by D)."""
    if mask is None:
        return err.mean()
    return (err * mask[..., None]).sum() / mask.sum()


class RectifiedFlowSampler:
    """Generation with a flow predictor ``v(z, t, mask, context)`` (the reference's
    sampler API, blocks/flow_matching.py:221-314): :meth:`sample` integrates with Euler
    steps from noise at t = 0 and returns the trajectory and the final sample,
    :meth:`ddim_sample` runs the DDIM-style schedule (t from 1 to 0 by default)."""

    def __init__(self, flow_predictor: Callable, config: Optional[FlowMatchingConfig] = None):
        self.flow_predictor = flow_predictor
        self.config = config or FlowMatchingConfig()

    def _velocity(self, context, mask):
        def v(z, t):
            return self.flow_predictor(z, t.expand(z.shape[0]), mask, context)
        return v

    @torch.no_grad()
    def sample(self, z_init: torch.Tensor, num_steps: Optional[int] = None,
               context: Optional[torch.Tensor] = None, guidance_scale: float = 1.0,
               mask: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        """``{'trajectory': [num_steps + 1, *z_init.shape], 'final_sample'}``. Guidance
        (``guidance_scale > 1`` with a context) mixes the conditional velocity with the
        one predicted without context."""
        n = num_steps or self.config.num_steps
        guided = guidance_scale > 1.0 and context is not None
        final, traj = euler_sample(self._velocity(context, mask), z_init, n,
                                   guidance_scale if guided else 1.0,
                                   self._velocity(None, mask) if guided else None,
                                   return_trajectory=True)
        return {"trajectory": traj, "final_sample": final}

    @torch.no_grad()
    def ddim_sample(self, z_init: torch.Tensor, num_steps: Optional[int] = None,
                    context: Optional[torch.Tensor] = None, eta: float = 0.0,
                    mask: Optional[torch.Tensor] = None, t_start: float = 1.0,
                    t_end: float = 0.0, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        return ddim_sample(self._velocity(context, mask), z_init, num_steps or self.config.num_steps,
                           eta, t_start, t_end, generator)


class FlowMatchingLoss:
    """Losses of flow-matching training (blocks/flow_matching.py:317-412): velocity MSE
    against ``z_1 - z_0``, distillation of a teacher's first Euler step, and consistency
    of the prediction under a small step along it (given a predictor)."""

    def __init__(self, config: Optional[FlowMatchingConfig] = None,
                 flow_predictor: Optional[Callable] = None):
        self.config = config or FlowMatchingConfig()
        self.flow_predictor = flow_predictor

    def __call__(self, v_pred, x0, x1):
        return flow_matching_loss(v_pred, x0, x1)

    def flow_matching_loss(self, flow_pred, z_0, z_1, t=None, mask=None) -> torch.Tensor:
        return _masked_mean((flow_pred - (z_1 - z_0)).pow(2), mask)

    @staticmethod
    def distillation_target(z_t: torch.Tensor, z_next: torch.Tensor, dt: float) -> torch.Tensor:
        return (z_next - z_t) / dt

    def distillation_loss(self, student_flow, teacher_trajectory, dt: float, mask=None) -> torch.Tensor:
        """``teacher_trajectory [steps + 1, B, T, D]``: the student's velocity against the
        teacher's first step ``(z_1 - z_0) / dt``."""
        target = self.distillation_target(teacher_trajectory[0], teacher_trajectory[1], dt)
        return _masked_mean((student_flow - target).pow(2), mask)

    def consistency_loss(self, flow_pred, z_t, t, dt: float = 0.01,
                         flow_predictor: Optional[Callable] = None) -> torch.Tensor:
        fp = flow_predictor or self.flow_predictor
        if fp is None:
            raise ValueError("consistency_loss needs a flow predictor")
        with torch.no_grad():
            z_next = z_t + dt * flow_pred
        return F.mse_loss(flow_pred, fp(z_next, (t + dt).clamp(0, 1)))


class FlowMatchingTrainer:
    """Plain training loop for a :class:`~drivedit_b200.models.blocks.FlowPredictor`
    with any torch optimizer (blocks/flow_matching.py:415-572): flow-matching steps (a
    consistency term every 10th step), teacher-to-student distillation of the first Euler
    step, and sampling with quality figures. The fused world-model trainer is
    :class:`drivedit_b200.training.trainer.WorldModelTrainer`."""

    consistency_every = 10
    consistency_weight = 0.1
    consistency_dt = 0.01
    clip_norm = 1.0

    def __init__(self, flow_predictor: nn.Module, config: Optional[FlowMatchingConfig] = None):
        self.flow_predictor = flow_predictor
        self.config = config or getattr(flow_predictor, "config", None) or FlowMatchingConfig()
        self.loss_fn = FlowMatchingLoss(self.config, flow_predictor)
        self.sampler = RectifiedFlowSampler(flow_predictor, self.config)

    def _device(self):
        return next(self.flow_predictor.parameters()).device

    def _update(self, loss, optimizer):
        optimizer.zero_grad()
        loss.backward()
        torch.nn.utils.clip_grad_norm_(self.flow_predictor.parameters(), self.clip_norm)
        optimizer.step()

    def train_step(self, batch: Dict[str, torch.Tensor], optimizer, step: int) -> Dict[str, float]:
        """``batch``: ``latents [B, T, D]`` (data), optional ``context``, ``mask``."""
        z1 = batch["latents"].to(self._device())
        context, mask = batch.get("context"), batch.get("mask")
        z0 = torch.randn_like(z1)
        t = torch.rand(z1.shape[0], device=z1.device)
        zt = interpolate(z0, z1, t)
        pred = self.flow_predictor(zt, t, None, context)
        losses = {"flow_matching": self.loss_fn.flow_matching_loss(pred, z0, z1, t, mask)}
        if step % self.consistency_every == 0:
            dt = self.consistency_dt
            with torch.no_grad():
                z_next = zt + dt * pred.detach()
            nxt = self.flow_predictor(z_next, (t + dt).clamp(0, 1), None, context)
            losses["consistency"] = self.consistency_weight * F.mse_loss(pred, nxt)
        self._update(sum(losses.values()), optimizer)
        return {k: float(v.detach()) for k, v in losses.items()}

    def distillation_step(self, teacher_predictor: nn.Module, batch: Dict[str, torch.Tensor],
                          optimizer) -> Dict[str, float]:
        """The student's velocity at t = 0 learns the teacher's first Euler step of a
        ``teacher_steps`` trajectory from the same noise."""
        z1 = batch["latents"].to(self._device())
        context, mask = batch.get("context"), batch.get("mask")
        z0 = torch.randn_like(z1)
        traj = RectifiedFlowSampler(teacher_predictor, self.config).sample(
            z0, self.config.teacher_steps, context)["trajectory"]
        student = self.flow_predictor(z0, torch.zeros(z1.shape[0], device=z1.device), None, context)
        loss = self.loss_fn.distillation_loss(student, traj, 1.0 / self.config.teacher_steps, mask)
        self._update(loss, optimizer)
        return {"distillation": float(loss.detach())}

    @torch.no_grad()
    def sample_and_evaluate(self, batch: Dict[str, torch.Tensor],
                            num_steps: Optional[int] = None) -> Dict[str, object]:
        z1 = batch["latents"].to(self._device())
        gen = self.sampler.sample(torch.randn_like(z1), num_steps or self.config.num_steps,
                                  batch.get("context"))["final_sample"]
        B = z1.shape[0]
        return {"generated_samples": gen,
                "mse": float(F.mse_loss(gen, z1)),
                "cosine_similarity": float(F.cosine_similarity(gen.reshape(B, -1),
                                                               z1.reshape(B, -1), dim=-1).mean())}


def create_flow_matching_components(config: FlowMatchingConfig):
    """``(FlowPredictor(config), FlowMatchingTrainer)`` (blocks/flow_matching.py:575-582)."""
    predictor = FlowPredictor(config)
    return predictor, FlowMatchingTrainer(predictor, config)
