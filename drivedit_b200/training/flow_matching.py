"""Rectified-flow / flow-matching objective and samplers.

Convention (reference ``blocks/flow_matching.py``): ``x_t = (1 - t) x0 + t x1`` with
``x0`` noise and ``x1`` data (:457), velocity target ``x1 - x0`` (:342), Euler
integration from t = 0 to 1 (:253-276) with optional classifier-free guidance
(:228-281). Time sampling: ``uniform`` (the reference, :454) or ``logit_normal``
(``sigmoid(N(m, s))``, the world-model presets).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn.functional as F


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


class RectifiedFlowSampler:
    """Euler sampler ``x += dt * v(x, t)`` from noise at t=0 to data at t=1."""

    def __init__(self, num_steps: int = 4, cfg_scale: float = 1.0):
        self.num_steps = num_steps
        self.cfg_scale = cfg_scale

    def timesteps(self, device=None) -> torch.Tensor:
        return torch.linspace(0.0, 1.0, self.num_steps + 1, device=device)

    @torch.no_grad()
    def sample(self, velocity_fn: Callable, x0: torch.Tensor,
               uncond_fn: Optional[Callable] = None) -> torch.Tensor:
        x = x0
        ts = self.timesteps(x0.device)
        for i in range(self.num_steps):
            t, dt = ts[i], ts[i + 1] - ts[i]
            v = velocity_fn(x, t)
            if uncond_fn is not None and self.cfg_scale != 1.0:
                vu = uncond_fn(x, t)
                v = vu + self.cfg_scale * (v - vu)
            x = x + dt * v
        return x

    @torch.no_grad()
    def ddim_sample(self, velocity_fn: Callable, z_init: torch.Tensor,
                    num_steps: Optional[int] = None, eta: float = 0.0,
                    t_start: float = 1.0, t_end: float = 0.0,
                    generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """DDIM-style sampler in the flow-matching parameterisation (reference
        ``RectifiedFlowSampler.ddim_sample``, blocks/flow_matching.py:283-314, whose
        schedule runs t from 1 to 0 by default).

        At each step the velocity gives both endpoint estimates, ``x1 = x + (1 - t) v``
        (data) and ``x0 = x - t v`` (noise), and the state moves to the next time on the
        straight path between them. With ``eta = 0`` that equals an Euler step of the
        ODE. With ``eta > 0`` the noise estimate is partly replaced by fresh Gaussian
        noise, ``x0 <- sqrt(1 - eta^2) x0 + eta * eps``, which keeps its variance (the
        stochastic DDIM family of Song et al. 2021)."""
        n = num_steps or self.num_steps
        ts = torch.linspace(t_start, t_end, n + 1, device=z_init.device, dtype=torch.float64)
        x = z_init
        for i in range(n):
            t, t_next = float(ts[i]), float(ts[i + 1])
            v = velocity_fn(x, ts[i].to(z_init.dtype))
            x1_hat = x + (1.0 - t) * v
            x0_hat = x - t * v
            if eta > 0.0:
                eps = torch.randn(x.shape, device=x.device, dtype=x.dtype, generator=generator)
                x0_hat = (1.0 - eta * eta) ** 0.5 * x0_hat + eta * eps
            x = (1.0 - t_next) * x0_hat + t_next * x1_hat
        return x


class FlowMatchingLoss(torch.nn.Module):
    """Velocity MSE plus the reference's distillation target ``(z_{t+dt} - z_t)/dt``
    (blocks/flow_matching.py:356-388)."""

    def forward(self, v_pred, x0, x1):
        return flow_matching_loss(v_pred, x0, x1)

    @staticmethod
    def distillation_target(z_t: torch.Tensor, z_next: torch.Tensor, dt: float) -> torch.Tensor:
        return (z_next - z_t) / dt
