"""Teacher -> student distillation for the latent world model (the reference's
``training/distill.py:33-598`` API: ``DistillationTrainer(teacher_model, student_model,
vae_model, optimizer, scheduler, device, use_wandb, distill_config)`` with
``train_epoch / validate / save_checkpoint / load_checkpoint`` and the loss terms
``flow_matching``, ``kl_divergence``, ``consistency`` and ``feature_matching``).

Both models are :class:`~drivedit_b200.models.world_dit.WorldDiT` velocity predictors on
latent video ``[B, T, C, H, W]``: the teacher bidirectional (``causal="none"``), the
student frame-causal. Per step, with ``x_t = (1 - t) x0 + t x1`` (noise ``x0``, data
``x1``):

* flow distillation (4 -> 1 step): the frozen teacher integrates ``flow_steps`` Euler steps
  from ``x_t`` to ``t = 1``; the student learns the single velocity
  ``(x1_teacher - x_t) / (1 - t)`` that lands on the teacher's endpoint;
* KL: per token, softmax over the patch channels of teacher and student velocities at
  ``temperature``; ``KL(teacher || student)``;
* consistency: the student's one-step endpoints from two points of the same teacher
  trajectory agree (the later one is the stop-gradient target);
* feature matching: MSE between the two models' hidden states at a middle layer (through a
  learned projection when the widths differ).

The reference constructs loss objects that do not exist (``FlowLoss(loss_type=...)``,
``ConsistencyTraining``; ``:79-83``) and never runs; this trainer does. When a VAE is given
and a batch carries RGB ``frames``, latents come from its frozen encoder; a batch may carry
``latents`` directly. ``use_wandb`` selects logging through the JSONL metrics sink (no network service).
"""
from __future__ import annotations

from collections import defaultdict
from typing import Dict, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F


_DEFAULTS = {"flow_steps": 4, "sigma_min": 0.002, "sigma_max": 80.0, "distill_weight": 1.0,
             "kl_weight": 0.1, "consistency_weight": 0.1, "feature_weight": 0.05, "guidance_scale": 1.0,
             "temperature": 1.0, "clip_grad_norm": 1.0, "feature_layer": None}


class DistillationTrainer:
    def __init__(self, teacher_model: nn.Module, student_model: nn.Module, vae_model: Optional[nn.Module],
                 optimizer: torch.optim.Optimizer, scheduler=None, device: str = "cuda",
                 use_wandb: bool = False, distill_config: Optional[Dict] = None, metrics_path: Optional[str] = None):
        self.teacher_model = teacher_model.eval()
        self.student_model = student_model
        self.vae_model = vae_model.eval() if vae_model is not None else None
        self.optimizer, self.scheduler = optimizer, scheduler
        self.device = torch.device(device)
        self.config = {**_DEFAULTS, **(distill_config or {})}
        for p in self.teacher_model.parameters():
            p.requires_grad_(False)
        if self.vae_model is not None:
            for p in self.vae_model.parameters():
                p.requires_grad_(False)
        ts, tt = student_model.cfg, teacher_model.cfg
        self.feature_layer_s = self.config["feature_layer"] or max(1, ts.n_layers // 2)
        self.feature_layer_t = max(1, round(self.feature_layer_s * tt.n_layers / ts.n_layers))
        self.feature_proj = (nn.Linear(ts.d_model, tt.d_model, bias=False).to(self.device)
                             if ts.d_model != tt.d_model else nn.Identity())
        if isinstance(self.feature_proj, nn.Linear):
            self.optimizer.add_param_group({"params": self.feature_proj.parameters()})
        self.metrics = None
        if use_wandb or metrics_path:
            from ..utils.observability import MetricsLogger

            self.metrics = MetricsLogger(metrics_path or "distill_logs")
        self.global_step = 0
        self.epoch = 0

    # ------------------------------------------------------------------ data
    @torch.no_grad()
    def _latents(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        if "latents" in batch:
            return batch["latents"].to(self.device).float()
        frames = batch["frames"].to(self.device)                 # [B, T, 3, H, W]
        if self.vae_model is None:
            raise ValueError("RGB frames need a VAE to encode them")
        enc = self.vae_model.encode(frames.permute(0, 2, 1, 3, 4))   # (mean, logvar)
        z = enc[0] if isinstance(enc, (tuple, list)) else enc        # the posterior mean
        return z.permute(0, 2, 1, 3, 4).float()

    def _actions(self, batch, B, T) -> torch.Tensor:
        A = self.student_model.cfg.action_dim
        a = batch.get("controls", batch.get("actions"))
        if a is None:
            return torch.zeros(B, T, A, device=self.device)
        a = a.to(self.device).float()[:, :T]
        return a[..., :A] if a.shape[-1] >= A else F.pad(a, (0, A - a.shape[-1]))

    # ------------------------------------------------------------------ losses
    @torch.no_grad()
    def _teacher_endpoint(self, x_t, t, actions, steps: int):
        """Euler integration of the teacher's velocity from ``t`` to 1."""
        x = x_t.float()
        tt = t.clone()
        dt = (1.0 - t) / steps
        for _ in range(steps):
            v = self.teacher_model(x.to(x_t.dtype), tt, actions).float()
            x = x + dt.view(-1, 1, 1, 1, 1) * v
            tt = tt + dt
        return x

    def _distillation_step(self, latents: torch.Tensor, actions: torch.Tensor) -> Dict[str, torch.Tensor]:
        c = self.config
        B = latents.shape[0]
        dtype = next(self.student_model.parameters()).dtype
        x1 = latents
        x0 = torch.randn_like(x1)
        t = torch.rand(B, device=self.device) * 0.9                 # keep 1 - t away from 0
        x_t = (1 - t.view(-1, 1, 1, 1, 1)) * x0 + t.view(-1, 1, 1, 1, 1) * x1
        with torch.no_grad():
            end_t = self._teacher_endpoint(x_t, t, actions, c["flow_steps"])
            v_target = (end_t - x_t) / (1 - t).view(-1, 1, 1, 1, 1)
            tv, _, tfeat = self.teacher_model(x_t.to(dtype), t, actions, return_aux=True,
                                              return_features=self.feature_layer_t)
        v_s, _, sfeat = self.student_model(x_t.to(dtype), t, actions, return_aux=True,
                                           return_features=self.feature_layer_s)
        v_s = v_s.float()
        losses = {"flow_matching": F.mse_loss(v_s, v_target)}
        # KL over each token's channels (patch channels of the velocity field)
        T_ = c["temperature"]
        ls = F.log_softmax(v_s.flatten(3) / T_, dim=2)
        lt = F.log_softmax(tv.float().flatten(3) / T_, dim=2)
        losses["kl_divergence"] = (lt.exp() * (lt - ls)).sum(2).mean()
        # consistency: endpoint from a later point of the teacher trajectory
        if c["consistency_weight"] > 0:
            with torch.no_grad():
                s = t + (1 - t) * 0.5
                x_s = x_t + (s - t).view(-1, 1, 1, 1, 1) * v_target
                v_late = self.student_model(x_s.to(dtype), s, actions).float()
                end_late = x_s + (1 - s).view(-1, 1, 1, 1, 1) * v_late
            end_early = x_t + (1 - t).view(-1, 1, 1, 1, 1) * v_s
            losses["consistency"] = F.mse_loss(end_early, end_late)
        if c["feature_weight"] > 0:
            losses["feature_matching"] = F.mse_loss(self.feature_proj(sfeat.float()), tfeat.float())
        return losses

    def _compute_total_loss(self, losses: Dict[str, torch.Tensor]) -> torch.Tensor:
        c = self.config
        w = {"flow_matching": c["distill_weight"], "kl_divergence": c["kl_weight"],
             "consistency": c["consistency_weight"], "feature_matching": c["feature_weight"]}
        return sum(w.get(k, 1.0) * v for k, v in losses.items())

    # ------------------------------------------------------------------ loops
    def train_step(self, batch: Dict[str, torch.Tensor]) -> Dict[str, float]:
        self.student_model.train()
        lat = self._latents(batch)
        act = self._actions(batch, lat.shape[0], lat.shape[1])
        losses = self._distillation_step(lat, act)
        total = self._compute_total_loss(losses)
        self.optimizer.zero_grad(set_to_none=True)
        total.backward()
        if self.config["clip_grad_norm"] > 0:
            torch.nn.utils.clip_grad_norm_(self.student_model.parameters(), self.config["clip_grad_norm"])
        self.optimizer.step()
        if self.scheduler is not None:
            self.scheduler.step()
        self.global_step += 1
        out = {k: float(v.detach()) for k, v in losses.items()}
        out["total"] = float(total.detach())
        if self.metrics is not None and self.global_step % 100 == 0:
            self.metrics.log(self.global_step, out, aggregate=False)
        return out

    def train_epoch(self, dataloader) -> Dict[str, float]:
        acc = defaultdict(list)
        for batch in dataloader:
            for k, v in self.train_step(batch).items():
                acc[k].append(v)
        self.epoch += 1
        return {k: float(np.mean(v)) for k, v in acc.items()}

    @torch.no_grad()
    def validate(self, val_dataloader) -> Dict[str, float]:
        """Student one-step endpoint error against the teacher's multi-step endpoint."""
        self.student_model.eval()
        errs = []
        for batch in val_dataloader:
            lat = self._latents(batch)
            B = lat.shape[0]
            act = self._actions(batch, B, lat.shape[1])
            x0 = torch.randn_like(lat)
            t = torch.zeros(B, device=self.device)
            end_t = self._teacher_endpoint(x0, t, act, self.config["flow_steps"])
            dtype = next(self.student_model.parameters()).dtype
            end_s = x0 + self.student_model(x0.to(dtype), t, act).float()
            errs.append(float(F.mse_loss(end_s, end_t)))
        self.student_model.train()
        return {"one_step_endpoint_mse": float(np.mean(errs)) if errs else float("nan")}

    def save_checkpoint(self, filepath: str, best_metric: Optional[float] = None):
        from .distributed import _atomic_save

        from pathlib import Path

        _atomic_save({"student": self.student_model.state_dict(), "optimizer": self.optimizer.state_dict(),
                      "scheduler": self.scheduler.state_dict() if self.scheduler is not None else None,
                      "feature_proj": self.feature_proj.state_dict(), "global_step": self.global_step,
                      "epoch": self.epoch, "best_metric": best_metric, "config": self.config}, Path(filepath))

    def load_checkpoint(self, filepath: str):
        from pathlib import Path

        from .distributed import _verified_load

        ck = _verified_load(Path(filepath))
        self.student_model.load_state_dict(ck["student"])
        self.optimizer.load_state_dict(ck["optimizer"])
        if self.scheduler is not None and ck.get("scheduler") is not None:
            self.scheduler.load_state_dict(ck["scheduler"])
        self.feature_proj.load_state_dict(ck["feature_proj"])
        self.global_step, self.epoch = ck["global_step"], ck["epoch"]
        return ck.get("best_metric")
