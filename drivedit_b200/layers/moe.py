"""DeepSeek-style Mixture-of-Experts FFN: routed SwiGLU experts + softmax-gated shared
experts, aux-loss-free bias balancing and an (optional) Switch-style aux loss.

Semantics follow the reference's ``layers/moe.py``:
  * ``Router`` (:73-228): ``logits = x W_g^T (+ jitter) + expert_bias``,
    ``p = softmax(logits)``, top-k of ``p``, renormalised over the k; in training the
    per-expert counts update an EMA load and ``expert_bias -= speed * (load_ema - 1/E)``
    (:164-181); metrics include ``E * sum(f * P)`` (:196-199).
  * ``MoEFFN`` (:231-424): default expert width ``4d/top_k`` rounded up to 8 (:273-275);
    shared experts gated by ``softmax(x W_shared^T)`` (:400-413).
  * ``MoEDiTBlock`` (:427-547): pre-norm attention + MoE FFN.

Differences:
  * routed-expert weights are stacked (``w_gate/w_value [E, F, d]``, ``w_out [E, d, F]``)
    so the grouped GEMM reads one tensor per projection; ``load_state_dict`` accepts the
    reference's per-expert keys ``experts.N.{w_gate,w_value,w_out}.weight`` and
    :meth:`MoEFFN.reference_state_dict` writes them back.
  * the aux load-balance loss ``E * sum_e f_e P_e`` (f = share of the N*k assignments,
    P = mean router probability) is returned for the objective (weight configurable);
    the reference only logs it.
  * with ``ep_group`` set, only this rank's ``E / ep`` experts live here and tokens are
    exchanged by the expert-parallel dispatch/combine in ``drivedit_b200.parallel.ep``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class MoEMetrics:
    expert_counts: torch.Tensor
    expert_probs: torch.Tensor
    load_balance_loss: float
    expert_utilization: float
    max_load_ratio: float
    entropy: float
    avg_expert_confidence: float
    routing_sparsity: float


@dataclass
class MoEOutput:
    output: torch.Tensor
    aux_loss: Optional[torch.Tensor] = None
    metrics: Optional[MoEMetrics] = None


def default_expert_dim(d_model: int, top_k: int) -> int:
    e = int(4 * d_model / top_k)
    return ((e + 7) // 8) * 8


class Router(nn.Module):
    def __init__(self, d_model: int, num_experts: int, top_k: int = 2,
                 jitter_noise: float = 0.0, bias_update_speed: float = 0.001):
        super().__init__()
        self.num_experts, self.top_k = num_experts, top_k
        self.jitter_noise, self.bias_update_speed = jitter_noise, bias_update_speed
        self.gate = nn.Linear(d_model, num_experts, bias=False)
        nn.init.normal_(self.gate.weight, std=0.02)
        self.register_buffer("expert_bias", torch.zeros(num_experts))
        self.register_buffer("expert_load_ema", torch.ones(num_experts) / num_experts)

    def probs(self, x: torch.Tensor) -> torch.Tensor:
        logits = self.gate(x).float()
        if self.training and self.jitter_noise > 0:
            logits = logits + torch.randn_like(logits) * self.jitter_noise
        return F.softmax(logits + self.expert_bias, dim=-1)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Returns (weights [N,k] fp32, experts [N,k] int64, probs [N,E] fp32)."""
        p = self.probs(x)
        w, e = torch.topk(p, self.top_k, dim=-1)
        w = w / (w.sum(-1, keepdim=True) + 1e-8)
        return w, e, p

    @torch.no_grad()
    def update_bias(self, counts: torch.Tensor, n_tokens: int):
        """Aux-loss-free balancing step from this step's expert counts."""
        if not self.training:
            return
        load = counts.float() / (n_tokens * self.top_k + 1e-8)
        self.expert_load_ema.mul_(1 - self.bias_update_speed).add_(load, alpha=self.bias_update_speed)
        self.expert_bias.add_(-self.bias_update_speed * (self.expert_load_ema - 1.0 / self.num_experts))


def aux_load_balance_loss(probs: torch.Tensor, experts: torch.Tensor, num_experts: int):
    """Switch-style ``E * sum_e f_e * P_e``; equals 1 for perfectly uniform routing."""
    N, k = experts.shape
    counts = torch.bincount(experts.reshape(-1), minlength=num_experts).float()
    f = counts / (N * k)
    P = probs.mean(0)
    return num_experts * (f * P).sum(), counts


def routing_metrics(probs, weights, experts, counts, num_experts) -> MoEMetrics:
    mean = counts.float().mean()
    lb = num_experts * ((counts.float() / max(experts.shape[0], 1)) * probs.mean(0)).sum()
    return MoEMetrics(
        expert_counts=counts,
        expert_probs=probs.mean(0),
        load_balance_loss=float(lb),
        expert_utilization=float((counts > 0).float().mean()),
        max_load_ratio=float(counts.float().max() / (mean + 1e-8)),
        entropy=float(-(probs * (probs + 1e-8).log()).sum(-1).mean()),
        avg_expert_confidence=float(weights[:, 0].mean()),
        routing_sparsity=float((probs < 1e-3).float().mean()),
    )


class ExpertFFN(nn.Module):
    """One SwiGLU expert (reference names ``w_gate``, ``w_value``, ``w_out``)."""

    def __init__(self, d_model: int, d_expert: int, bias: bool = False):
        super().__init__()
        self.w_gate = nn.Linear(d_model, d_expert, bias=bias)
        self.w_value = nn.Linear(d_model, d_expert, bias=bias)
        self.w_out = nn.Linear(d_expert, d_model, bias=bias)
        nn.init.normal_(self.w_gate.weight, std=0.02)
        nn.init.normal_(self.w_value.weight, std=0.02)
        nn.init.normal_(self.w_out.weight, std=0.02 / math.sqrt(2))

    def forward(self, x):
        return self.w_out(F.silu(self.w_gate(x)) * self.w_value(x))


class MoEFFN(nn.Module):
    def __init__(self, d_model: int, num_experts: int = 8, top_k: int = 2,
                 expert_dim: Optional[int] = None, num_shared_experts: int = 0,
                 dropout: float = 0.0, bias: bool = False, jitter_noise: float = 0.0,
                 bias_update_speed: float = 0.001, aux_loss_weight: float = 0.0,
                 expert_range: Optional[Tuple[int, int]] = None):
        super().__init__()
        assert not bias, "routed experts are bias-free"
        self.d_model, self.num_experts, self.top_k = d_model, num_experts, top_k
        self.expert_dim = expert_dim or default_expert_dim(d_model, top_k)
        self.num_shared_experts = num_shared_experts
        self.aux_loss_weight = aux_loss_weight
        self.expert_range = expert_range or (0, num_experts)
        e_local = self.expert_range[1] - self.expert_range[0]
        Fh = self.expert_dim
        self.router = Router(d_model, num_experts, top_k, jitter_noise, bias_update_speed)
        self.w_gate = nn.Parameter(torch.randn(e_local, Fh, d_model) * 0.02)
        self.w_value = nn.Parameter(torch.randn(e_local, Fh, d_model) * 0.02)
        self.w_out = nn.Parameter(torch.randn(e_local, d_model, Fh) * (0.02 / math.sqrt(2)))
        if num_shared_experts > 0:
            self.shared_experts = nn.ModuleList(
                [ExpertFFN(d_model, Fh) for _ in range(num_shared_experts)])
            self.shared_gate = nn.Linear(d_model, num_shared_experts, bias=False)
        else:
            self.shared_experts = None
            self.shared_gate = None
        self._register_load_state_dict_pre_hook(self._load_reference_keys)

    # -------------------------------------------------------------- checkpoint compat
    def _load_reference_keys(self, state_dict, prefix, *args):
        key0 = prefix + "experts.0.w_gate.weight"
        if key0 not in state_dict:
            return
        lo, hi = self.expert_range
        for name in ("w_gate", "w_value", "w_out"):
            ws = [state_dict.pop(f"{prefix}experts.{e}.{name}.weight")
                  for e in range(self.num_experts)
                  if f"{prefix}experts.{e}.{name}.weight" in state_dict]
            state_dict[prefix + name] = torch.stack(ws[lo:hi]) if len(ws) == self.num_experts else torch.stack(ws)

    def reference_state_dict(self, prefix: str = "") -> Dict[str, torch.Tensor]:
        """Per-expert keys in the reference's layout (``experts.N.w_gate.weight`` ...)."""
        out = {}
        lo, _ = self.expert_range
        for name in ("w_gate", "w_value", "w_out"):
            w = getattr(self, name).detach()
            for i in range(w.shape[0]):
                out[f"{prefix}experts.{lo + i}.{name}.weight"] = w[i].clone()
        for k, v in self.state_dict().items():
            if k.split(".")[0] not in ("w_gate", "w_value", "w_out"):
                out[prefix + k] = v
        return out

    # -------------------------------------------------------------- compute
    def experts_forward(self, x: torch.Tensor, weights: torch.Tensor, experts: torch.Tensor):
        """Reference-math routed output (stable sort by expert, loop over experts)."""
        N, D = x.shape
        out = torch.zeros(N, D, dtype=torch.float32, device=x.device)
        flat_e = experts.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        tok = order // self.top_k
        counts = torch.bincount(flat_e, minlength=self.num_experts)
        lo, hi = self.expert_range
        starts = torch.cumsum(counts, 0) - counts
        for e in range(lo, hi):
            c = int(counts[e])
            if c == 0:
                continue
            idx = order[int(starts[e]):int(starts[e]) + c]
            t = tok[int(starts[e]):int(starts[e]) + c]
            xe = x[t]
            i = e - lo
            h = F.silu(xe @ self.w_gate[i].t()) * (xe @ self.w_value[i].t())
            ye = (h @ self.w_out[i].t()).float()
            out.index_add_(0, t, ye * weights.reshape(-1)[idx, None].float())
        return out

    def shared_forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.shared_experts is None:
            return torch.zeros_like(x, dtype=torch.float32)
        g = F.softmax(self.shared_gate(x).float(), -1)
        out = 0
        for i, ex in enumerate(self.shared_experts):
            out = out + g[:, i:i + 1] * ex(x).float()
        return out

    def forward(self, x: torch.Tensor, return_metrics: bool = False) -> MoEOutput:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        w, e, p = self.router(xf)
        aux, counts = aux_load_balance_loss(p, e, self.num_experts)
        self.router.update_bias(counts, xf.shape[0])
        y = self.experts_forward(xf, w, e) + self.shared_forward(xf)
        metrics = routing_metrics(p, w, e, counts, self.num_experts) if return_metrics else None
        return MoEOutput(y.to(x.dtype).view(shape), aux * self.aux_loss_weight, metrics)

    def get_load_balance_stats(self) -> Dict[str, float]:
        r = self.router
        return {
            "load_ema_std": float(r.expert_load_ema.std()),
            "load_ema_max": float(r.expert_load_ema.max()),
            "load_ema_min": float(r.expert_load_ema.min()),
            "bias_std": float(r.expert_bias.std()),
            "bias_max": float(r.expert_bias.max()),
            "bias_min": float(r.expert_bias.min()),
        }
