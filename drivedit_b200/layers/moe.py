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
  * expert weights are stacked in the kernel layout (``w13 [E + ns, 2F, d]`` with gate and
    value rows interleaved by 32, ``w2 [E + ns, d, F]``, shared experts last) so the
    grouped GEMMs read one tensor per projection; ``load_state_dict`` accepts the
    reference's per-expert keys ``experts.N.{w_gate,w_value,w_out}.weight``,
    ``shared_experts.N.*``, ``router.gate.weight``, ``shared_gate.weight`` and
    :meth:`MoEFFN.reference_state_dict` writes them back.
  * the aux load-balance loss ``E * sum_e f_e P_e`` (f = share of the N*k assignments,
    P = mean router probability) is returned for the objective (weight configurable);
    the reference only logs it.
  * on CUDA the whole FFN runs as routing / dispatch / grouped-GEMM / combine kernels
    (:mod:`drivedit_b200.ops.moe`); shared experts are routed to every token with their
    softmax gate and share that path.
  * expert parallelism (:meth:`MoEFFN.shard_experts`, :mod:`drivedit_b200.parallel.expert`):
    each rank keeps its ``E / world`` routed experts in ``w13 / w2`` and the replicated
    shared experts in ``w13_shared / w2_shared``; tokens travel to their expert's rank
    and back. The reference has no expert parallelism.
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
    probs, weights = probs.detach(), weights.detach()
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

    def __init__(self, d_model: int, d_expert: int, dropout: float = 0.0, bias: bool = False):
        super().__init__()
        self.w_gate = nn.Linear(d_model, d_expert, bias=bias)
        self.w_value = nn.Linear(d_model, d_expert, bias=bias)
        self.w_out = nn.Linear(d_expert, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        nn.init.normal_(self.w_gate.weight, std=0.02)
        nn.init.normal_(self.w_value.weight, std=0.02)
        nn.init.normal_(self.w_out.weight, std=0.02 / math.sqrt(2))

    def forward(self, x):
        return self.w_out(self.dropout(F.silu(self.w_gate(x)) * self.w_value(x)))


class MoEFFN(nn.Module):
    """Routed + shared SwiGLU experts in the kernel layout.

    Parameters: ``router_weight [Epad, d]`` — rows ``[0, E)`` are the router gate, rows
    ``[E, E + ns)`` the shared-expert gate, the rest zero padding to a multiple of 32;
    ``w13 [E + ns, 2F, d]`` — each expert's gate and value rows interleaved in groups of
    32 (``layers/mlp.py: pack_swiglu``), shared experts last; ``w2 [E + ns, d, F]``.
    """

    def __init__(self, d_model: int, num_experts: int = 8, top_k: int = 2,
                 expert_dim: Optional[int] = None, num_shared_experts: int = 0,
                 dropout: float = 0.0, bias: bool = False, jitter_noise: float = 0.0,
                 bias_update_speed: float = 0.001, aux_loss_weight: float = 0.0):
        super().__init__()
        assert not bias, "experts are bias-free"
        from .mlp import pack_swiglu

        self.d_model, self.num_experts, self.top_k = d_model, num_experts, top_k
        self.expert_dim = expert_dim or default_expert_dim(d_model, top_k)
        self.num_shared_experts = num_shared_experts
        self.aux_loss_weight = aux_loss_weight
        self.jitter_noise, self.bias_update_speed = jitter_noise, bias_update_speed
        E, ns, Fh = num_experts, num_shared_experts, self.expert_dim
        self.n_total = E + ns
        self.e_pad = ((E + ns + 31) // 32) * 32
        rw = torch.zeros(self.e_pad, d_model)
        rw[:E + ns].normal_(0, 0.02)
        self.router_weight = nn.Parameter(rw)
        self.register_buffer("expert_bias", torch.zeros(E))
        self.register_buffer("expert_load_ema", torch.ones(E) / E)
        wg = torch.randn(E + ns, Fh, d_model) * 0.02
        wv = torch.randn(E + ns, Fh, d_model) * 0.02
        self.w13 = nn.Parameter(torch.stack([pack_swiglu(wg[i], wv[i]) for i in range(E + ns)]))
        self.w2 = nn.Parameter(torch.randn(E + ns, d_model, Fh) * (0.02 / math.sqrt(2)))
        self.ep = None          # ExpertParallel context once the experts are sharded
        self.ep_slot = -1       # this layer's index among the EP layers (return-buffer slot)
        self._register_load_state_dict_pre_hook(self._load_reference_keys)

    # -------------------------------------------------------------- expert parallelism
    def shard_experts(self, ep) -> None:
        """Keep only this rank's routed experts (``ep.local_range()``) in ``w13 / w2``
        and move the shared experts to ``w13_shared / w2_shared``. Every rank must hold
        identical full weights when this is called (same seed or a loaded checkpoint)."""
        assert self.ep is None, "experts already sharded"
        assert ep.num_experts == self.num_experts
        lo, hi = ep.local_range()
        E, ns = self.num_experts, self.num_shared_experts
        with torch.no_grad():
            w13, w2 = self.w13.detach(), self.w2.detach()
            self.w13 = nn.Parameter(w13[lo:hi].clone())
            self.w2 = nn.Parameter(w2[lo:hi].clone())
            if ns:
                self.w13_shared = nn.Parameter(w13[E:E + ns].clone())
                self.w2_shared = nn.Parameter(w2[E:E + ns].clone())
        self.ep = ep
        self.ep_slot = ep.register(self)

    def expert_parameter_names(self, prefix: str = ""):
        """Names of the rank-local (not replicated) parameters under expert parallelism."""
        return [prefix + "w13", prefix + "w2"] if self.ep is not None else []

    # -------------------------------------------------------------- checkpoint compat
    def _load_reference_keys(self, state_dict, prefix, *args):
        from .mlp import pack_swiglu

        if prefix + "experts.0.w_gate.weight" not in state_dict:
            return
        assert self.ep is None, "load reference checkpoints before sharding the experts"
        E, ns = self.num_experts, self.num_shared_experts
        rw = self.router_weight.detach().clone()
        rw[:E] = state_dict.pop(prefix + "router.gate.weight")
        if ns:
            rw[E:E + ns] = state_dict.pop(prefix + "shared_gate.weight")
        state_dict[prefix + "router_weight"] = rw
        for b in ("expert_bias", "expert_load_ema"):
            if prefix + "router." + b in state_dict:
                state_dict[prefix + b] = state_dict.pop(prefix + "router." + b)
        w13, w2 = [], []
        for i in range(E + ns):
            base = f"{prefix}experts.{i}." if i < E else f"{prefix}shared_experts.{i - E}."
            g = state_dict.pop(base + "w_gate.weight")
            v = state_dict.pop(base + "w_value.weight")
            w13.append(pack_swiglu(g, v))
            w2.append(state_dict.pop(base + "w_out.weight"))
        state_dict[prefix + "w13"] = torch.stack(w13)
        state_dict[prefix + "w2"] = torch.stack(w2)

    def reference_state_dict(self, prefix: str = "") -> Dict[str, torch.Tensor]:
        """Per-expert keys in the reference's layout (``experts.N.w_gate.weight`` ...)."""
        from .mlp import unpack_swiglu

        assert self.ep is None, "reference export needs the full expert set (gather the shards first)"
        E, ns = self.num_experts, self.num_shared_experts
        out = {prefix + "router.gate.weight": self.router_weight[:E].detach().clone(),
               prefix + "router.expert_bias": self.expert_bias.clone(),
               prefix + "router.expert_load_ema": self.expert_load_ema.clone()}
        if ns:
            out[prefix + "shared_gate.weight"] = self.router_weight[E:E + ns].detach().clone()
        for i in range(E + ns):
            base = f"{prefix}experts.{i}." if i < E else f"{prefix}shared_experts.{i - E}."
            g, v = unpack_swiglu(self.w13[i].detach())
            out[base + "w_gate.weight"] = g.clone()
            out[base + "w_value.weight"] = v.clone()
            out[base + "w_out.weight"] = self.w2[i].detach().clone()
        return out

    # -------------------------------------------------------------- routing
    def route(self, x: torch.Tensor):
        """(weights [N,k], experts [N,k], probs [N,E], shared gates [N,ns])."""
        E, ns = self.num_experts, self.num_shared_experts
        logits = (x @ self.router_weight[:E + ns].to(x.dtype).t()).float()
        rl = logits[:, :E]
        if self.training and self.jitter_noise > 0:
            rl = rl + torch.randn_like(rl) * self.jitter_noise
        p = F.softmax(rl + self.expert_bias, dim=-1)
        w, e = torch.topk(p, self.top_k, dim=-1)
        w = w / (w.sum(-1, keepdim=True) + 1e-8)
        g = F.softmax(logits[:, E:E + ns], -1) if ns else None
        return w, e, p, g

    @torch.no_grad()
    def update_bias(self, counts: torch.Tensor, n_tokens: int):
        """Aux-loss-free balancing (reference layers/moe.py:164-181). The step's
        per-expert counts stay on the device in ``last_counts`` for monitoring."""
        self.last_counts = counts.detach()
        if not self.training or getattr(self, "frozen_bias", False):
            return
        s = self.bias_update_speed
        load = counts.float() / (n_tokens * self.top_k + 1e-8)
        self.expert_load_ema.mul_(1 - s).add_(load, alpha=s)
        self.expert_bias.add_(-s * (self.expert_load_ema - 1.0 / self.num_experts))

    def _expert(self, i: int, x: torch.Tensor) -> torch.Tensor:
        """Expert ``i`` of ``w13 / w2`` (under expert parallelism: local index)."""
        return self._swiglu(self.w13[i], self.w2[i], x)

    def _shared_expert(self, s: int, x: torch.Tensor) -> torch.Tensor:
        if self.ep is not None:
            return self._swiglu(self.w13_shared[s], self.w2_shared[s], x)
        return self._expert(self.num_experts + s, x)

    @staticmethod
    def _swiglu(w13, w2, x):
        from .mlp import split_gu

        g, u = split_gu(x @ w13.to(x.dtype).t())
        return (F.silu(g) * u) @ w2.to(x.dtype).t()

    def experts_forward(self, x, weights, experts):
        N, D = x.shape
        out = torch.zeros(N, D, dtype=torch.float32, device=x.device)
        flat_e = experts.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        counts = torch.bincount(flat_e, minlength=self.num_experts)
        starts = torch.cumsum(counts, 0) - counts
        for e in range(self.num_experts):
            c = int(counts[e])
            if c == 0:
                continue
            idx = order[int(starts[e]):int(starts[e]) + c]
            t = idx // self.top_k
            out.index_add_(0, t, self._expert(e, x[t]).float() * weights.reshape(-1)[idx, None].float())
        return out

    def shared_forward(self, x, gates):
        out = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
        for s in range(self.num_shared_experts):
            out = out + gates[:, s:s + 1] * self._shared_expert(s, x).float()
        return out

    def forward(self, x: torch.Tensor, return_metrics: bool = False) -> MoEOutput:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        w, e, p, g = self.route(xf)
        aux, counts = aux_load_balance_loss(p, e, self.num_experts)
        if self.ep is None:
            self.update_bias(counts, xf.shape[0])
            y = self.experts_forward(xf, w, e)
        else:
            from ..parallel.expert import ep_experts_forward_torch

            y, table = ep_experts_forward_torch(self, xf, w, e)
            # every rank applies the same bias update from the global counts
            gcounts = torch.as_tensor(table.sum(0), device=xf.device)
            self.update_bias(gcounts, xf.shape[0] * self.ep.world)
        if self.num_shared_experts:
            y = y + self.shared_forward(xf, g)
        metrics = routing_metrics(p, w, e, counts, self.num_experts) if return_metrics else None
        return MoEOutput(y.to(x.dtype).view(shape), aux * self.aux_loss_weight, metrics)

    def get_load_balance_stats(self) -> Dict[str, float]:
        return {
            "load_ema_std": float(self.expert_load_ema.std()),
            "load_ema_max": float(self.expert_load_ema.max()),
            "load_ema_min": float(self.expert_load_ema.min()),
            "bias_std": float(self.expert_bias.std()),
            "bias_max": float(self.expert_bias.max()),
            "bias_min": float(self.expert_bias.min()),
        }
