"""C-JEPA: object-centric causal prediction with whole-trajectory object masking.

API of the reference ``core/causal_jepa.py``: ``CausalJEPAConfig`` (:27-67) and presets
(:70-79), ``SlotAttention`` (GRU-updated iterative attention, :82-165),
``ObjectSlotEncoder`` (slots + positions + existence per frame, :168-240),
``InteractionEncoder`` (pairwise features, interaction types, causal influence,
:243-321), ``TrajectoryPredictor`` (transformer decoder over per-object context,
:324-406), ``CausalJEPAPredictor`` (mask whole object trajectories, predict them;
counterfactual removal, :409-602), ``CausalJEPALoss`` (:605-725) and the factory.

Differences by design: frames are encoded in one batched slot-attention call (time
folded into the batch, not a per-frame Python loop), mask indices are sampled for the
whole batch at once on the device, and the trajectory NLL compares predictions with the
last ``horizon`` frames of the targets (the reference compares tensors of different
lengths when the horizon differs from the clip length).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class CausalJEPAConfig:
    max_objects: int = 32
    slot_dim: int = 256
    num_slot_iterations: int = 3
    slot_mlp_hidden_dim: int = 512
    input_dim: int = 256
    num_heads: int = 8
    dropout: float = 0.1
    interaction_dim: int = 128
    num_interaction_heads: int = 4
    max_interaction_distance: float = 50.0
    predictor_dim: int = 512
    predictor_depth: int = 4
    prediction_horizon: int = 8
    min_objects_masked: int = 2
    max_objects_masked: int = 8
    mask_ratio: float = 0.75
    enable_counterfactual: bool = True
    num_counterfactuals: int = 4
    slot_reconstruction_weight: float = 1.0
    trajectory_prediction_weight: float = 0.5
    interaction_weight: float = 0.3
    contrastive_weight: float = 0.2
    counterfactual_weight: float = 0.2


def get_default_causal_jepa_config() -> CausalJEPAConfig:
    return CausalJEPAConfig()


def get_minimal_causal_jepa_config() -> CausalJEPAConfig:
    return CausalJEPAConfig(max_objects=16, slot_dim=128, num_slot_iterations=2, slot_mlp_hidden_dim=256,
                            predictor_dim=256, predictor_depth=2, prediction_horizon=4)


class SlotAttention(nn.Module):
    """Slot Attention (Locatello et al. 2020): slots compete for inputs (softmax over
    slots), weighted-mean updates, GRU + residual MLP, ``num_iterations`` rounds."""

    def __init__(self, num_slots: int, slot_dim: int, input_dim: int, num_iterations: int = 3,
                 epsilon: float = 1e-8, hidden_dim: int = 512):
        super().__init__()
        self.num_slots, self.slot_dim, self.num_iterations, self.eps = num_slots, slot_dim, num_iterations, epsilon
        self.scale = slot_dim ** -0.5
        self.slots_mu = nn.Parameter(torch.randn(1, 1, slot_dim) * 0.02)
        self.slots_log_sigma = nn.Parameter(torch.zeros(1, 1, slot_dim))
        self.norm_inputs = nn.LayerNorm(input_dim)
        self.norm_slots = nn.LayerNorm(slot_dim)
        self.norm_mlp = nn.LayerNorm(slot_dim)
        self.to_q = nn.Linear(slot_dim, slot_dim, bias=False)
        self.to_k = nn.Linear(input_dim, slot_dim, bias=False)
        self.to_v = nn.Linear(input_dim, slot_dim, bias=False)
        self.gru = nn.GRUCell(slot_dim, slot_dim)
        self.mlp = nn.Sequential(nn.Linear(slot_dim, hidden_dim), nn.ReLU(), nn.Linear(hidden_dim, slot_dim))

    def forward(self, inputs: torch.Tensor, generator: Optional[torch.Generator] = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        B, N, _ = inputs.shape
        x = self.norm_inputs(inputs)
        k, v = self.to_k(x), self.to_v(x)
        noise = torch.randn(B, self.num_slots, self.slot_dim, device=inputs.device, dtype=inputs.dtype,
                            generator=generator)
        slots = self.slots_mu + self.slots_log_sigma.exp() * noise
        attn = None
        for _ in range(self.num_iterations):
            prev = slots
            q = self.to_q(self.norm_slots(slots))
            logits = torch.einsum("bsd,bnd->bsn", q, k) * self.scale
            attn = logits.softmax(dim=1) + self.eps             # competition over slots
            w = attn / attn.sum(-1, keepdim=True)
            updates = torch.einsum("bsn,bnd->bsd", w, v)
            slots = self.gru(updates.reshape(-1, self.slot_dim), prev.reshape(-1, self.slot_dim))
            slots = slots.view(B, self.num_slots, self.slot_dim)
            slots = slots + self.mlp(self.norm_mlp(slots))
        return slots, attn


class ObjectSlotEncoder(nn.Module):
    def __init__(self, input_dim: int, slot_dim: int, max_objects: int, num_iterations: int = 3,
                 hidden_dim: int = 512, num_heads: int = 8, dropout: float = 0.1):
        super().__init__()
        self.input_dim, self.slot_dim, self.max_objects = input_dim, slot_dim, max_objects
        self.slot_attention = SlotAttention(max_objects, slot_dim, input_dim, num_iterations,
                                            hidden_dim=hidden_dim)
        self.position_head = nn.Linear(slot_dim, 4)
        self.existence_head = nn.Linear(slot_dim, 1)

    def forward(self, features: torch.Tensor, masks: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        """``features [B, T, N, D]`` -> slots ``[B, T, K, S]``, positions ``[B, T, K, 4]``,
        existence ``[B, T, K]`` (all frames in one slot-attention call)."""
        B, T, N, D = features.shape
        slots, _ = self.slot_attention(features.reshape(B * T, N, D))
        slots = slots.view(B, T, self.max_objects, self.slot_dim)
        return {"slots": slots, "positions": self.position_head(slots),
                "existence_probs": torch.sigmoid(self.existence_head(slots).squeeze(-1))}


class InteractionEncoder(nn.Module):
    def __init__(self, slot_dim: int, interaction_dim: int, num_heads: int = 4, max_distance: float = 50.0):
        super().__init__()
        self.interaction_dim, self.max_distance = interaction_dim, max_distance
        self.interaction_net = nn.Sequential(nn.Linear(2 * slot_dim + 4, 2 * interaction_dim), nn.ReLU(),
                                             nn.Linear(2 * interaction_dim, interaction_dim))
        self.interaction_type = nn.Linear(interaction_dim, 8)
        self.causal_influence = nn.Linear(interaction_dim, 1)

    def forward(self, slots: torch.Tensor, positions: torch.Tensor, existence_mask: torch.Tensor):
        B, N, D = slots.shape
        rel = positions[:, :, None, :2] - positions[:, None, :, :2]          # [B, N, N, 2]
        dist = rel.norm(dim=-1, keepdim=True) / self.max_distance
        pair = torch.cat([slots[:, :, None].expand(B, N, N, D), slots[:, None].expand(B, N, N, D), rel, dist,
                          dist.clamp(max=1.0)], -1)
        feat = self.interaction_net(pair)
        mask = existence_mask[:, :, None] * existence_mask[:, None, :]
        feat = feat * mask[..., None]
        return {"interaction_features": feat, "interaction_types": self.interaction_type(feat),
                "causal_influence": torch.sigmoid(self.causal_influence(feat).squeeze(-1)) * mask}


class TrajectoryPredictor(nn.Module):
    def __init__(self, slot_dim: int, predictor_dim: int, num_layers: int = 4, num_heads: int = 8,
                 prediction_horizon: int = 8, dropout: float = 0.1, interaction_dim: Optional[int] = None):
        super().__init__()
        self.predictor_dim, self.prediction_horizon = predictor_dim, prediction_horizon
        self.input_proj = nn.Linear(slot_dim, predictor_dim)
        self.pos_encoding = nn.Parameter(torch.randn(1, prediction_horizon, predictor_dim) * 0.02)
        layer = nn.TransformerDecoderLayer(predictor_dim, num_heads, 4 * predictor_dim, dropout, batch_first=True)
        self.transformer_decoder = nn.TransformerDecoder(layer, num_layers)
        # each object's context also sees the (masked) sum of its pairwise interaction
        # features; zero-initialised so it starts as a no-op
        self.interaction_proj = nn.Linear(interaction_dim, predictor_dim) if interaction_dim else None
        if self.interaction_proj is not None:
            nn.init.zeros_(self.interaction_proj.weight)
            nn.init.zeros_(self.interaction_proj.bias)
        self.output_proj = nn.Linear(predictor_dim, slot_dim)
        self.position_head = nn.Linear(predictor_dim, 4)
        self.uncertainty_head = nn.Linear(predictor_dim, slot_dim)

    def forward(self, context_slots: torch.Tensor, interaction_features: Optional[torch.Tensor] = None,
                num_steps: Optional[int] = None) -> Dict[str, torch.Tensor]:
        n = num_steps or self.prediction_horizon
        B, T, K, S = context_slots.shape
        ctx = self.input_proj(context_slots.permute(0, 2, 1, 3).reshape(B * K, T, S))
        if interaction_features is not None and self.interaction_proj is not None:
            inter = interaction_features.sum(2)                              # [B, K, I]
            ctx = ctx + self.interaction_proj(inter).reshape(B * K, 1, -1)
        q = self.pos_encoding[:, :n].expand(B * K, -1, -1)
        mask = nn.Transformer.generate_square_subsequent_mask(n, device=ctx.device)
        h = self.transformer_decoder(q, ctx, tgt_mask=mask)
        to_btk = lambda y: y.view(B, K, n, -1).permute(0, 2, 1, 3)
        return {"predicted_slots": to_btk(self.output_proj(h)), "predicted_positions": to_btk(self.position_head(h)),
                "uncertainty": to_btk(F.softplus(self.uncertainty_head(h)))}


class CausalJEPAPredictor(nn.Module):
    def __init__(self, config: Optional[CausalJEPAConfig] = None):
        super().__init__()
        c = self.config = config or get_default_causal_jepa_config()
        self.slot_encoder = ObjectSlotEncoder(c.input_dim, c.slot_dim, c.max_objects, c.num_slot_iterations,
                                              c.slot_mlp_hidden_dim, c.num_heads, c.dropout)
        self.interaction_encoder = InteractionEncoder(c.slot_dim, c.interaction_dim, c.num_interaction_heads,
                                                      c.max_interaction_distance)
        self.trajectory_predictor = TrajectoryPredictor(c.slot_dim, c.predictor_dim, c.predictor_depth,
                                                        c.num_heads, c.prediction_horizon, c.dropout,
                                                        c.interaction_dim)
        if c.enable_counterfactual:
            self.counterfactual_encoder = nn.Sequential(nn.Linear(2 * c.slot_dim, c.predictor_dim), nn.ReLU(),
                                                        nn.Linear(c.predictor_dim, c.slot_dim))
        self.mask_token = nn.Parameter(torch.randn(1, 1, c.slot_dim) * 0.02)

    def _sample_mask_indices(self, batch_size: int, existence_probs: torch.Tensor) -> torch.Tensor:
        """``[B, max_objects_masked]`` object indices, drawn without replacement with
        probability proportional to average existence; each row masks between
        ``min_objects_masked`` and ``max_objects_masked`` objects (the rest of the row
        repeats the first index)."""
        c = self.config
        p = existence_probs.mean(1) + 1e-8                                     # [B, K]
        M = min(c.max_objects_masked, p.shape[1])
        idx = torch.multinomial(p, M, replacement=False)
        n = torch.randint(min(c.min_objects_masked, M), M + 1, (batch_size, 1), device=p.device)
        keep = torch.arange(M, device=p.device)[None] < n
        return torch.where(keep, idx, idx[:, :1])

    def _apply_trajectory_mask(self, slots: torch.Tensor, mask_indices: torch.Tensor):
        B, T, K, S = slots.shape
        m = torch.zeros(B, K, dtype=torch.bool, device=slots.device)
        m[torch.arange(B, device=slots.device)[:, None], mask_indices] = True
        masked = torch.where(m[:, None, :, None], self.mask_token.to(slots.dtype).view(1, 1, 1, S), slots)
        return masked, slots.clone()

    def forward(self, features: torch.Tensor, masks: Optional[torch.Tensor] = None,
                object_mask_indices: Optional[torch.Tensor] = None, return_interactions: bool = True):
        B = features.shape[0]
        so = self.slot_encoder(features, masks)
        slots, exist, pos = so["slots"], so["existence_probs"], so["positions"]
        if object_mask_indices is None:
            object_mask_indices = self._sample_mask_indices(B, exist)
        masked, targets = self._apply_trajectory_mask(slots, object_mask_indices)
        inter = None
        if return_interactions:
            inter = self.interaction_encoder(slots.mean(1), pos.mean(1), (exist.mean(1) > 0.5).float())
        pred = self.trajectory_predictor(masked, inter["interaction_features"] if inter else None)
        return {"slots": slots, "masked_slots": masked, "predicted_slots": pred["predicted_slots"],
                "predictions": pred, "mask_targets": targets, "object_mask_indices": object_mask_indices,
                "interactions": inter, "existence_probs": exist, "positions": pos}

    def predict_counterfactual(self, features: torch.Tensor, removed_object_indices: torch.Tensor, masks=None):
        if not self.config.enable_counterfactual:
            raise ValueError("Counterfactual prediction is disabled")
        out = self.forward(features, masks, return_interactions=True)
        cf = out["slots"].clone()
        B = features.shape[0]
        cf[torch.arange(B, device=cf.device)[:, None], :, removed_object_indices] = 0.0
        cfp = self.trajectory_predictor(cf)
        effect = (out["predictions"]["predicted_slots"] - cfp["predicted_slots"]).pow(2).mean((1, 2, 3))
        return {"original_predictions": out["predictions"], "counterfactual_predictions": cfp,
                "causal_effect": effect, "removed_objects": removed_object_indices}


class CausalJEPALoss(nn.Module):
    def __init__(self, config: Optional[CausalJEPAConfig] = None):
        super().__init__()
        self.config = config or get_default_causal_jepa_config()
        self.temperature = nn.Parameter(torch.tensor(0.07))

    def forward(self, outputs: Dict, targets: Optional[Dict] = None) -> Dict[str, torch.Tensor]:
        c = self.config
        L: Dict[str, torch.Tensor] = {}
        if "predicted_slots" in outputs and "mask_targets" in outputs:
            L["slot_prediction"] = self._slot_prediction_loss(outputs["predicted_slots"], outputs["mask_targets"],
                                                              outputs["object_mask_indices"]) * c.slot_reconstruction_weight
        if "predictions" in outputs:
            L["trajectory"] = self._trajectory_loss(outputs["predictions"], outputs.get("mask_targets")) \
                * c.trajectory_prediction_weight
        if "slots" in outputs and "predicted_slots" in outputs:
            L["contrastive"] = self._contrastive_loss(outputs["slots"], outputs["predicted_slots"]) * c.contrastive_weight
        if "counterfactual_predictions" in outputs:
            L["counterfactual"] = self._counterfactual_loss(outputs) * c.counterfactual_weight
        L["total"] = torch.stack(list(L.values())).sum()
        return L

    @staticmethod
    def _slot_prediction_loss(pred, target, mask_indices):
        B, T, K, S = target.shape
        tgt = target[:, -pred.shape[1]:]
        m = torch.zeros(B, K, device=pred.device)
        m[torch.arange(B, device=pred.device)[:, None], mask_indices] = 1.0
        m = m[:, None, :, None]
        return ((pred - tgt.detach()) ** 2 * m).sum() / (m.sum() * pred.shape[1] * S + 1e-8)

    @staticmethod
    def _trajectory_loss(predictions, targets):
        pp, unc = predictions["predicted_positions"], predictions["uncertainty"]
        if targets is None:
            return (pp[:, 1:] - pp[:, :-1]).pow(2).mean() + 0.1 * unc.mean()
        tgt = targets[:, -predictions["predicted_slots"].shape[1]:].detach()
        var = unc.pow(2) + 1e-8
        return ((predictions["predicted_slots"] - tgt) ** 2 / (2 * var) + 0.5 * torch.log(var)).mean()

    def _contrastive_loss(self, slots, pred):
        n = pred.shape[1]
        a = F.normalize(pred.reshape(-1, pred.shape[-1]), dim=-1)
        b = F.normalize(slots[:, -n:].reshape(-1, slots.shape[-1]).detach(), dim=-1)
        logits = a @ b.t() / self.temperature.clamp_min(1e-3)
        return F.cross_entropy(logits, torch.arange(a.shape[0], device=a.device))

    @staticmethod
    def _counterfactual_loss(outputs):
        # a removal must change the prediction (hinged), and the change must stay bounded
        eff = outputs["causal_effect"]
        return (F.relu(0.01 - eff) + 0.01 * eff).mean()


def create_causal_jepa_predictor(config: Optional[CausalJEPAConfig] = None) -> CausalJEPAPredictor:
    return CausalJEPAPredictor(config)
