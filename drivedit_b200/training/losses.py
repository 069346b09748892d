"""Unified training losses (v1).

Same surface and arithmetic as the reference ``training/losses.py``: ``UnifiedLoss``
(reconstruction MSE + L1 + grey-level "perceptual" L1, flow matching, temporal
frame-difference consistency, JEPA positive/negative margin loss, curriculum ramps, loss
history; :20-290), ``FlowMatchingLoss`` (rectified-flow / velocity-matching with SNR
weighting / trajectory distillation, :293-365), ``ReconstructionLoss`` (multi-scale,
gradient, :368-411), ``TemporalConsistencyLoss`` (frame differences, second-order
smoothness, :414-439) and ``create_unified_loss`` (:442+).

The loss history stores detached device tensors; statistics are produced on demand
(no per-step host synchronisation).
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn.functional as F


class UnifiedLoss:
    def __init__(self, training_config=None):
        self.config = training_config
        self.step = 0
        self.loss_history: Dict[str, List[torch.Tensor]] = {}
        self.weights = {"reconstruction": 1.0,
                        "flow_matching": 1.0 if getattr(training_config, "enable_flow_matching", False) else 0.0,
                        "temporal_consistency": 0.2, "jepa": 0.1, "perceptual": 0.1, "l1": 0.1}

    def __call__(self, predictions: Dict[str, torch.Tensor], targets: Dict[str, torch.Tensor],
                 step: Optional[int] = None) -> Dict[str, torch.Tensor]:
        if step is not None:
            self.step = step
        losses: Dict[str, torch.Tensor] = {}
        if "predictions" in predictions and "frames" in targets:
            losses.update(self._reconstruction_losses(predictions["predictions"], targets["frames"]))
            losses["temporal_consistency"] = self._temporal_consistency_loss(predictions["predictions"],
                                                                             targets["frames"])
        if getattr(self.config, "enable_flow_matching", False) and "flow_predictions" in predictions:
            losses["flow_matching"] = self._flow_matching_loss(predictions, targets)
        if "jepa_predictions" in predictions:
            losses["jepa"] = self._jepa_loss(predictions, targets)
        if getattr(self.config, "enable_curriculum", False):
            losses = self._apply_curriculum_weights(losses)
        losses["total"] = self._compute_total_loss(losses)
        self._update_history(losses)
        return losses

    def _reconstruction_losses(self, pred, target):
        if pred.shape[1] != target.shape[1]:
            target = target[:, -pred.shape[1]:]
        pred, target = pred.float(), target.float()
        return {"reconstruction": F.mse_loss(pred, target) * self.weights["reconstruction"],
                "l1": F.l1_loss(pred, target) * self.weights["l1"],
                "perceptual": F.l1_loss(pred.mean(2, keepdim=True), target.mean(2, keepdim=True))
                * self.weights["perceptual"]}

    def _flow_matching_loss(self, predictions, targets):
        fp = predictions["flow_predictions"].float()
        if "flow_target" in targets:
            tgt = targets["flow_target"].float()
        elif "predictions" in predictions and "frames" in targets:
            tgt = targets["frames"].float() - predictions["predictions"].float()
        else:
            return fp.new_zeros(())
        return F.mse_loss(fp, tgt) * self.weights["flow_matching"]

    def _temporal_consistency_loss(self, pred, target):
        if pred.shape[1] != target.shape[1]:
            target = target[:, -pred.shape[1]:]
        if pred.shape[1] <= 1:
            return pred.new_zeros((), dtype=torch.float32)
        pd = pred[:, 1:].float() - pred[:, :-1].float()
        td = target[:, 1:].float() - target[:, :-1].float()
        return F.mse_loss(pd, td) * self.weights["temporal_consistency"]

    def _jepa_loss(self, predictions, targets):
        jp = predictions["jepa_predictions"].float()
        if "hidden_states" not in predictions:
            return jp.new_zeros(())
        B, L, _ = jp.shape
        hs = predictions["hidden_states"].float()
        tgt = hs[:, -L:] if hs.shape[1] > L else hs[:, -1:].expand(-1, L, -1)
        pos = F.mse_loss(jp, tgt)
        neg = F.mse_loss(jp, tgt[torch.randperm(B, device=jp.device)])
        return (pos + torch.clamp(1.0 - neg, min=0.0)) * self.weights["jepa"]

    def _apply_curriculum_weights(self, losses):
        p = min(1.0, self.step / getattr(self.config, "curriculum_warmup_steps", 10000))
        cw = {"reconstruction": 1.0, "l1": 1.0, "perceptual": 1.0, "flow_matching": 0.1 + 0.9 * p,
              "temporal_consistency": p, "jepa": max(0.0, p - 0.3) / 0.7}
        return {k: v * cw.get(k, 1.0) for k, v in losses.items()}

    @staticmethod
    def _compute_total_loss(losses):
        vals = [v for k, v in losses.items() if k != "total"]
        return torch.stack([v.float() for v in vals]).sum() if vals else torch.zeros(())

    def _update_history(self, losses):
        for k, v in losses.items():
            h = self.loss_history.setdefault(k, [])
            h.append(v.detach() if torch.is_tensor(v) else torch.tensor(float(v)))
            if len(h) > 1000:
                del h[:-500]

    def get_loss_stats(self) -> Dict[str, float]:
        out = {}
        for k, h in self.loss_history.items():
            if h:
                r = torch.stack([x.float().cpu() for x in h[-100:]])
                out[f"{k}_mean"], out[f"{k}_std"] = float(r.mean()), float(r.std(unbiased=False))
                out[f"{k}_current"] = float(r[-1])
        return out


class FlowMatchingLoss:
    @staticmethod
    def rectified_flow_loss(flow_pred, z_0, z_1, t=None):
        return F.mse_loss(flow_pred.float(), (z_1 - z_0).float())

    @staticmethod
    def velocity_matching_loss(pred_velocity, target_velocity, timesteps=None, weighting: str = "uniform"):
        loss = F.mse_loss(pred_velocity.float(), target_velocity.float(), reduction="none")
        if timesteps is not None and weighting != "uniform":
            snr = 1.0 / (timesteps.float() + 1e-8)
            if weighting == "truncated_snr":
                snr = snr.clamp(0, 1000)
            if weighting in ("snr", "truncated_snr"):
                loss = loss * snr.view(-1, *([1] * (loss.dim() - 1)))
        return loss.mean()

    @staticmethod
    def distillation_loss(student_flow, teacher_trajectory, dt: float = None):
        v = (teacher_trajectory[-1] - teacher_trajectory[0]) / (len(teacher_trajectory) - 1)
        return F.mse_loss(student_flow.float(), v.float())


class ReconstructionLoss:
    @staticmethod
    def multi_scale_loss(pred, target, scales=(1, 2, 4)):
        p, t = pred.reshape(-1, *pred.shape[-3:]).float(), target.reshape(-1, *target.shape[-3:]).float()
        total = p.new_zeros(())
        for s in scales:
            ps, ts = (F.avg_pool2d(p, s), F.avg_pool2d(t, s)) if s > 1 else (p, t)
            total = total + F.mse_loss(ps, ts) / s
        return total

    @staticmethod
    def gradient_loss(pred, target):
        p, t = pred.float(), target.float()
        return (F.l1_loss(p[..., :-1, :] - p[..., 1:, :], t[..., :-1, :] - t[..., 1:, :])
                + F.l1_loss(p[..., :, :-1] - p[..., :, 1:], t[..., :, :-1] - t[..., :, 1:]))


class TemporalConsistencyLoss:
    @staticmethod
    def frame_difference_loss(pred_sequence, target_sequence):
        if pred_sequence.shape[1] <= 1:
            return pred_sequence.new_zeros((), dtype=torch.float32)
        return F.mse_loss((pred_sequence[:, 1:] - pred_sequence[:, :-1]).float(),
                          (target_sequence[:, 1:] - target_sequence[:, :-1]).float())

    @staticmethod
    def smoothness_loss(frames):
        if frames.shape[1] < 3:
            return frames.new_zeros((), dtype=torch.float32)
        acc = frames[:, 2:].float() - 2 * frames[:, 1:-1].float() + frames[:, :-2].float()
        return acc.pow(2).mean()


def create_unified_loss(training_config=None) -> UnifiedLoss:
    return UnifiedLoss(training_config)
