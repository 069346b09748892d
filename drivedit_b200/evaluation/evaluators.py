"""Sequence / batch / real-time evaluators (reference ``evaluation/evaluators.py``:
``SequenceEvaluator`` :18-222, ``BatchEvaluator`` :225-361, ``RealTimeEvaluator``
:364-626) over the streaming rollout of a :class:`WorldDiT`."""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence

import torch

from .benchmarks import _pct, _time_ms
from .metrics import LatentMetrics, TemporalConsistencyMetrics, VideoMetrics


class SequenceEvaluator:
    def __init__(self, model, device: str = "cuda", context_frames: int = 2, flow_steps: int = 2,
                 chunk_frames: int = 1):
        self.model, self.device = model, torch.device(device)
        self.context_frames, self.flow_steps, self.chunk_frames = context_frames, flow_steps, chunk_frames

    @torch.no_grad()
    def _generate_sequence(self, latents: torch.Tensor, actions: torch.Tensor) -> torch.Tensor:
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        rc = RolloutConfig(total_frames=latents.shape[1], chunk_frames=self.chunk_frames, flow_steps=self.flow_steps,
                           window_frames=32, context_frames=self.context_frames, batch=latents.shape[0])
        return StreamingRollout(self.model, rc).run(latents[:, :self.context_frames].to(self.device),
                                                    actions.to(self.device)).frames.float()

    def _compute_sequence_metrics(self, pred: torch.Tensor, gt: torch.Tensor) -> Dict[str, float]:
        c = self.context_frames
        p, g = pred[:, c:], gt[:, c:].float().to(pred.device)
        return {"mse": float(VideoMetrics.mse(p, g)), "mae": float(VideoMetrics.mae(p, g)),
                "cosine": float(LatentMetrics.latent_cosine_similarity(p, g)),
                "temporal_mse": float(TemporalConsistencyMetrics.temporal_mse(p)) if p.shape[1] > 1 else 0.0}

    def evaluate_sequence(self, latents: torch.Tensor, actions: torch.Tensor) -> Dict[str, float]:
        return self._compute_sequence_metrics(self._generate_sequence(latents, actions), latents)

    def evaluate_batch(self, batches: Sequence[Dict[str, torch.Tensor]]) -> Dict[str, float]:
        return self._average_metrics([self.evaluate_sequence(b["latents"], b["actions"]) for b in batches])

    @staticmethod
    def _average_metrics(ms: List[Dict[str, float]]) -> Dict[str, float]:
        return {k: sum(m[k] for m in ms) / len(ms) for k in ms[0]} if ms else {}


class BatchEvaluator:
    def __init__(self, model, device: str = "cuda", frames: int = 4):
        self.model, self.device, self.frames = model, torch.device(device), frames

    def _inputs(self, B):
        m = self.model.cfg
        return (torch.randn(B, self.frames, m.latent_channels, m.latent_h, m.latent_w, device=self.device),
                torch.rand(B, device=self.device), torch.rand(B, self.frames, m.action_dim, device=self.device))

    @torch.no_grad()
    def evaluate_batch_efficiency(self, batch_sizes=(1, 2, 4)) -> Dict[str, Dict[str, float]]:
        out = {}
        for B in batch_sizes:
            x, t, a = self._inputs(B)
            ms = _time_ms(lambda: self.model(x, t, a), self.device)
            mean = sum(ms) / len(ms)
            out[f"batch_{B}"] = {"ms": mean, "frames_per_s": B * self.frames / (mean / 1000.0),
                                 "ms_per_sample": mean / B}
        return out

    def find_optimal_batch_size(self, batch_sizes=(1, 2, 4, 8)) -> int:
        eff = self.evaluate_batch_efficiency(batch_sizes)
        return max(batch_sizes, key=lambda b: eff[f"batch_{b}"]["frames_per_s"])


class RealTimeEvaluator:
    """Can the rollout sustain ``target_fps``? Per-chunk device latency percentiles."""

    def __init__(self, model, device: str = "cuda"):
        self.model, self.device = model, torch.device(device)

    def evaluate_real_time_performance(self, target_fps: float = 20.0, frames: int = 16, chunk_frames: int = 4,
                                       flow_steps: int = 4, batch: int = 1) -> Dict[str, Any]:
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        m = self.model.cfg
        rc = RolloutConfig(total_frames=4 + frames, chunk_frames=chunk_frames, flow_steps=flow_steps,
                           window_frames=32, context_frames=4, batch=batch)
        r = StreamingRollout(self.model, rc)
        ctx = torch.randn(batch, 4, m.latent_channels, m.latent_h, m.latent_w, device=self.device)
        act = torch.rand(batch, 4 + frames, m.action_dim, device=self.device) * 2 - 1
        r.run(ctx, act, total_frames=4 + chunk_frames)
        res = r.run(ctx, act)
        fps = res.frames_per_s(batch, chunk_frames)
        budget = 1000.0 * chunk_frames / target_fps
        return {"fps": fps, "meets_target": fps >= target_fps, "p50_chunk_ms": res.percentile_ms(50),
                "p95_chunk_ms": res.percentile_ms(95), "p99_chunk_ms": res.percentile_ms(99),
                "chunk_budget_ms": budget,
                "frames_over_budget": sum(1 for c in res.chunk_ms if c > budget) / max(len(res.chunk_ms), 1)}
