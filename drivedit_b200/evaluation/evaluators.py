"""Sequence / batch / real-time / comparison / ablation evaluators (reference
``evaluation/evaluators.py``: ``SequenceEvaluator`` :18-222, ``BatchEvaluator``
:225-361, ``RealTimeEvaluator`` :364-478, ``ComparisonEvaluator`` :481-551,
``AblationEvaluator`` :554-626) over the streaming rollout of a :class:`WorldDiT`."""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence

import torch

from .benchmarks import _pct, _time_ms
from .metrics import LatentMetrics, TemporalConsistencyMetrics, VideoMetrics


class SequenceEvaluator:
    """Rolls a world model out from the first ``context_frames`` latent frames of each
    sequence and scores the generated frames. Takes the reference's arguments
    (``model, vae_model, device, compute_expensive_metrics``, evaluation/evaluators.py);
    ``SequenceEvaluator(model, device)`` also works. Evaluation is in latent space, so
    ``vae_model`` is kept for callers that decode."""

    def __init__(self, model, vae_model=None, device: str = "cuda",
                 compute_expensive_metrics: bool = True, context_frames: int = 2,
                 flow_steps: int = 2, chunk_frames: int = 1):
        if isinstance(vae_model, (str, torch.device)):   # (model, device, ...)
            vae_model, device = None, vae_model
        self.vae_model, self.compute_expensive_metrics = vae_model, compute_expensive_metrics
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

    @torch.no_grad()
    def evaluate_streaming_performance(self, total_duration_s: float = 10.0, chunk_frames: int = 4,
                                       source_fps: float = 30.0, flow_steps: int = 4,
                                       batch: int = 1) -> Dict[str, Any]:
        """Stream ``total_duration_s`` of video at ``source_fps`` through the chunked
        rollout; real-time factor = video seconds produced per wall-clock second
        (reference :430-478). Chunk times are device times (CUDA events) on a GPU."""
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        m = self.model.cfg
        frames = max(chunk_frames, int(total_duration_s * source_fps))
        rc = RolloutConfig(total_frames=4 + frames, chunk_frames=chunk_frames, flow_steps=flow_steps,
                           window_frames=32, context_frames=4, batch=batch)
        r = StreamingRollout(self.model, rc)
        ctx = torch.randn(batch, 4, m.latent_channels, m.latent_h, m.latent_w, device=self.device)
        act = torch.rand(batch, 4 + frames, m.action_dim, device=self.device) * 2 - 1
        cuda = self.device.type == "cuda"
        mem0 = torch.cuda.memory_allocated(self.device) if cuda else 0
        if cuda:
            torch.cuda.reset_peak_memory_stats(self.device)
        res = r.run(ctx, act)
        ms = torch.tensor(res.chunk_ms, dtype=torch.float64)
        wall = float(ms.sum()) / 1000.0
        return {"total_duration_s": frames / source_fps, "total_chunks": len(res.chunk_ms),
                "actual_duration_s": wall, "mean_chunk_time_ms": float(ms.mean()),
                "max_chunk_time_ms": float(ms.max()),
                "chunk_time_variance": float(ms.var()) if ms.numel() > 1 else 0.0,
                "real_time_factor": (frames / source_fps) / max(wall, 1e-9),
                "peak_memory_mb": (torch.cuda.max_memory_allocated(self.device) - mem0) / 2 ** 20
                if cuda else 0.0}


def _improved(metric: str, change: float) -> bool:
    from .visualization import lower_is_better

    return change < 0 if lower_is_better(metric) else change > 0


class ComparisonEvaluator:
    """Several models on the same sequences (reference :481-551): per-model metrics and,
    per metric, the best and worst model (direction by metric name)."""

    def __init__(self, models: Dict[str, torch.nn.Module], device: str = "cuda", **seq_kwargs):
        self.models = {n: m.eval() for n, m in models.items()}
        self.device = device
        self.seq_kwargs = seq_kwargs

    def compare_models(self, batches: Sequence[Dict[str, torch.Tensor]],
                       metrics_to_compare: Optional[List[str]] = None) -> Dict[str, Any]:
        results = {}
        for name, model in self.models.items():
            ev = SequenceEvaluator(model, device=self.device, **self.seq_kwargs)
            r = ev.evaluate_batch(batches)
            if metrics_to_compare:
                r = {k: v for k, v in r.items() if k in metrics_to_compare}
            results[name] = r
        return {"individual_results": results,
                "comparison_summary": self._create_comparison_summary(
                    results, metrics_to_compare or sorted({k for r in results.values() for k in r}))}

    @staticmethod
    def _create_comparison_summary(results: Dict[str, Dict[str, float]],
                                   metrics: Sequence[str]) -> Dict[str, Any]:
        from .visualization import lower_is_better

        out = {}
        for m in metrics:
            vals = {n: r[m] for n, r in results.items() if m in r}
            if not vals:
                continue
            order = sorted(vals, key=vals.get, reverse=not lower_is_better(m))
            out[m] = {"best_model": order[0], "best_value": vals[order[0]],
                      "worst_model": order[-1], "worst_value": vals[order[-1]], "all_values": vals}
        return out


class AblationEvaluator:
    """Ablations of a :class:`~drivedit_b200.models.world_dit.WorldDiT` (reference
    :554-626, whose model construction is a placeholder). Each ablation config is
    ``{"name": ..., "overrides": {"attention": "dense", "n_layers": 6, ...}}``: the model
    is rebuilt from the base config with those ``ModelConfig`` fields changed and every
    base weight whose name and shape still match is copied in; the rest keep their
    initialisation. Results are compared to the base model metric by metric."""

    def __init__(self, base_model, device: str = "cuda", **seq_kwargs):
        self.base_model = base_model
        self.device = device
        self.seq_kwargs = seq_kwargs

    def _create_ablated_model(self, config: Dict[str, Any]):
        import dataclasses

        from ..models.world_dit import WorldDiT

        cfg = dataclasses.replace(self.base_model.cfg, **config.get("overrides", {}))
        model = WorldDiT(cfg)
        own = model.state_dict()
        base = {k: v for k, v in self.base_model.state_dict().items()
                if k in own and own[k].shape == v.shape}
        model.load_state_dict(base, strict=False)
        return model.to(next(self.base_model.parameters()).device).eval()

    def evaluate_component_ablation(self, batches: Sequence[Dict[str, torch.Tensor]],
                                    ablation_configs: List[Dict[str, Any]]) -> Dict[str, Any]:
        results = {"base_model": SequenceEvaluator(self.base_model, device=self.device,
                                                   **self.seq_kwargs).evaluate_batch(batches)}
        for i, c in enumerate(ablation_configs):
            model = self._create_ablated_model(c)
            results[c.get("name", f"ablation_{i}")] = SequenceEvaluator(
                model, device=self.device, **self.seq_kwargs).evaluate_batch(batches)
        return {"results": results, "analysis": self._analyze_ablation_results(results)}

    @staticmethod
    def _analyze_ablation_results(results: Dict[str, Dict[str, float]]) -> Dict[str, Any]:
        base = results.get("base_model")
        if base is None:
            return {}
        out = {}
        for name, r in results.items():
            if name == "base_model":
                continue
            out[name] = {}
            for m, v in r.items():
                b = base.get(m)
                if isinstance(v, (int, float)) and isinstance(b, (int, float)) and b != 0:
                    rel = (v - b) / abs(b)
                    out[name][m] = {"absolute_change": v - b, "relative_change": rel,
                                    "improved": _improved(m, rel)}
        return out
