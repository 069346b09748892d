"""World-model benchmarks (reference ``evaluation/benchmarks.py``: ``WorldModelBenchmark``
:18-249, ``GenerationBenchmark`` :252-347, ``ControlBenchmark`` :350-377,
``PerformanceBenchmark`` with FPS = B*T/time and latency p50/p95/p99 :380-544,
``MemoryBenchmark`` :547-623). Device timings use CUDA events after warm-up; on CPU,
wall-clock."""
from __future__ import annotations

import json
import time
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch

from .metrics import ControlMetrics, TemporalConsistencyMetrics, VideoMetrics


def _time_ms(fn: Callable[[], Any], device: torch.device, warmup: int = 2, iters: int = 5) -> List[float]:
    for _ in range(warmup):
        fn()
    out = []
    for _ in range(iters):
        if device.type == "cuda":
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            out.append(s.elapsed_time(e))
        else:
            t0 = time.perf_counter()
            fn()
            out.append((time.perf_counter() - t0) * 1000.0)
    return out


def _pct(xs: Sequence[float], q: float) -> float:
    s = sorted(xs)
    return s[min(len(s) - 1, max(0, int(round(q / 100 * (len(s) - 1)))))] if s else 0.0


class GenerationBenchmark:
    """Rollout speed of a world model (frames/s, per-chunk latency)."""

    def __init__(self, model, device: str = "cuda"):
        self.model, self.device = model, torch.device(device)

    def benchmark_generation_speed(self, batch_sizes=(1,), num_frames: int = 16, context_frames: int = 4,
                                   chunk_frames: int = 4, flow_steps: int = 4) -> Dict[str, Any]:
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        m = self.model.cfg
        out = {}
        for B in batch_sizes:
            rc = RolloutConfig(total_frames=context_frames + num_frames, chunk_frames=chunk_frames,
                               flow_steps=flow_steps, window_frames=32, context_frames=context_frames, batch=B)
            r = StreamingRollout(self.model, rc)
            ctx = torch.randn(B, context_frames, m.latent_channels, m.latent_h, m.latent_w, device=self.device)
            act = torch.rand(B, context_frames + num_frames, m.action_dim, device=self.device) * 2 - 1
            r.run(ctx, act, total_frames=context_frames + chunk_frames)
            res = r.run(ctx, act)
            out[f"batch_{B}"] = {"fps": res.frames_per_s(B, chunk_frames), "p50_chunk_ms": res.percentile_ms(50),
                                 "p99_chunk_ms": res.percentile_ms(99)}
        return out

    def benchmark_memory_efficiency(self, batch_sizes=(1, 2), num_frames: int = 8) -> Dict[str, Any]:
        if self.device.type != "cuda":
            return {"available": False}
        out = {}
        for B in batch_sizes:
            torch.cuda.reset_peak_memory_stats(self.device)
            self.benchmark_generation_speed((B,), num_frames)
            out[f"batch_{B}"] = torch.cuda.max_memory_allocated(self.device) / 2 ** 30
        return out


class ControlBenchmark:
    def __init__(self, model, device: str = "cuda"):
        self.model, self.device = model, torch.device(device)

    @torch.no_grad()
    def benchmark_control_response(self, num_trials: int = 4, frames: int = 4) -> Dict[str, float]:
        """Mean latent change caused by flipping the actions (higher = more control)."""
        m = self.model.cfg
        g = torch.Generator(device=self.device).manual_seed(0)
        x = torch.randn(num_trials, frames, m.latent_channels, m.latent_h, m.latent_w, device=self.device, generator=g)
        t = torch.full((num_trials,), 0.5, device=self.device)
        a = torch.rand(num_trials, frames, m.action_dim, device=self.device, generator=g) * 2 - 1
        v1 = self.model(x, t, a).float()
        v2 = self.model(x, t, -a).float()
        return {"control_sensitivity": float((v1 - v2).pow(2).mean()), "response_norm": float(v1.pow(2).mean())}


class PerformanceBenchmark:
    def __init__(self, model, device: str = "cuda", batch_sizes=(1, 2, 4), frames: int = 4):
        self.model, self.device = model, torch.device(device)
        self.batch_sizes, self.frames = batch_sizes, frames
        self.results: Dict[str, Any] = {}

    def _inputs(self, B):
        m = self.model.cfg
        return (torch.randn(B, self.frames, m.latent_channels, m.latent_h, m.latent_w, device=self.device),
                torch.rand(B, device=self.device), torch.rand(B, self.frames, m.action_dim, device=self.device))

    @torch.no_grad()
    def _benchmark_throughput(self) -> Dict[str, float]:
        out = {}
        for B in self.batch_sizes:
            x, t, a = self._inputs(B)
            ms = _time_ms(lambda: self.model(x, t, a), self.device)
            out[f"batch_{B}_fps"] = B * self.frames / (statistics_mean(ms) / 1000.0)
        return out

    @torch.no_grad()
    def _benchmark_latency(self) -> Dict[str, float]:
        x, t, a = self._inputs(1)
        ms = _time_ms(lambda: self.model(x, t, a), self.device, iters=20)
        return {"p50_ms": _pct(ms, 50), "p95_ms": _pct(ms, 95), "p99_ms": _pct(ms, 99), "mean_ms": statistics_mean(ms)}

    def _benchmark_memory(self) -> Dict[str, float]:
        if self.device.type != "cuda":
            return {"available": False}
        torch.cuda.reset_peak_memory_stats(self.device)
        with torch.no_grad():
            self.model(*self._inputs(max(self.batch_sizes)))
        return {"peak_gb": torch.cuda.max_memory_allocated(self.device) / 2 ** 30}

    def _benchmark_scalability(self) -> Dict[str, Any]:
        thr = self._benchmark_throughput()
        b0 = min(self.batch_sizes)
        return {k: v / thr[f"batch_{b0}_fps"] for k, v in thr.items()}

    def run_performance_suite(self) -> Dict[str, Any]:
        self.results = {"throughput": self._benchmark_throughput(), "latency": self._benchmark_latency(),
                        "memory": self._benchmark_memory(), "scalability": self._benchmark_scalability()}
        return self.results


def statistics_mean(xs):
    return sum(xs) / max(len(xs), 1)


class MemoryBenchmark:
    def __init__(self, model, device: str = "cuda"):
        self.model, self.device = model, torch.device(device)

    def _fits(self, B: int, frames: int) -> bool:
        m = self.model.cfg
        try:
            with torch.no_grad():
                self.model(torch.randn(B, frames, m.latent_channels, m.latent_h, m.latent_w, device=self.device),
                           torch.rand(B, device=self.device), torch.rand(B, frames, m.action_dim, device=self.device))
            return True
        except torch.OutOfMemoryError:
            if self.device.type == "cuda":
                torch.cuda.empty_cache()
            return False

    def find_max_batch_size(self, frames: int = 4, start: int = 1, limit: int = 256) -> int:
        B, best = start, 0
        while B <= limit and self._fits(B, frames):
            best, B = B, B * 2
        return best

    def find_max_sequence_length(self, batch: int = 1, start: int = 2, limit: int = 256) -> int:
        F_, best = start, 0
        while F_ <= min(limit, self.model.cfg.max_frames) and self._fits(batch, F_):
            best, F_ = F_, F_ * 2
        return best


class WorldModelBenchmark:
    """Quality / temporal / control / long-sequence suite over a test batch
    ``{'latents': [B, T, C, H, W], 'actions': [B, T, A]}``."""

    def __init__(self, model, vae_model=None, device: str = "cuda", save_path: Optional[str] = None,
                 output_dir: Optional[str] = None):
        """The reference's arguments (``model, vae_model, device, save_path``,
        evaluation/benchmarks.py); ``WorldModelBenchmark(model, device)`` also works."""
        if isinstance(vae_model, (str, torch.device)):   # (model, device, ...)
            vae_model, device = None, vae_model
        self.vae_model = vae_model
        self.model, self.device = model, torch.device(device)
        out = save_path or output_dir
        self.output_dir = Path(out) if out else None
        self.results: Dict[str, Any] = {}

    def run_full_benchmark(self, test_data: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        self.results = {"generation": self._benchmark_generation(test_data),
                        "quality": self._benchmark_quality(test_data),
                        "temporal_consistency": self._benchmark_temporal_consistency(test_data),
                        "control_conditioning": self._benchmark_control_conditioning(test_data),
                        "long_sequences": self._benchmark_long_sequences(test_data)}
        self._save_results()
        return self.results

    def _benchmark_generation(self, test_data):
        return GenerationBenchmark(self.model, str(self.device)).benchmark_generation_speed(
            (test_data["latents"].shape[0],), num_frames=4, context_frames=2, chunk_frames=2, flow_steps=2)

    @torch.no_grad()
    def _rollout(self, test_data, ctx: int):
        from ..config import RolloutConfig
        from ..inference.rollout import StreamingRollout

        lat, act = test_data["latents"].to(self.device), test_data["actions"].to(self.device)
        T = lat.shape[1]
        rc = RolloutConfig(total_frames=T, chunk_frames=1, flow_steps=2, window_frames=32, context_frames=ctx,
                           batch=lat.shape[0])
        return StreamingRollout(self.model, rc).run(lat[:, :ctx], act).frames.float(), lat.float()

    def _benchmark_quality(self, test_data):
        pred, gt = self._rollout(test_data, max(1, test_data["latents"].shape[1] // 2))
        return {"latent_mse": float(VideoMetrics.mse(pred, gt)), "latent_mae": float(VideoMetrics.mae(pred, gt))}

    def _benchmark_temporal_consistency(self, test_data):
        pred, _ = self._rollout(test_data, 1)
        return {"temporal_mse": float(TemporalConsistencyMetrics.temporal_mse(pred))}

    def _benchmark_control_conditioning(self, test_data):
        return ControlBenchmark(self.model, str(self.device)).benchmark_control_response(2, 2)

    def _benchmark_long_sequences(self, test_data):
        pred, gt = self._rollout(test_data, 1)
        err = (pred - gt).pow(2).flatten(2).mean(-1).mean(0)
        return {"error_growth": err.tolist()}

    def _save_results(self):
        if self.output_dir is not None:
            self.output_dir.mkdir(parents=True, exist_ok=True)
            (self.output_dir / "benchmark_results.json").write_text(json.dumps(self.results, indent=2, default=float))
