"""Inference optimisation and benchmarking (the reference's ``inference/optimization.py``
interface: ``CompileMode``, ``PrecisionMode``, ``OptimizationConfig``, ``BenchmarkResult``,
``ModelCompiler``, ``InferenceOptimizer``, ``FrameMetrics``, ``StreamingInference``,
``MemoryTracker``, ``benchmark_inference``, ``profile_bottlenecks``,
``optimize_for_deployment``, ``compare_optimization_modes``).

B200 design: "compiling" a model means capturing its forward for fixed input shapes in a
CUDA graph (warm-up on a side stream, capture, replay with the inputs copied into static
buffers), so a step costs one graph launch instead of hundreds of kernel launches; there is
no tracing compiler on the path. ``CompileMode.NONE`` runs eagerly; every other mode
captures. Precision ``AUTO`` / ``FP16`` / ``BF16`` select bf16 autocast on sm_100a (bf16 has
fp32's range, so no loss scaling); ``INT8`` is rejected, as it has no kernels here (the
reference only lists it). Timings are CUDA events on the launching stream.
"""
from __future__ import annotations

import contextlib
import gc
import time
from collections import deque
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Callable, Dict, Iterator, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn as nn


class CompileMode(Enum):
    REDUCE_OVERHEAD = "reduce-overhead"
    MAX_AUTOTUNE = "max-autotune"
    DEFAULT = "default"
    NONE = None


class PrecisionMode(Enum):
    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    INT8 = "int8"
    AUTO = "auto"


@dataclass
class OptimizationConfig:
    compile_mode: CompileMode = CompileMode.REDUCE_OVERHEAD
    compile_dynamic: bool = False
    compile_fullgraph: bool = False
    warmup_iterations: int = 3
    precision_mode: PrecisionMode = PrecisionMode.BF16
    use_autocast: bool = True
    kv_cache_max_length: int = 512
    kv_cache_truncate_to: int = 256
    kv_cache_detach_interval: int = 8
    max_memory_gb: float = 16.0
    memory_cleanup_threshold: float = 0.85
    chunk_size: int = 4
    use_gradient_checkpointing: bool = False
    frame_buffer_size: int = 8
    target_fps: float = 20.0
    latency_budget_ms: float = 50.0
    auto_tune_batch_size: bool = True
    max_batch_size: int = 32
    min_batch_size: int = 1


@dataclass
class BenchmarkResult:
    avg_latency_ms: float = 0.0
    min_latency_ms: float = 0.0
    max_latency_ms: float = 0.0
    p50_latency_ms: float = 0.0
    p95_latency_ms: float = 0.0
    p99_latency_ms: float = 0.0
    fps: float = 0.0
    throughput_samples_per_sec: float = 0.0
    peak_memory_mb: float = 0.0
    avg_memory_mb: float = 0.0
    memory_reserved_mb: float = 0.0
    batch_size: int = 1
    sequence_length: int = 1
    warmup_iterations: int = 0
    benchmark_iterations: int = 0
    device: str = "cuda"
    operation_times: Dict[str, float] = field(default_factory=dict)

    def to_dict(self) -> Dict[str, Any]:
        return {"latency": {"avg_ms": self.avg_latency_ms, "min_ms": self.min_latency_ms,
                            "max_ms": self.max_latency_ms, "p50_ms": self.p50_latency_ms,
                            "p95_ms": self.p95_latency_ms, "p99_ms": self.p99_latency_ms},
                "throughput": {"fps": self.fps, "samples_per_sec": self.throughput_samples_per_sec},
                "memory": {"peak_mb": self.peak_memory_mb, "avg_mb": self.avg_memory_mb,
                           "reserved_mb": self.memory_reserved_mb},
                "config": {"batch_size": self.batch_size, "sequence_length": self.sequence_length,
                           "device": self.device, "warmup": self.warmup_iterations,
                           "iterations": self.benchmark_iterations},
                "operations": dict(self.operation_times)}

    def summary(self) -> str:
        return (f"Benchmark Results:\n  Latency: {self.avg_latency_ms:.2f}ms avg (p50: {self.p50_latency_ms:.2f}ms, "
                f"p95: {self.p95_latency_ms:.2f}ms)\n  FPS: {self.fps:.1f} "
                f"({self.throughput_samples_per_sec:.1f} samples/sec)\n  Memory: {self.peak_memory_mb:.1f}MB peak, "
                f"{self.avg_memory_mb:.1f}MB avg\n  Config: batch={self.batch_size}, "
                f"seq_len={self.sequence_length}, device={self.device}")


def _dtype(mode: PrecisionMode) -> Optional[torch.dtype]:
    if mode == PrecisionMode.INT8:
        raise ValueError("int8 inference has no kernels in this framework")
    return None if mode == PrecisionMode.FP32 else torch.bfloat16


# ----------------------------------------------------------------------------- CUDA graphs
class GraphedModule(nn.Module):
    """Replays a CUDA graph of ``module(*static_inputs)``; inputs of the captured shapes
    are copied into the static buffers, other shapes run eagerly."""

    def __init__(self, module: nn.Module, example_inputs: Sequence[torch.Tensor], warmup: int = 3,
                 autocast_dtype: Optional[torch.dtype] = None):
        super().__init__()
        self.module = module
        self.autocast_dtype = autocast_dtype
        self.static_in = [x.detach().clone() for x in example_inputs]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s), torch.no_grad():
            for _ in range(max(warmup, 1)):
                self._call(*self.static_in)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.static_out = self._call(*self.static_in)

    def _call(self, *xs):
        ctx = (torch.autocast("cuda", dtype=self.autocast_dtype) if self.autocast_dtype is not None
               else contextlib.nullcontext())
        with ctx:
            return self.module(*xs)

    def forward(self, *xs):
        if len(xs) != len(self.static_in) or any(x.shape != s.shape for x, s in zip(xs, self.static_in)):
            with torch.no_grad():
                return self._call(*xs)
        for s, x in zip(self.static_in, xs):
            s.copy_(x)
        self.graph.replay()
        return self.static_out


class ModelCompiler:
    """Captures models / sub-modules into CUDA graphs (see :class:`GraphedModule`).

    Takes the reference's arguments (``mode, dynamic, fullgraph, backend,
    disable_cudagraphs``, inference/optimization.py:210-235) or an
    :class:`OptimizationConfig` as its first argument. ``dynamic``, ``fullgraph`` and
    ``backend`` are recorded only (there is no tracing compiler); ``disable_cudagraphs``
    makes :meth:`compile` return the model unchanged."""

    def __init__(self, mode=CompileMode.REDUCE_OVERHEAD, dynamic: bool = False, fullgraph: bool = False,
                 backend: str = "inductor", disable_cudagraphs: bool = False,
                 config: Optional[OptimizationConfig] = None):
        if isinstance(mode, OptimizationConfig):
            config, mode = mode, mode.compile_mode
        self.config = config or OptimizationConfig(compile_mode=mode, compile_dynamic=dynamic,
                                                   compile_fullgraph=fullgraph)
        self.mode, self.dynamic, self.fullgraph = self.config.compile_mode, dynamic, fullgraph
        self.backend, self.disable_cudagraphs = backend, disable_cudagraphs
        self._compiled: Dict[int, nn.Module] = {}
        self._warm: set = set()
        self._errors: Dict[int, Exception] = {}

    def compile(self, model: nn.Module, example_inputs: Optional[Sequence[torch.Tensor]] = None,
                mode: Optional[CompileMode] = None) -> nn.Module:
        mode = mode or self.config.compile_mode
        if (mode == CompileMode.NONE or self.disable_cudagraphs or example_inputs is None
                or not torch.cuda.is_available()):
            return model
        if isinstance(example_inputs, torch.Tensor):
            example_inputs = (example_inputs,)
        try:
            dt = _dtype(self.config.precision_mode) if self.config.use_autocast else None
            g = GraphedModule(model, example_inputs, self.config.warmup_iterations, dt)
        except Exception as e:  # noqa: BLE001 - capture can fail for host-synchronising models
            self._errors[id(model)] = e
            return model
        self._compiled[id(g)] = g
        self._warm.add(id(g))
        return g

    def compile_submodule(self, model: nn.Module, name: str, example_inputs, mode=None) -> nn.Module:
        sub = model.get_submodule(name)
        g = self.compile(sub, example_inputs, mode)
        parent_name, _, attr = name.rpartition(".")
        setattr(model.get_submodule(parent_name) if parent_name else model, attr, g)
        return model

    def compile_multiple_submodules(self, model: nn.Module, specs: Dict[str, Sequence[torch.Tensor]],
                                    mode=None) -> nn.Module:
        for name, ex in specs.items():
            self.compile_submodule(model, name, ex, mode)
        return model

    def warmup(self, model: nn.Module, example_inputs, iterations: Optional[int] = None) -> float:
        """Runs the model ``iterations`` times; returns the mean time of the last half (ms)."""
        if isinstance(example_inputs, torch.Tensor):
            example_inputs = (example_inputs,)
        n = iterations or self.config.warmup_iterations
        times = []
        with torch.no_grad():
            for _ in range(max(n, 1)):
                t0 = time.perf_counter()
                model(*example_inputs)
                if torch.cuda.is_available():
                    torch.cuda.synchronize()
                times.append((time.perf_counter() - t0) * 1000)
        self._warm.add(id(model))
        return float(np.mean(times[len(times) // 2:]))

    def is_compiled(self, model: nn.Module) -> bool:
        return isinstance(model, GraphedModule)

    def is_warmed_up(self, model: nn.Module) -> bool:
        return id(model) in self._warm

    def get_compilation_error(self, model: nn.Module) -> Optional[Exception]:
        return self._errors.get(id(model))

    def reset(self) -> None:
        self._compiled.clear()
        self._warm.clear()
        self._errors.clear()


class InferenceOptimizer:
    def __init__(self, config: Optional[OptimizationConfig] = None):
        self.config = config or OptimizationConfig()
        self.compiler = ModelCompiler(self.config)
        self._kv_cache = None
        self._optimal_batch: Optional[int] = None

    def _get_dtype(self) -> torch.dtype:
        dt = _dtype(self.config.precision_mode)
        return dt or torch.float32

    def optimize_model(self, model: nn.Module, example_input=None, compile_model: bool = True,
                       warmup: bool = True) -> nn.Module:
        model.eval()
        if self.config.use_gradient_checkpointing:
            self._enable_gradient_checkpointing(model)
        if compile_model and example_input is not None:
            model = self.compiler.compile(model, example_input)
        elif warmup and example_input is not None:
            self.compiler.warmup(model, example_input)
        return model

    def _enable_gradient_checkpointing(self, model: nn.Module) -> None:
        for m in model.modules():
            if hasattr(m, "gradient_checkpointing"):
                m.gradient_checkpointing = True

    @contextlib.contextmanager
    def inference_context(self, dtype: Optional[torch.dtype] = None) -> Iterator[None]:
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        dt = dtype or self._get_dtype()
        use = self.config.use_autocast and dt != torch.float32
        with torch.inference_mode(), torch.autocast(dev, dtype=dt, enabled=use):
            yield

    def initialize_kv_cache(self, num_layers: int = 12, device=None):
        from ..training.self_forcing import RollingKVCache

        self._kv_cache = RollingKVCache(self.config.kv_cache_max_length, self.config.kv_cache_truncate_to,
                                        self.config.kv_cache_detach_interval, num_layers, device)
        return self._kv_cache

    def reset_kv_cache(self) -> None:
        if self._kv_cache is not None:
            self._kv_cache.reset()

    def get_kv_cache(self):
        return self._kv_cache

    def chunked_attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, chunk_size: int = 1024,
                          causal: bool = False, scale: Optional[float] = None) -> torch.Tensor:
        """``[B, H, T, D]`` attention computed over query chunks (bounded memory)."""
        T = q.shape[2]
        S = k.shape[2]
        out = []
        for s in range(0, T, chunk_size):
            e = min(T, s + chunk_size)
            mask = None
            if causal:
                qi = torch.arange(s, e, device=q.device)[:, None] + (S - T)
                mask = torch.arange(S, device=q.device)[None] <= qi
            out.append(torch.nn.functional.scaled_dot_product_attention(q[:, :, s:e], k, v, attn_mask=mask,
                                                                        scale=scale))
        return torch.cat(out, 2)

    def auto_tune_batch_size(self, model: nn.Module, make_input: Callable[[int], Any],
                             latency_budget_ms: Optional[float] = None) -> int:
        """Largest batch (powers of two between min and max) whose latency fits the
        budget and that does not run out of memory."""
        budget = latency_budget_ms or self.config.latency_budget_ms
        best = self.config.min_batch_size
        b = self.config.min_batch_size
        while b <= self.config.max_batch_size:
            try:
                x = make_input(b)
                ms = self.compiler.warmup(model, x if isinstance(x, tuple) else (x,), 3)
            except torch.cuda.OutOfMemoryError:
                self.cleanup_memory(force=True)
                break
            if ms > budget:
                break
            best = b
            b *= 2
        self._optimal_batch = best
        return best

    def get_optimal_batch_size(self) -> Optional[int]:
        return self._optimal_batch

    def cleanup_memory(self, force: bool = False) -> None:
        if not torch.cuda.is_available():
            return
        used = torch.cuda.memory_allocated() / 1e9
        if force or used > self.config.memory_cleanup_threshold * self.config.max_memory_gb:
            gc.collect()
            torch.cuda.empty_cache()


@dataclass
class FrameMetrics:
    """Per generated frame (the reference's fields, inference/optimization.py:821-827,
    plus whether the frame met the latency budget)."""
    frame_idx: int
    generation_time_ms: float
    total_latency_ms: float
    memory_mb: float
    kv_cache_length: int = 0
    meets_deadline: bool = True


class StreamingInference:
    """Chunked streaming generation with per-chunk latency tracking. ``model`` is a
    :class:`~drivedit_b200.models.world_dit.WorldDiT`; frames come from
    :class:`~drivedit_b200.inference.rollout.StreamingRollout`."""

    def __init__(self, model: nn.Module, config: Optional[OptimizationConfig] = None, device: str = "cuda"):
        self.model = model
        self.config = config or OptimizationConfig()
        self.device = torch.device(device)
        self.optimizer = InferenceOptimizer(self.config)
        self.frame_buffer: deque = deque(maxlen=self.config.frame_buffer_size)
        self.frame_metrics: List[FrameMetrics] = []
        self._latency_history: deque = deque(maxlen=100)
        self._frame_deadline_ms = 1000.0 / self.config.target_fps
        self._is_streaming = False

    def initialize(self, num_layers: int = 12, compile_model: bool = False, example_input=None) -> None:
        self.model = self.model.to(self.device).eval()
        self.optimizer.initialize_kv_cache(num_layers, self.device)

    def reset(self) -> None:
        self.frame_buffer.clear()
        self.frame_metrics.clear()
        self._latency_history.clear()
        self.optimizer.reset_kv_cache()
        self._is_streaming = False

    def _rollout(self, total_frames: int):
        from ..config import RolloutConfig
        from .rollout import StreamingRollout

        cfg = RolloutConfig(total_frames=total_frames, chunk_frames=self.config.chunk_size,
                            window_frames=max(8, 2 * self.config.chunk_size))
        return StreamingRollout(self.model, cfg)

    @torch.no_grad()
    def generate_stream(self, context: torch.Tensor, controls: torch.Tensor,
                        num_frames: int) -> Iterator[Tuple[torch.Tensor, FrameMetrics]]:
        """Yields ``(frame [B, C, H, W], metrics)`` for each generated frame."""
        self._is_streaming = True
        Fc = context.shape[1]
        t0 = time.perf_counter()
        ro = self._rollout(Fc + num_frames)
        res = ro.run(context.to(self.device), controls.to(self.device), Fc + num_frames)
        per_frame = [ms / self.config.chunk_size for ms in res.chunk_ms for _ in range(self.config.chunk_size)]
        for i in range(num_frames):
            gen_ms = per_frame[i] if i < len(per_frame) else 0.0
            self._latency_history.append(gen_ms)
            m = FrameMetrics(Fc + i, gen_ms, (time.perf_counter() - t0) * 1000,
                             torch.cuda.memory_allocated(self.device) / 1e6 if self.device.type == "cuda" else 0.0,
                             kv_cache_length=min(Fc + i, ro.cfg.window_frames),  # frames in the KV window
                             meets_deadline=gen_ms <= self._frame_deadline_ms)
            self.frame_metrics.append(m)
            frame = res.frames[:, Fc + i]
            self.frame_buffer.append(frame)
            yield frame, m
        self._is_streaming = False

    def generate_frame(self, context: torch.Tensor, control: torch.Tensor, frame_idx: int = 0):
        ctl = control if control.dim() == 3 else control.unsqueeze(1).expand(-1, context.shape[1] + 1, -1)
        return next(self.generate_stream(context, ctl, 1))

    def generate_batch(self, contexts: torch.Tensor, controls: torch.Tensor, num_frames: int) -> torch.Tensor:
        return torch.stack([f for f, _ in self.generate_stream(contexts, controls, num_frames)], 1)

    def get_streaming_stats(self) -> Dict[str, Any]:
        lat = np.asarray(self._latency_history or [0.0])
        return {"frames": len(self.frame_metrics), "avg_latency_ms": float(lat.mean()),
                "p50_latency_ms": float(np.percentile(lat, 50)), "p95_latency_ms": float(np.percentile(lat, 95)),
                "fps": float(1000.0 / lat.mean()) if lat.mean() > 0 else 0.0,
                "deadline_hit_rate": float(np.mean([m.meets_deadline for m in self.frame_metrics] or [0.0])),
                "target_fps": self.config.target_fps}

    def is_meeting_target_fps(self) -> bool:
        return self.get_streaming_stats()["fps"] >= self.config.target_fps


class MemoryTracker:
    def __init__(self, history_size: int = 1000):
        self.history: deque = deque(maxlen=history_size)

    def record(self, label: str = "") -> Dict[str, float]:
        if torch.cuda.is_available():
            r = {"label": label, "allocated_mb": torch.cuda.memory_allocated() / 1e6,
                 "reserved_mb": torch.cuda.memory_reserved() / 1e6,
                 "peak_mb": torch.cuda.max_memory_allocated() / 1e6}
        else:
            r = {"label": label, "allocated_mb": 0.0, "reserved_mb": 0.0, "peak_mb": 0.0}
        self.history.append(r)
        return r

    def get_peak_memory(self) -> float:
        return max((r["peak_mb"] for r in self.history), default=0.0)

    def get_average_memory(self) -> float:
        return float(np.mean([r["allocated_mb"] for r in self.history])) if self.history else 0.0

    def reset(self) -> None:
        self.history.clear()
        if torch.cuda.is_available():
            torch.cuda.reset_peak_memory_stats()

    def get_report(self) -> Dict[str, Any]:
        return {"peak_mb": self.get_peak_memory(), "avg_mb": self.get_average_memory(), "samples": len(self.history)}


def _time_calls(fn: Callable[[], Any], n: int, device: torch.device) -> List[float]:
    out = []
    for _ in range(n):
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
            out.append((time.perf_counter() - t0) * 1000)
    return out


def benchmark_inference(model: nn.Module, input_shape: Tuple[int, ...], device: str = "cuda",
                        num_warmup: int = 10, num_iterations: int = 100, use_autocast: bool = True,
                        dtype: torch.dtype = torch.bfloat16, verbose: bool = False,
                        make_input: Optional[Callable[[], Sequence[torch.Tensor]]] = None) -> BenchmarkResult:
    dev = torch.device(device)
    model = model.to(dev).eval()
    xs = make_input() if make_input is not None else (torch.randn(input_shape, device=dev),)
    ctx = (torch.autocast(dev.type, dtype=dtype) if use_autocast and dev.type == "cuda"
           else contextlib.nullcontext())
    tracker = MemoryTracker()
    tracker.reset()

    def call():
        with torch.no_grad(), ctx:
            model(*xs)

    _time_calls(call, num_warmup, dev)
    ts = np.asarray(_time_calls(call, num_iterations, dev))
    tracker.record("after")
    B = input_shape[0] if input_shape else 1
    T = input_shape[1] if len(input_shape) > 1 else 1
    r = BenchmarkResult(avg_latency_ms=float(ts.mean()), min_latency_ms=float(ts.min()), max_latency_ms=float(ts.max()),
                        p50_latency_ms=float(np.percentile(ts, 50)), p95_latency_ms=float(np.percentile(ts, 95)),
                        p99_latency_ms=float(np.percentile(ts, 99)), fps=float(B * T * 1000 / ts.mean()),
                        throughput_samples_per_sec=float(B * 1000 / ts.mean()), peak_memory_mb=tracker.get_peak_memory(),
                        avg_memory_mb=tracker.get_average_memory(),
                        memory_reserved_mb=(torch.cuda.memory_reserved() / 1e6 if dev.type == "cuda" else 0.0),
                        batch_size=B, sequence_length=T, warmup_iterations=num_warmup,
                        benchmark_iterations=num_iterations, device=str(dev))
    if verbose:
        print(r.summary())
    return r


def profile_bottlenecks(model: nn.Module, example_input, num_iterations: int = 10, verbose: bool = False,
                        device: Optional[str] = None, top_k: int = 20) -> Dict[str, Any]:
    """Device time per kernel (PyTorch profiler) over ``num_iterations`` forward calls
    (the reference's arguments, inference/optimization.py); the device is the input's
    unless given; ``verbose`` prints the top operations."""
    from torch.profiler import ProfilerActivity, profile

    first = example_input[0] if isinstance(example_input, (tuple, list)) else example_input
    dev = torch.device(device) if device is not None else first.device
    xs = example_input if isinstance(example_input, (tuple, list)) else (example_input,)
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if dev.type == "cuda" else [])
    with torch.no_grad():
        model(*xs)
        with profile(activities=acts) as prof:
            for _ in range(num_iterations):
                model(*xs)
            if dev.type == "cuda":
                torch.cuda.synchronize()
    rows = []
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", 0.0) if dev.type == "cuda" else e.cpu_time_total
        rows.append({"name": e.key, "calls": e.count, "total_ms": t / 1000.0})
    rows.sort(key=lambda r: -r["total_ms"])
    total = sum(r["total_ms"] for r in rows) or 1.0
    for r in rows:
        r["share"] = r["total_ms"] / total
    if verbose:
        for r in rows[:top_k]:
            print(f"{r['total_ms']:10.3f} ms {100 * r['share']:5.1f}%  {r['name']}")
    return {"top_operations": rows[:top_k], "total_ms": total / num_iterations}


def optimize_for_deployment(model: nn.Module, example_input, optimization_level: str = "balanced",
                            verbose: bool = False) -> Tuple[nn.Module, Dict[str, Any]]:
    """``minimal``: eval + bf16; ``balanced`` / ``aggressive``: also a CUDA graph of the
    forward for the example shapes."""
    if optimization_level not in ("minimal", "balanced", "aggressive"):
        raise ValueError(f"unknown optimization level {optimization_level!r}")
    xs = example_input if isinstance(example_input, (tuple, list)) else (example_input,)
    dev = xs[0].device
    report: Dict[str, Any] = {"optimizations_applied": ["eval"]}
    model = model.eval()
    call = lambda m: (lambda: m(*xs))
    with torch.no_grad():
        report["original_latency_ms"] = float(np.mean(_time_calls(call(model), 5, dev)))
        cfg = OptimizationConfig(compile_mode=CompileMode.NONE if optimization_level == "minimal"
                                 else CompileMode.REDUCE_OVERHEAD)
        opt = InferenceOptimizer(cfg).optimize_model(model, xs if dev.type == "cuda" else None)
        if opt is not model:
            report["optimizations_applied"].append("cuda_graph")
        report["optimized_latency_ms"] = float(np.mean(_time_calls(call(opt), 5, dev)))
    report["speedup"] = report["original_latency_ms"] / max(report["optimized_latency_ms"], 1e-9)
    if verbose:
        print(report)
    return opt, report


def compare_optimization_modes(model: nn.Module, input_shape: Tuple[int, ...], device: str = "cuda",
                               verbose: bool = False) -> Dict[str, BenchmarkResult]:
    dev = torch.device(device)
    x = torch.randn(input_shape, device=dev)
    results = {"baseline": benchmark_inference(model, input_shape, device, 3, 10, use_autocast=False)}
    if dev.type == "cuda":
        results["bf16"] = benchmark_inference(model, input_shape, device, 3, 10, use_autocast=True)
        g = ModelCompiler(OptimizationConfig()).compile(model, (x,))
        results["cuda_graph_bf16"] = benchmark_inference(g, input_shape, device, 3, 10, use_autocast=False)
    if verbose:
        for k, r in results.items():
            print(k, f"{r.avg_latency_ms:.3f} ms")
    return results
