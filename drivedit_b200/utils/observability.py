"""Observability: JSONL metrics (per rank + rank-0 aggregate), NVTX ranges, device
timers and a torch.profiler wrapper.

NVTX ranges are free when ``DDB_NVTX`` is unset; with ``DDB_NVTX=1`` every
``nvtx_range`` (blocks, collectives, optimizer) is visible in Nsight timelines.
"""
from __future__ import annotations

import contextlib
import json
import os
import time
from pathlib import Path
from typing import Any, Dict, Iterator, List, Optional

import torch

_NVTX = os.environ.get("DDB_NVTX", "0") not in ("", "0")


@contextlib.contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class DeviceTimer:
    """CUDA-event interval timer on the current stream (wall clock on CPU)."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled and torch.cuda.is_available()
        self.intervals: Dict[str, List[Any]] = {}

    @contextlib.contextmanager
    def time(self, name: str):
        if self.enabled:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            yield
            e.record()
            self.intervals.setdefault(name, []).append((s, e))
        else:
            t0 = time.perf_counter()
            yield
            self.intervals.setdefault(name, []).append((time.perf_counter() - t0) * 1000.0)

    def summary(self) -> Dict[str, float]:
        """ms per interval name (synchronises once)."""
        if self.enabled:
            torch.cuda.synchronize()
        out = {}
        for k, v in self.intervals.items():
            ms = [s.elapsed_time(e) if isinstance(s, torch.cuda.Event) else s for s, e in
                  ((x if isinstance(x, tuple) else (x, None)) for x in v)]
            out[k] = sum(ms) / len(ms)
        self.intervals.clear()
        return out


class MetricsLogger:
    """Appends one JSON object per ``log`` call to ``<dir>/metrics_rank{r}.jsonl``; rank 0
    also writes ``metrics.jsonl`` with values averaged over ranks (one all-reduce)."""

    def __init__(self, log_dir: str, rank: int = 0, world_size: int = 1, config: Optional[Dict] = None):
        self.dir = Path(log_dir)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.rank, self.world_size = rank, world_size
        self.f_rank = open(self.dir / f"metrics_rank{rank}.jsonl", "a")
        self.f_all = open(self.dir / "metrics.jsonl", "a") if rank == 0 else None
        if config is not None and rank == 0:
            (self.dir / "config.json").write_text(json.dumps(config, indent=2, default=str))

    def log(self, step: int, metrics: Dict[str, Any], aggregate: bool = True) -> Dict[str, float]:
        vals = {k: float(v) for k, v in metrics.items()}
        rec = {"step": step, "time": time.time(), "rank": self.rank, **vals}
        self.f_rank.write(json.dumps(rec) + "\n")
        self.f_rank.flush()
        agg = vals
        if aggregate and self.world_size > 1:
            from ..training.distributed import reduce_dict

            agg = reduce_dict(vals, self.world_size)
        if self.f_all is not None:
            self.f_all.write(json.dumps({"step": step, "time": time.time(), **agg}) + "\n")
            self.f_all.flush()
        return agg

    def close(self):
        self.f_rank.close()
        if self.f_all is not None:
            self.f_all.close()


def profile_steps(fn, steps: int = 5, warmup: int = 2, trace_dir: Optional[str] = None, row_limit: int = 20) -> str:
    """Runs ``fn()`` under torch.profiler (CPU + CUDA activities); returns the top
    ``row_limit`` ops by device time (the reference's profile_bottlenecks report)."""
    from torch.profiler import ProfilerActivity, profile, schedule

    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    kw = {}
    if trace_dir:
        from torch.profiler import tensorboard_trace_handler

        kw["on_trace_ready"] = tensorboard_trace_handler(trace_dir)
    with profile(activities=acts, schedule=schedule(wait=0, warmup=warmup, active=steps), **kw) as prof:
        for _ in range(warmup + steps):
            fn()
            prof.step()
    key = "self_cuda_time_total" if torch.cuda.is_available() else "self_cpu_time_total"
    return prof.key_averages().table(sort_by=key, row_limit=row_limit)
