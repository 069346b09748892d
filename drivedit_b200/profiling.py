"""Profiling tools: training-step throughput, a per-kernel time breakdown of one step, and
a static dead-code report of the package.

``python -m drivedit_b200.profiling step --config moe_dit_l [key=value ...]``
    times ``--steps`` training steps with CUDA events (after ``--warmup``) and then records
    one more step with the PyTorch profiler (CUPTI kernel records) to list the kernels by
    total device time, grouped by name, with their share of the step.
``python -m drivedit_b200.profiling cpu-step [--config tiny] [--steps 30]``
    the fp32 CPU training step (forward, backward, AdamW) of a preset, median wall time
    over ``--steps`` after ``--warmup``; the ``tiny`` preset is the 4-layer d256 workload
    on which the reference's own modules run at 6,902 latent tok/s (74.2 ms/step) on this
    machine class (an 8-thread 2.7 GHz Xeon).
``python -m drivedit_b200.profiling deadcode [package_dir]``
    functions and classes defined in the package that no other module names.

The reference's ``scripts/profile_codebase.py`` has the same two roles (an AST dead-code
detector :43-145 and a ``ThroughputProfiler`` :152-340); this module measures on the
device and attributes time to this framework's own kernels.
"""
from __future__ import annotations

import argparse
import ast
import json
import os
import sys
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class StepProfile:
    config: str
    ms_per_step: float
    tokens_per_s: float
    kernels: List[Dict] = field(default_factory=list)   # name, calls, total_ms, share

    def table(self, top: int = 25) -> str:
        lines = [f"{self.config}: {self.ms_per_step:.2f} ms/step, {self.tokens_per_s:,.0f} tok/s",
                 f"{'kernel':70s} {'calls':>6s} {'ms':>9s} {'share':>7s}"]
        for k in self.kernels[:top]:
            lines.append(f"{k['name'][:70]:70s} {k['calls']:6d} {k['total_ms']:9.3f} {100 * k['share']:6.1f}%")
        return "\n".join(lines)


class ThroughputProfiler:
    """Times training steps of a preset on one GPU with CUDA events."""

    def __init__(self, config: str = "dit_b", overrides: Optional[List[str]] = None, device="cuda:0"):
        import torch

        from .config import get_config
        from .data.synthetic import make_batch
        from .models.world_dit import WorldDiT
        from .training.trainer import WorldModelTrainer

        self.cfg = get_config(config, overrides or [])
        self.name = config
        torch.manual_seed(self.cfg.train.seed)
        self.device = torch.device(device)
        self.model = WorldDiT(self.cfg.model)
        self.trainer = WorldModelTrainer(self.model, self.cfg.train, self.device)
        rgb = self.cfg.train.frames if self.cfg.model.repa is not None else 0
        self.batch = make_batch(self.cfg, device=self.device, generator=torch.Generator().manual_seed(0),
                                rgb_frames=rgb)
        self.tokens = self.cfg.train.batch_per_gpu * self.cfg.train.frames * self.cfg.model.tokens_per_frame

    def time_steps(self, steps: int = 5, warmup: int = 3) -> float:
        import torch

        for _ in range(warmup):
            self.trainer.train_step(self.batch)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            self.trainer.train_step(self.batch)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / steps

    def kernel_breakdown(self) -> List[Dict]:
        """One step under the PyTorch profiler: device time per kernel name."""
        import torch
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            self.trainer.train_step(self.batch)
            torch.cuda.synchronize()
        agg: Dict[str, List[float]] = defaultdict(lambda: [0, 0.0])
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                a = agg[ev.name]
                a[0] += 1
                a[1] += ev.device_time_total / 1000.0 if hasattr(ev, "device_time_total") else ev.cuda_time_total / 1000.0
        total = sum(v[1] for v in agg.values()) or 1.0
        rows = [{"name": n, "calls": int(c), "total_ms": t, "share": t / total} for n, (c, t) in agg.items()]
        rows.sort(key=lambda r: -r["total_ms"])
        return rows

    def run(self, steps: int = 5, warmup: int = 3) -> StepProfile:
        ms = self.time_steps(steps, warmup)
        return StepProfile(self.name, ms, self.tokens / (ms / 1000.0), self.kernel_breakdown())


# ----------------------------------------------------------------------------- CPU step
REFERENCE_TINY_CPU_TOK_S = 6902.0  # reference modules, same workload, measured on this CPU class


def cpu_step(config: str = "tiny", steps: int = 30, warmup: int = 5, overrides=None) -> Dict:
    """Median wall time of the fp32 CPU training step of a preset."""
    import statistics
    import time

    import torch

    from .config import get_config
    from .data.synthetic import make_batch
    from .models.world_dit import WorldDiT
    from .training.trainer import WorldModelTrainer

    cfg = get_config(config, overrides)
    cfg.train.dtype = "fp32"
    torch.manual_seed(cfg.train.seed)
    tr = WorldModelTrainer(WorldDiT(cfg.model), cfg.train, "cpu")
    batch = make_batch(cfg, generator=torch.Generator().manual_seed(0))
    tokens = cfg.train.batch_per_gpu * cfg.train.frames * cfg.model.tokens_per_frame
    for _ in range(warmup):
        tr.train_step(batch)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        tr.train_step(batch)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    out = {"config": config, "device": "cpu", "dtype": "fp32", "threads": torch.get_num_threads(),
           "tokens_per_step": tokens, "ms_per_step": round(med * 1000, 2),
           "tokens_per_s": round(tokens / med, 1)}
    if config == "tiny" and not overrides:
        out["reference_tokens_per_s"] = REFERENCE_TINY_CPU_TOK_S
        out["vs_reference"] = round(out["tokens_per_s"] / REFERENCE_TINY_CPU_TOK_S, 3)
    return out


# ----------------------------------------------------------------------------- dead code
def dead_code(package_dir: str) -> List[str]:
    """``module:line name`` of top-level functions / classes (and methods not starting
    with an underscore) that no file of the package mentions outside their definition."""
    defs = []
    sources = {}
    for root, _, files in os.walk(package_dir):
        for f in files:
            if f.endswith(".py"):
                p = os.path.join(root, f)
                with open(p) as fh:
                    sources[p] = fh.read()
    for p, src in sources.items():
        try:
            tree = ast.parse(src)
        except SyntaxError:
            continue
        for node in ast.walk(tree):
            if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
                if node.name.startswith("__"):
                    continue
                defs.append((p, node.lineno, node.name))
    text = "\n".join(sources.values())
    out = []
    for p, line, name in defs:
        if text.count(name) <= 1:
            out.append(f"{os.path.relpath(p, package_dir)}:{line} {name}")
    return sorted(out)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    st = sub.add_parser("step")
    st.add_argument("--config", default="dit_b")
    st.add_argument("--steps", type=int, default=5)
    st.add_argument("--warmup", type=int, default=3)
    st.add_argument("--top", type=int, default=30)
    st.add_argument("--json", default=None, help="write the breakdown as JSON here")
    st.add_argument("override", nargs="*")
    cs = sub.add_parser("cpu-step")
    cs.add_argument("--config", default="tiny")
    cs.add_argument("--steps", type=int, default=30)
    cs.add_argument("--warmup", type=int, default=5)
    cs.add_argument("override", nargs="*")
    dc = sub.add_parser("deadcode")
    dc.add_argument("package", nargs="?", default=os.path.dirname(os.path.abspath(__file__)))
    a = ap.parse_args(argv)
    if a.cmd == "cpu-step":
        print(json.dumps(cpu_step(a.config, a.steps, a.warmup, a.override or None)))
        return 0
    if a.cmd == "deadcode":
        for line in dead_code(a.package):
            print(line)
        return 0
    prof = ThroughputProfiler(a.config, a.override).run(a.steps, a.warmup)
    print(prof.table(a.top))
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"config": prof.config, "ms_per_step": prof.ms_per_step,
                       "tokens_per_s": prof.tokens_per_s, "kernels": prof.kernels}, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
