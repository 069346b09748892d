"""Training-throughput benchmark: latent tokens/s of the DiT-B world model (SLA attention).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config dit_b] [--impl ours|reference]

For N > 1 launch one rank per GPU (``torchrun --nproc-per-node N ... bench.py --gpus N``).
Workload (``dit_b`` preset): 12 layers, d=768, 12 heads, SwiGLU 3072, AdaLN, 3-D RoPE,
frame-causal SLA (64x64 blocks, top 12.5 %); per GPU a batch of 8 clips of 16 latent
frames x 16 ch x 32x64 (patch 2 -> 512 tokens/frame, 8192 tokens/clip), 3-D actions,
logit-normal flow time, velocity-MSE loss, AdamW. Synthetic data, random-init weights.

Timing: W untimed warm-up steps, then K steps between a barrier + device sync on each
side, timed with CUDA events on the training stream; each step first overwrites a
256 MiB buffer to flush L2. The reported ms/step is the max over ranks; ``value`` is the
whole-job token rate. ``e2e`` repeats the measurement through the public trainer API
with each step's inputs copied from pinned host memory and the loss read back.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "train latent tok/s (max over ranks)"
BASELINE_VALUE = None  # the reference publishes no measured number
L2_FLUSH_BYTES = 256 << 20


# --------------------------------------------------------------------------- helpers
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, local):
    torch.cuda.set_device(local)
    if ws > 1 and not dist.is_initialized():
        import datetime

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))


def max_over_ranks(x: float) -> float:
    if dist.is_initialized():
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier():
    if dist.is_initialized():
        dist.barrier()


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def launch_count():
    try:
        from drivedit_b200.ops._ext import ext

        return int(ext().launch_count())
    except Exception:
        return 0


# --------------------------------------------------------------------------- our arm
def run_ours(args, ws, rank, local):
    sys.path.insert(0, ROOT)
    from drivedit_b200.config import get_config
    from drivedit_b200.data.synthetic import make_batch
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.ops._ext import check_device_status
    from drivedit_b200.training.trainer import WorldModelTrainer

    cfg = get_config(args.config, args.override)
    torch.manual_seed(cfg.train.seed + rank)
    dev = torch.device("cuda", local)
    model = WorldDiT(cfg.model)
    trainer = WorldModelTrainer(model, cfg.train, dev,
                                process_group=dist.group.WORLD if ws > 1 else None)
    B, Fr = cfg.train.batch_per_gpu, cfg.train.frames
    tokens_per_step = B * Fr * cfg.model.tokens_per_frame
    gen = torch.Generator().manual_seed(1234 + rank)
    rgb = Fr if cfg.model.repa is not None else 0  # REPA teacher frames (RGB ~U[0,1])
    dev_batch = make_batch(cfg, device=dev, generator=gen, rgb_frames=rgb)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev, dtype=torch.float32)

    for _ in range(args.warmup):
        trainer.train_step(dev_batch)
    torch.cuda.synchronize()
    check_device_status()

    barrier()
    torch.cuda.synchronize()
    n0 = launch_count()
    with ClockSampler(local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                      int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])) as clk:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            flush.zero_()
            loss = trainer.train_step(dev_batch)
        end.record()
        torch.cuda.synchronize()
    barrier()
    n_launch = launch_count() - n0  # this extension's kernels only (the L2 flush is not one)
    ms = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms)
    check_device_status()

    # ---- end to end through the public API: pinned host inputs in, loss out
    host = [make_batch(cfg, generator=gen, pin=True, rgb_frames=rgb) for _ in range(2)]
    h2d = host[0].nbytes()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    s2 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    s2.record()
    losses = []
    for i in range(e2e_steps):
        flush.zero_()  # same cold-L2 start as the device-timed steps
        b = host[i % 2].to(dev, non_blocking=True)
        losses.append(float(trainer.train_step(b).item()))
    e2.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / e2e_steps)
    barrier()

    value = ws * tokens_per_step / (ms / 1000.0)
    e2e_value = ws * tokens_per_step / (e2e_ms / 1000.0)
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tok/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
        "dtype": "bf16",
        "data": "synthetic latents/actions/flow-time, random-init weights" + (
            ", RGB frames ~U[0,1] for the random-init frozen ViT-L REPA teacher"
            if cfg.model.repa is not None else ""),
        "config": {
            "model": cfg.model.name,
            "layers": cfg.model.n_layers, "d_model": cfg.model.d_model,
            "heads": cfg.model.n_heads, "mlp_hidden": cfg.model.mlp_hidden,
            "attention": cfg.model.attention,
            "global_batch": B * ws, "seq_len": Fr * cfg.model.tokens_per_frame,
            "frames": Fr, "latent": [cfg.model.latent_channels, cfg.model.latent_h,
                                     cfg.model.latent_w],
            "parallelism": (f"fsdp{ws}+ep{ws}" if trainer.ep is not None else f"fsdp{ws}")
                           if ws > 1 else "single",
            "sharding": (("gradients reduce-scattered and weights all-gathered by the fused "
                          "NVLink optimizer kernel" if trainer.engine.transport == "fused" else
                          "NCCL reduce_scatter / all_gather around a local AdamW")
                         + "; AdamW state sharded") if ws > 1 else None,
            "expert_parallel": None if trainer.ep is None else (
                f"{cfg.model.moe.num_experts // ws} routed experts per rank; token rows "
                + ("pushed once per owner over NVLink peer memory (P2P stores) by the EP kernels"
                   if trainer.ep.transport == "fused" else "exchanged by NCCL all_to_all")),
            "l2": "256 MiB buffer overwritten before every timed step (device-timed and end-to-end)",
        },
        "clocks": clk.summary(),
        "e2e": {"value": round(e2e_value, 1), "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": n_launch,
        "final_loss": losses[-1] if losses else None,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)


# --------------------------------------------------------------------------- reference arm
def run_reference(args, ws, rank, local):
    from baseline.reference_arm import run

    out = run(args, ws, rank, local)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--config", default="dit_b")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("override", nargs="*", help="config overrides key=value")
    args = p.parse_args()
    if args.warmup < 3:
        args.warmup = 3  # timing rules: at least 3 warm-up steps
    ws, rank, local = dist_env()
    if ws != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={ws}", file=sys.stderr)
    if not torch.cuda.is_available():
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "no CUDA device"}))
        else:
            print(json.dumps({"metric": METRIC, "unavailable": "no CUDA device"}))
        return
    init_dist(ws, local)
    try:
        if args.impl == "reference":
            run_reference(args, ws, rank, local)
        else:
            run_ours(args, ws, rank, local)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
