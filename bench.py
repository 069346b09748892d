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
whole-job token rate. ``e2e`` repeats the measurement (same step count) through the
public trainer API with each step's inputs copied from pinned host memory and the loss
read back. ``extras`` adds, unless ``--no-extras``: MoE DiT-L training tok/s (fsdp +
expert parallel over the job's ranks) and streaming-rollout frames/s with p50 / p99
chunk latency at batch 1 and 16 (tensor parallel over the job's ranks). Rank 0 prints
one JSON line. ``--impl reference`` runs the reference arm (``baseline/reference_arm.py``)
and prints the same line with ``"impl": "reference"``.
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


def init_dist(ws, local, timeout_s=300):
    torch.cuda.set_device(local)
    if ws > 1 and not dist.is_initialized():
        import datetime

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))


def check_device_free(rank, local, min_free_frac=0.5, wait_s=120.0):
    """Print this rank's free / total device memory. A GPU that another process still
    fills (a job that is being torn down) is polled every 2 s for up to ``wait_s``
    seconds; the run refuses to start if the memory is not released by then."""
    t0 = time.time()
    while True:
        free, total = torch.cuda.mem_get_info(local)
        if free >= min_free_frac * total or time.time() - t0 >= wait_s:
            break
        if time.time() - t0 < 2.5:
            print(f"[rank {rank}] cuda:{local} free {free / 2**30:.1f} GiB: waiting for "
                  f"another process to release the GPU", file=sys.stderr, flush=True)
        time.sleep(2.0)
    print(f"[rank {rank}] cuda:{local} free {free / 2**30:.1f} / {total / 2**30:.1f} GiB",
          file=sys.stderr, flush=True)
    if free < min_free_frac * total:
        raise RuntimeError(f"rank {rank}: cuda:{local} has only {free / 2**30:.1f} GiB of "
                           f"{total / 2**30:.1f} GiB free after {wait_s:.0f} s; another "
                           f"process holds the GPU")


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
def _gpu_index(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(vis.split(",")[local]) if vis else local


def _train_throughput(cfg_name, overrides, steps, warmup, ws, rank, local, e2e_steps=0,
                      clocks=False):
    """Device-timed training throughput of one preset through the public trainer API.

    Returns (result dict, trainer summary dict). ``e2e_steps`` > 0 adds the end-to-end
    measurement (pinned host batch copied in, loss read back, every step)."""
    from drivedit_b200.config import get_config
    from drivedit_b200.data.synthetic import make_batch
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.ops._ext import check_device_status
    from drivedit_b200.training.trainer import WorldModelTrainer

    cfg = get_config(cfg_name, overrides)
    torch.manual_seed(cfg.train.seed + rank)
    dev = torch.device("cuda", local)
    with torch.device(dev):  # random init on the device (the 2B-active MoE has 9.4B params)
        model = WorldDiT(cfg.model)
    trainer = WorldModelTrainer(model, cfg.train, dev,
                                process_group=dist.group.WORLD if ws > 1 else None)
    B, Fr = cfg.train.batch_per_gpu, cfg.train.frames
    tokens_per_step = B * Fr * cfg.model.tokens_per_frame
    gen = torch.Generator().manual_seed(1234 + rank)
    rgb = Fr if cfg.model.repa is not None else 0  # REPA teacher frames (RGB ~U[0,1])
    dev_batch = make_batch(cfg, device=dev, generator=gen, rgb_frames=rgb)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev, dtype=torch.float32)

    for _ in range(warmup):
        trainer.train_step(dev_batch)
    torch.cuda.synchronize()
    check_device_status()

    barrier()
    torch.cuda.synchronize()
    n0 = launch_count()
    clk = ClockSampler(_gpu_index(local)) if clocks else None
    if clk is not None:
        clk.__enter__()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        flush.zero_()
        loss = trainer.train_step(dev_batch)
    end.record()
    torch.cuda.synchronize()
    if clk is not None:
        clk.__exit__()
    barrier()
    n_launch = launch_count() - n0  # this extension's kernels only (the L2 flush is not one)
    ms = max_over_ranks(start.elapsed_time(end) / steps)
    check_device_status()
    peak = max_over_ranks(torch.cuda.max_memory_allocated(dev) / 2**30)
    out = {"ms_per_step": ms, "value": ws * tokens_per_step / (ms / 1000.0),
           "gpu_launches": n_launch, "tokens_per_step_per_gpu": tokens_per_step,
           "final_loss": float(loss.item()), "peak_mem_gib": round(peak, 1)}
    if clk is not None:
        out["clocks"] = clk.summary()

    if e2e_steps > 0:
        # end to end through the public API: pinned host inputs in, loss out, every step
        host = [make_batch(cfg, generator=gen, pin=True, rgb_frames=rgb) for _ in range(2)]
        h2d = host[0].nbytes()
        barrier()
        torch.cuda.synchronize()
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
        out["e2e"] = {"value": round(ws * tokens_per_step / (e2e_ms / 1000.0), 1),
                      "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                      "ms_per_step": round(e2e_ms, 3), "steps": e2e_steps}
        out["final_loss"] = losses[-1]
    summary = {
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
        "repa": cfg.model.repa is not None,
    }
    trainer.close()
    del trainer, model, dev_batch, flush
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out, summary


def _rollout_ours(batch, ws):
    """Streaming rollout of the causal DiT-B student: tensor parallel over the job's
    ranks when ws > 1 (fused all-gather / reduce-scatter GEMMs)."""
    from drivedit_b200.inference.bench_rollout import run

    res = run(batch, 120)
    return {"batch": batch, "frames_per_s": res["value"], "p50_chunk_ms": res["p50_chunk_ms"],
            "p99_chunk_ms": res["p99_chunk_ms"], "chunks": res["chunks"],
            "tensor_parallel": res["tensor_parallel"]}


def run_ours(args, ws, rank, local):
    sys.path.insert(0, ROOT)
    res, summary = _train_throughput(args.config, args.override, args.steps, args.warmup, ws,
                                     rank, local, e2e_steps=args.steps, clocks=True)
    value, ms = res["value"], res["ms_per_step"]
    summary["l2"] = ("256 MiB buffer overwritten before every timed step "
                     "(device-timed and end-to-end)")
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
            if summary["repa"] else ""),
        "config": summary,
        "clocks": res["clocks"],
        "e2e": res["e2e"],
        "gpu_launches": res["gpu_launches"],
        "final_loss": res["final_loss"],
        "peak_mem_gib_per_gpu": res["peak_mem_gib"],
    }
    if not args.no_extras:
        extras = {}
        # MoE DiT-L (fsdp + expert parallel over the job's ranks)
        mres, msum = _train_throughput("moe_dit_l", [], args.extra_steps, 3, ws, rank, local)
        extras["moe_dit_l"] = {"value": round(mres["value"], 1), "unit": "tok/s",
                               "ms_per_step": round(mres["ms_per_step"], 3),
                               "steps": args.extra_steps, "warmup": 3,
                               "gpu_launches": mres["gpu_launches"],
                               "parallelism": msum["parallelism"],
                               "global_batch": msum["global_batch"],
                               "seq_len": msum["seq_len"]}
        # streaming rollout (frames/s, p50 / p99 chunk latency)
        extras["rollout"] = [_rollout_ours(b, ws) for b in (1, 16)]
        out["extras"] = extras
    if rank == 0:
        print(json.dumps(out), flush=True)


# --------------------------------------------------------------------------- reference arm
def run_reference(args, ws, rank, local):
    from baseline.reference_arm import run, run_rollout

    out = run(args, ws, rank, local)
    if not args.no_extras and out is not None:
        extras = {}
        rolls = []
        for b in (1, 16):
            r = run_rollout(b)
            if "frames_per_s" in r:
                # every rank runs its own rollouts (the reference has no tensor
                # parallelism): the slowest rank's rate, times the ranks
                per = max_over_ranks(1.0 / r["frames_per_s"])
                r["frames_per_s_per_rank"] = round(1.0 / per, 2)
                r["frames_per_s"] = round(ws / per, 2)
                r["tensor_parallel"] = 1
                r["replicas"] = ws
            rolls.append(r)
        extras["rollout"] = rolls
        out["extras"] = extras
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--extra-steps", type=int, default=10,
                   help="timed steps of the extra workloads (MoE DiT-L)")
    p.add_argument("--no-extras", action="store_true",
                   help="only the headline DiT-B training number")
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
    try:
        check_device_free(rank, local)
        init_dist(ws, local)
        if args.impl == "reference":
            run_reference(args, ws, rank, local)
        else:
            run_ours(args, ws, rank, local)
    except BaseException:
        # every rank reports its own failure before it exits non-zero
        import traceback

        print(f"[rank {rank}/{ws}] bench.py ({args.impl}) failed:\n{traceback.format_exc()}",
              file=sys.stderr, flush=True)
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    from torch.distributed.elastic.multiprocessing.errors import record

    record(main)()
