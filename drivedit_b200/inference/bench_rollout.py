"""Streaming-rollout benchmark: frames/s and per-chunk latency (p50 / p99).

    python -m drivedit_b200.inference.bench_rollout [--batch 1 16] [--frames 120]
    torchrun --nproc-per-node N -m drivedit_b200.inference.bench_rollout [--tp-transport fused|nccl]

Workload (``rollout_dit_b`` preset): the causal DiT-B student (12 layers, d=768, 12 heads,
frame-causal attention, 3-D RoPE), 4 context frames ~N(0,1), then 116 more latent frames of
16 ch x 32x64 (512 tokens) generated in chunks of 4 frames with 4 Euler flow steps per chunk
and a 32-frame rolling KV window; 3-D actions ~U[-1,1]; random-init weights; bf16.
Per-chunk latency is device time (CUDA events) around the 4 denoising forwards plus the
cache-fill forward; frames/s = batch * generated frames / sum of chunk times. One JSON
line per batch size. Under torchrun the model runs tensor-parallel over the N ranks
(:mod:`drivedit_b200.parallel.tensor`); chunk times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch


def run(batch: int, frames: int, warm_chunks: int = 2, overrides=None, tp_transport: str = "fused"):
    from ..config import get_config
    from ..models.world_dit import WorldDiT
    from ..parallel.flat import FlatParamGroup
    from .rollout import StreamingRollout

    cfg = get_config("rollout_dit_b", overrides)
    torch.manual_seed(0)
    model = WorldDiT(cfg.model).cuda().eval()
    group = FlatParamGroup(model.flat_layout(model.named_parameters()), "cuda")
    model.enable_fused(group=group)
    tp = None
    world = 1
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size() > 1:
        from ..parallel.tensor import TensorParallelWorldDiT

        world = dist.get_world_size()
        tp = TensorParallelWorldDiT(model, transport=tp_transport)
    r = StreamingRollout(tp if tp is not None else model, cfg.rollout)
    m = cfg.model
    g = torch.Generator(device="cuda").manual_seed(1)
    ctx = torch.randn(batch, cfg.rollout.context_frames, m.latent_channels, m.latent_h, m.latent_w,
                      device="cuda", generator=g)
    act = torch.rand(batch, frames, m.action_dim, device="cuda", generator=g) * 2 - 1
    # warm-up: a short rollout (kernels, tensor maps, allocator)
    r.run(ctx, act, total_frames=cfg.rollout.context_frames + warm_chunks * cfg.rollout.chunk_frames,
          generator=g)
    torch.cuda.synchronize()
    res = r.run(ctx, act, total_frames=frames, generator=g)
    torch.cuda.synchronize()
    from ..ops._ext import check_device_status

    check_device_status()
    if world > 1:
        ms = torch.tensor(res.chunk_ms, device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        res.chunk_ms = ms.tolist()
        tp.close()
    return {
        "metric": "rollout frames/s",
        "value": round(res.frames_per_s(batch, cfg.rollout.chunk_frames), 2),
        "unit": "frames/s",
        "batch": batch,
        "frames": frames,
        "chunk_frames": cfg.rollout.chunk_frames,
        "flow_steps": cfg.rollout.flow_steps,
        "window_frames": cfg.rollout.window_frames,
        "chunks": len(res.chunk_ms),
        "p50_chunk_ms": round(res.percentile_ms(50), 3),
        "p99_chunk_ms": round(res.percentile_ms(99), 3),
        "chunk_ms": [round(x, 3) for x in res.chunk_ms],
        "dtype": "bf16",
        "data": "synthetic context latents/actions, random-init weights",
        "model": cfg.model.name,
        "tensor_parallel": world,
        "tp_transport": tp_transport if world > 1 else None,
    }


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, nargs="+", default=[1, 16])
    p.add_argument("--frames", type=int, default=120)
    p.add_argument("--tp-transport", default="fused")
    p.add_argument("--kv-splits", type=int, default=0,
                   help="attention split-KV: 0 = chosen per launch, n >= 1 = n splits")
    p.add_argument("override", nargs="*")
    a = p.parse_args()
    if not torch.cuda.is_available():
        print(json.dumps({"metric": "rollout frames/s", "unavailable": "no CUDA device"}))
        return
    import os

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if a.kv_splits:
        from ..ops._ext import ext

        ext().attn_fwd_set_kv_splits(a.kv_splits)
    for b in a.batch:
        out = run(b, a.frames, overrides=a.override, tp_transport=a.tp_transport)
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(out), flush=True)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
