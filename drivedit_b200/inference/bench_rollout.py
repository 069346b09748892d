"""Streaming-rollout benchmark: frames/s and per-chunk latency (p50 / p99).

    python -m drivedit_b200.inference.bench_rollout [--batch 1 16] [--frames 120]

Workload (``rollout_dit_b`` preset): the causal DiT-B student (12 layers, d=768, 12 heads,
frame-causal attention, 3-D RoPE), 4 context frames ~N(0,1), then 116 more latent frames of
16 ch x 32x64 (512 tokens) generated in chunks of 4 frames with 4 Euler flow steps per chunk
and a 32-frame rolling KV window; 3-D actions ~U[-1,1]; random-init weights; bf16.
Per-chunk latency is device time (CUDA events) around the 4 denoising forwards plus the
cache-fill forward; frames/s = batch * generated frames / sum of chunk times. One JSON
line per batch size.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch


def run(batch: int, frames: int, warm_chunks: int = 2, overrides=None):
    from ..config import get_config
    from ..models.world_dit import WorldDiT
    from ..parallel.flat import FlatParamGroup
    from .rollout import StreamingRollout

    cfg = get_config("rollout_dit_b", overrides)
    torch.manual_seed(0)
    model = WorldDiT(cfg.model).cuda().eval()
    group = FlatParamGroup(model.named_parameters(), "cuda")
    model.enable_fused(group=group)
    r = StreamingRollout(model, cfg.rollout)
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
        "dtype": "bf16",
        "data": "synthetic context latents/actions, random-init weights",
        "model": cfg.model.name,
    }


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, nargs="+", default=[1, 16])
    p.add_argument("--frames", type=int, default=120)
    p.add_argument("override", nargs="*")
    a = p.parse_args()
    if not torch.cuda.is_available():
        print(json.dumps({"metric": "rollout frames/s", "unavailable": "no CUDA device"}))
        return
    for b in a.batch:
        print(json.dumps(run(b, a.frames, overrides=a.override)), flush=True)


if __name__ == "__main__":
    main()
