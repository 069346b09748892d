"""Reference arm of ``bench.py``: the unmodified reference (installed under
``baseline/_ref``) trained through its own modules and its own trainer.

The model is assembled from the reference's public building blocks at the DiT-B shape:
``blocks.dit_block.DiTBlock`` (AdaLN conditioning, SwiGLU, 1-D RoPE) with its attention
swapped for the reference's drop-in ``layers.sla.CausalSparseLinearAttention``
(64-token blocks), ``blocks.flow_matching.TimestepEmbedding`` for the flow time and
``layers.nn_helpers.RMSNorm`` for the head. Multi-GPU runs wrap the model with the
reference's own FSDP wrapper (``OptimizedTrainer._wrap_fsdp``, training/cuda_optimized.py
:571-615: FULL_SHARD, bf16 params / fp32 reduce, 1M-parameter auto-wrap) and the
optimizer is the reference's ``create_optimized_optimizer`` (fused AdamW with decay /
no-decay groups). The step is bf16 autocast forward, MSE, backward, clip 1.0, AdamW —
the body of ``OptimizedTrainer.train_step``. ``OptimizedTrainer.__init__`` itself cannot
run on this PyTorch: it calls ``torch.cuda.amp.autocast(device_type=...)``, which raises
TypeError (training/cuda_optimized.py:19,518), so its step is reproduced here without
torch.compile (whose autotuning of the reference's Python SLA block loop would not
finish) and without activation checkpointing. The only glue code is patchify /
unpatchify, the action MLP and the loss.
"""
from __future__ import annotations

import os
import sys
import time

import torch
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _unavailable(why):
    return {"impl": "reference", "unavailable": why}


def build(cfg, device):
    sys.path.insert(0, REF)
    from blocks.dit_block import DiTBlock
    from blocks.flow_matching import TimestepEmbedding
    from layers.nn_helpers import RMSNorm
    from layers.sla import CausalSparseLinearAttention, SLAConfig

    m = cfg.model
    T = cfg.train.frames * m.tokens_per_frame

    class RefWorldDiT(nn.Module):
        def __init__(self):
            super().__init__()
            d = m.d_model
            self.patch_embed = nn.Linear(m.patch_dim, d)
            self.t_embed = TimestepEmbedding(d)
            self.a_embed = nn.Sequential(nn.Linear(m.action_dim, d), nn.SiLU(), nn.Linear(d, d))
            blocks = []
            for _ in range(m.n_layers):
                blk = DiTBlock(d, m.n_heads, d_ff=m.mlp_hidden, mlp_type="swiglu", causal=True,
                               max_seq_len=T, cond_dim=d)
                if m.attention == "sla":
                    blk.attn = CausalSparseLinearAttention(
                        d, m.n_heads, SLAConfig(block_size=m.sla.block_size, causal=True),
                        rope_layer=blk.rope_layer)
                blocks.append(blk)
            self.blocks = nn.ModuleList(blocks)
            self.norm = RMSNorm(d)
            self.out = nn.Linear(d, m.patch_dim)

        def forward(self, x_t, t, actions, target=None):
            B, Fr, C, H, W = x_t.shape
            p = m.patch
            tok = x_t.reshape(B, Fr, C, H // p, p, W // p, p).permute(0, 1, 3, 5, 2, 4, 6)
            tok = tok.reshape(B, Fr * (H // p) * (W // p), C * p * p)
            x = self.patch_embed(tok)
            c = self.t_embed(t)[:, None] + self.a_embed(actions)          # [B, F, d]
            c = c.repeat_interleave(x.shape[1] // Fr, dim=1)
            for blk in self.blocks:
                x, _ = blk(x, cond=c)
            y = self.out(self.norm(x))
            y = y.reshape(B, Fr, H // p, W // p, C, p, p).permute(0, 1, 4, 2, 5, 3, 6)
            return y.reshape(B, Fr, C, H, W)

    return RefWorldDiT().to(device)


def run(args, ws, rank, local):
    if not os.path.isdir(os.path.join(REF, "layers")):
        return _unavailable("reference not installed under baseline/_ref")
    sys.path.insert(0, ROOT)
    from drivedit_b200.config import get_config

    cfg = get_config(args.config, args.override)
    sys.path.insert(0, REF)
    import types

    import torch.distributed as dist
    from training.cuda_optimized import (CUDAOptimizedConfig, OptimizedTrainer,
                                         create_optimized_optimizer)

    dev = torch.device("cuda", local)
    torch.manual_seed(cfg.train.seed + rank)
    model = build(cfg, dev)
    ocfg = CUDAOptimizedConfig(compile_mode="default", amp_dtype=torch.bfloat16,
                               grad_scaler_enabled=False, use_fsdp=ws > 1,
                               gradient_checkpointing=False)
    if ws > 1:
        holder = types.SimpleNamespace(config=ocfg, device=dev)
        model = OptimizedTrainer._wrap_fsdp(holder, model)
    opt = create_optimized_optimizer(model, lr=cfg.train.lr, weight_decay=cfg.train.weight_decay,
                                     betas=tuple(cfg.train.betas))

    class _Step:
        def train_step(self, batch, optimizer, loss_fn):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = model(**batch)
                loss = loss_fn(out, batch)["total"]
            loss.backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), ocfg.gradient_clip_norm)
            optimizer.step()
            optimizer.zero_grad(set_to_none=True)
            return {"loss": loss.item()}

    trainer = _Step()
    m = cfg.model
    B, Fr = cfg.train.batch_per_gpu, cfg.train.frames
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    def make():
        x1 = torch.randn(B, Fr, m.latent_channels, m.latent_h, m.latent_w, device=dev, generator=g)
        x0 = torch.randn(x1.shape, device=dev, generator=g)
        t = torch.sigmoid(torch.randn(B, device=dev, generator=g))
        x_t = (1 - t[:, None, None, None, None]) * x0 + t[:, None, None, None, None] * x1
        a = torch.rand(B, Fr, m.action_dim, device=dev, generator=g) * 2 - 1
        return {"x_t": x_t, "t": t, "actions": a, "target": x1 - x0}

    def loss_fn(out, batch):
        return {"total": F.mse_loss(out.float(), batch["target"])}

    batch = make()
    try:
        for _ in range(args.warmup):
            trainer.train_step(batch, opt, loss_fn)
        torch.cuda.synchronize()
    except torch.OutOfMemoryError as exc:
        # the unmodified reference does not fit this config (eager SLA block loop, no
        # activation checkpointing): report it instead of a number
        return _unavailable(f"out of memory on one GPU in the reference's training step at "
                            f"{B} x {Fr * m.tokens_per_frame} tokens per GPU "
                            f"({str(exc).splitlines()[0][:160]})")
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    flush = torch.empty(64 << 20, device=dev)
    s.record()
    for _ in range(args.steps):
        flush.zero_()
        trainer.train_step(batch, opt, loss_fn)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    if dist.is_initialized():
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    tokens = B * Fr * m.tokens_per_frame
    value = ws * tokens / (ms / 1000.0)
    return {
        "impl": "reference",
        "metric": "train latent tok/s (max over ranks)",
        "value": round(value, 1), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic latents/actions/flow-time, random-init weights",
        "config": {"model": cfg.model.name, "global_batch": B * ws,
                   "seq_len": Fr * m.tokens_per_frame, "attention": m.attention,
                   "parallelism": f"fsdp{ws}" if ws > 1 else "single",
                   "stack": "reference DiTBlock + CausalSparseLinearAttention + _wrap_fsdp + fused AdamW",
                   "l2": "256 MiB buffer overwritten before every timed step"},
    }
