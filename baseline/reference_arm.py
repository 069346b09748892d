"""Reference arm of ``bench.py``: the unmodified reference (copied under ``baseline/_ref``)
run through its own modules and its own trainer code path.

Training (``--config dit_b`` / ``moe_dit_l``). The model is assembled from the reference's
public blocks at the preset's shape: ``blocks.dit_block.DiTBlock`` (dense SwiGLU) or
``layers.moe.MoEDiTBlock`` (64 routed + 2 shared experts, every expert local, the
reference's per-expert loop, layers/moe.py:372-424), each with AdaLN conditioning and
1-D RoPE, its attention swapped for the reference's drop-in
``layers.sla.CausalSparseLinearAttention`` (64-token blocks, layers/sla.py:440-456);
``blocks.flow_matching.TimestepEmbedding`` embeds the flow time and
``layers.nn_helpers.RMSNorm`` normalises the head. The step is the body of
``OptimizedTrainer.train_step`` (training/cuda_optimized.py:636-707) with the
reference's defaults: bf16 autocast, gradient checkpointing ON through the reference's
own ``MemoryOptimizer.memory_checkpoint_context`` (:466-488, default
``gradient_checkpointing=True`` at :78), clip 1.0, ``create_optimized_optimizer``
(fused AdamW), and for N > 1 the reference's FSDP wrapper ``OptimizedTrainer._wrap_fsdp``
(:571-615, FULL_SHARD, bf16 params / fp32 reduce). ``OptimizedTrainer.__init__`` itself
does not run on this PyTorch (``torch.cuda.amp.autocast(device_type=...)`` raises
TypeError, :19,518) and torch.compile is left off (autotuning the Python SLA loop does
not finish), so the step body is driven directly.

The reference's SLA is an eager Python loop over every (query block, key block) pair
with two host synchronisations per pair (layers/sla.py:201-241); a DiT-B step at
8 x 8192 tokens runs for minutes. Before any collective, every rank therefore runs one
block forward + backward at the full per-GPU shape on its own (a probe), predicts the
step's peak memory and duration from it, and the ranks agree on the worst prediction
with one ``all_reduce`` (nothing else in flight). If the step cannot fit in memory, or
two steps cannot finish inside the time budget (``DDB_REF_BUDGET_S``, default 480 s),
every rank returns the same ``unavailable`` line. Otherwise the arm runs as many of the
requested warm-up and timed steps as the budget allows (at least one of each) and
reports the counts it used.

Rollout (:func:`run_rollout`). The causal reference ``DiTBlock`` stack with its KV-cache
concatenation (layers/mha.py:359-369) and the reference's Euler sampler
``RectifiedFlowSampler.sample`` (blocks/flow_matching.py:228-281), driven chunk by
chunk: 4-frame chunks, 4 flow steps, a rolling 32-frame window (the cache is trimmed
after each chunk's cache-fill forward). The reference has no tensor parallelism, so each
rank runs its own rollouts (TP = 1).
"""
from __future__ import annotations

import math
import os
import sys
import time
import traceback

import torch
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
METRIC = "train latent tok/s (max over ranks)"


def _unavailable(why):
    return {"impl": "reference", "unavailable": why}


def _ref_path():
    if REF not in sys.path:
        sys.path.insert(0, REF)


class _RefWorldDiT(nn.Module):
    """Latent patchify -> reference blocks -> RMSNorm -> unpatchify. The glue is the
    patch/unpatch reshapes, the per-frame action MLP and the conditioning broadcast."""

    def __init__(self, m, tokens, block_factory):
        super().__init__()
        _ref_path()
        from blocks.flow_matching import TimestepEmbedding
        from layers.nn_helpers import RMSNorm

        d = m.d_model
        self.m = m
        self.patch_embed = nn.Linear(m.patch_dim, d)
        self.t_embed = TimestepEmbedding(d)
        self.a_embed = nn.Sequential(nn.Linear(m.action_dim, d), nn.SiLU(), nn.Linear(d, d))
        self.blocks = nn.ModuleList([block_factory() for _ in range(m.n_layers)])
        self.norm = RMSNorm(d)
        self.out = nn.Linear(d, m.patch_dim)

    def patchify(self, x):
        B, Fr, C, H, W = x.shape
        p = self.m.patch
        tok = x.reshape(B, Fr, C, H // p, p, W // p, p).permute(0, 1, 3, 5, 2, 4, 6)
        return tok.reshape(B, Fr * (H // p) * (W // p), C * p * p)

    def unpatchify(self, y, Fr):
        m, p = self.m, self.m.patch
        B = y.shape[0]
        y = y.reshape(B, Fr, m.latent_h // p, m.latent_w // p, m.latent_channels, p, p)
        return y.permute(0, 1, 4, 2, 5, 3, 6).reshape(B, Fr, m.latent_channels, m.latent_h,
                                                      m.latent_w)

    def embed(self, tok, t, actions):
        x = self.patch_embed(tok)
        Fr = actions.shape[1]
        c = self.t_embed(t)[:, None] + self.a_embed(actions)          # [B, F, d]
        return x, c.repeat_interleave(x.shape[1] // Fr, dim=1)

    def forward(self, x_t, t, actions, target=None):
        Fr = x_t.shape[1]
        x, c = self.embed(self.patchify(x_t), t, actions)
        for blk in self.blocks:
            x, _ = blk(x, cond=c)
        return self.unpatchify(self.out(self.norm(x)), Fr)


def build(cfg, device, max_seq_len=None):
    """The reference model for ``cfg.model`` on ``device`` (train shape by default)."""
    _ref_path()
    from blocks.dit_block import DiTBlock
    from layers.moe import MoEDiTBlock
    from layers.sla import CausalSparseLinearAttention, SLAConfig

    m = cfg.model
    T = max_seq_len or cfg.train.frames * m.tokens_per_frame

    def block():
        if m.moe is not None:
            blk = MoEDiTBlock(m.d_model, m.n_heads, num_experts=m.moe.num_experts,
                              top_k=m.moe.top_k, expert_dim=m.moe.expert_dim,
                              num_shared_experts=m.moe.num_shared, causal=True,
                              max_seq_len=T, cond_dim=m.d_model,
                              bias_update_speed=m.moe.bias_update_speed)
        else:
            blk = DiTBlock(m.d_model, m.n_heads, d_ff=m.mlp_hidden, mlp_type="swiglu",
                           causal=True, max_seq_len=T, cond_dim=m.d_model)
        if m.attention == "sla":
            blk.attn = CausalSparseLinearAttention(
                m.d_model, m.n_heads, SLAConfig(block_size=m.sla.block_size, causal=True),
                rope_layer=blk.rope_layer)
        return blk

    return _RefWorldDiT(m, T, block).to(device)


def _synthetic(cfg, dev, g):
    m = cfg.model
    B, Fr = cfg.train.batch_per_gpu, cfg.train.frames
    x1 = torch.randn(B, Fr, m.latent_channels, m.latent_h, m.latent_w, device=dev, generator=g)
    x0 = torch.randn(x1.shape, device=dev, generator=g)
    t = torch.sigmoid(torch.randn(B, device=dev, generator=g))
    tt = t[:, None, None, None, None]
    a = torch.rand(B, Fr, m.action_dim, device=dev, generator=g) * 2 - 1
    return {"x_t": (1 - tt) * x0 + tt * x1, "t": t, "actions": a, "target": x1 - x0}


def _probe(model, batch):
    """One block forward + backward at the full per-GPU shape, local (no collectives).

    Returns (fits_probe, block_fwd_s, block_bwd_s, block_peak_bytes, saved_bytes_per_layer,
    resident_bytes)."""
    dev = batch["x_t"].device
    torch.cuda.synchronize()
    resident = torch.cuda.memory_allocated(dev)
    try:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            x, c = model.embed(model.patchify(batch["x_t"]), batch["t"], batch["actions"])
        x = x.detach().requires_grad_(True)
        c = c.detach()
        saved = x.numel() * x.element_size()
        blk = model.blocks[0]
        # twice: the first pass pays one-time costs (library handles, allocator growth)
        for _ in range(2):
            x.grad = None
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats(dev)
            base = torch.cuda.memory_allocated(dev)
            t0 = time.perf_counter()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y, _ = blk(x, cond=c)
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            y.float().square().mean().backward()
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            peak = torch.cuda.max_memory_allocated(dev) - base
            del y
            for p in blk.parameters():
                p.grad = None
        del x, c
        torch.cuda.empty_cache()
        return True, t1 - t0, t2 - t1, peak, saved + c_bytes(batch, model), resident
    except torch.OutOfMemoryError:
        for p in model.parameters():
            p.grad = None
        torch.cuda.empty_cache()
        return False, 0.0, 0.0, 0, 0, resident


def c_bytes(batch, model):
    # the broadcast conditioning [B, T, d] is one tensor shared by every checkpointed
    # block; count it once, spread over the layers
    B, Fr = batch["actions"].shape[:2]
    T = model.patchify(batch["x_t"][:, :1]).shape[1] * Fr
    return B * T * model.m.d_model * 2 // max(1, len(model.blocks))


def _agree_max(values, dev):
    import torch.distributed as dist

    t = torch.tensor(values, device=dev, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run(args, ws, rank, local):
    """Reference training arm (dense DiT or MoE DiT, SLA attention)."""
    if not os.path.isdir(os.path.join(REF, "layers")):
        return _unavailable("reference not installed under baseline/_ref")
    sys.path.insert(0, ROOT)
    from drivedit_b200.config import get_config

    import torch.distributed as dist

    cfg = get_config(args.config, args.override)
    _ref_path()
    from training.cuda_optimized import (CUDAOptimizedConfig, MemoryOptimizer, OptimizedTrainer,
                                         create_optimized_optimizer)

    budget = float(os.environ.get("DDB_REF_BUDGET_S", "480"))
    dev = torch.device("cuda", local)
    torch.manual_seed(cfg.train.seed)
    model = build(cfg, dev)
    m = cfg.model
    B, Fr = cfg.train.batch_per_gpu, cfg.train.frames
    tokens = B * Fr * m.tokens_per_frame
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    batch = _synthetic(cfg, dev, g)

    # ---- probe + collective go/no-go (before the first FSDP collective)
    ok, fwd_s, bwd_s, blk_peak, saved, resident = _probe(model, batch)
    n_params = sum(p.numel() for p in model.parameters())
    # fp32 weights + grads + two AdamW moments (sharded 1/ws under FULL_SHARD) and
    # the bf16 gather of the largest FSDP unit
    state = 16 * n_params / ws + 2 * n_params / max(1, m.n_layers)
    pred_peak = state + m.n_layers * saved + blk_peak * 1.10
    # checkpointing runs each block's forward twice (forward, recompute) and its backward
    pred_step = m.n_layers * (2 * fwd_s + bwd_s) * 1.05
    total_mem = torch.cuda.mem_get_info(dev)[1]
    fail, pred_peak, pred_step = _agree_max([0.0 if ok else 1.0, pred_peak, pred_step], dev)
    detail = (f"{B} x {Fr * m.tokens_per_frame} tokens per GPU, {m.n_layers} layers, "
              f"world size {ws}")
    if fail > 0:
        return _unavailable(f"out of memory in one reference block's forward+backward at "
                            f"{detail} (gradient checkpointing on)")
    if pred_peak > 0.95 * total_mem:
        return _unavailable(f"predicted peak {pred_peak / 2**30:.1f} GiB over the "
                            f"{total_mem / 2**30:.1f} GiB device at {detail} "
                            f"(gradient checkpointing on)")
    n_fit = int(budget // max(pred_step, 1e-3))
    if n_fit < 2:
        return _unavailable(f"one reference step is predicted at {pred_step:.0f} s at {detail} "
                            f"(SLA Python block loop, checkpointing on); a warm-up and a timed "
                            f"step do not fit the {budget:.0f} s budget")
    warm = max(1, min(args.warmup, n_fit // 2))
    steps = max(1, min(args.steps, n_fit - warm))

    ocfg = CUDAOptimizedConfig(compile_mode="default", amp_dtype=torch.bfloat16,
                               grad_scaler_enabled=False, use_fsdp=ws > 1)
    assert ocfg.gradient_checkpointing  # the reference default, applied below
    if ws > 1:
        import types

        holder = types.SimpleNamespace(config=ocfg, device=dev)
        model = OptimizedTrainer._wrap_fsdp(holder, model)
    memopt = MemoryOptimizer(ocfg)
    opt = create_optimized_optimizer(model, lr=cfg.train.lr, weight_decay=cfg.train.weight_decay,
                                     betas=tuple(cfg.train.betas))

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            with memopt.memory_checkpoint_context(model):
                out = model(**batch)
                loss = F.mse_loss(out.float(), batch["target"])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), ocfg.gradient_clip_norm)
        opt.step()
        opt.zero_grad(set_to_none=True)
        memopt.maybe_empty_cache()
        return loss

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    flush = torch.empty(64 << 20, device=dev)
    s.record()
    for _ in range(steps):
        flush.zero_()
        loss = step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    ms = _agree_max([ms], dev)[0]
    loss_v = float(loss.item())
    if dist.is_initialized():
        dist.barrier()
    value = ws * tokens / (ms / 1000.0)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 1), "unit": "tok/s", "n_gpus": ws, "steps": steps,
        "warmup": warm, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic latents/actions/flow-time, random-init weights",
        "requested": {"steps": args.steps, "warmup": args.warmup},
        "budget": {"seconds": budget, "predicted_step_s": round(pred_step, 1),
                   "predicted_peak_gib": round(pred_peak / 2**30, 1),
                   "note": "steps/warm-up reduced to what the time budget allows"
                   if (steps, warm) != (args.steps, args.warmup) else "as requested"},
        "final_loss": loss_v,
        "config": {"model": cfg.model.name, "global_batch": B * ws,
                   "seq_len": Fr * m.tokens_per_frame, "attention": m.attention,
                   "parallelism": f"fsdp{ws}" if ws > 1 else "single",
                   "stack": ("reference " + ("MoEDiTBlock" if m.moe is not None else "DiTBlock")
                             + " + CausalSparseLinearAttention + MemoryOptimizer gradient "
                             "checkpointing + _wrap_fsdp + fused AdamW"),
                   "l2": "256 MiB buffer overwritten before every timed step"},
    }


# --------------------------------------------------------------------------- rollout
class _Timer:
    """CUDA events on a GPU, wall clock on the CPU."""

    def __init__(self, dev):
        self.cuda = dev.type == "cuda"
        self.marks = []

    def start(self):
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            return ev
        return time.perf_counter()

    def stop(self, s):
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append((s, ev))
        else:
            self.marks.append((s, time.perf_counter()))

    def ms(self):
        if self.cuda:
            torch.cuda.synchronize()
            return [a.elapsed_time(b) for a, b in self.marks]
        return [(b - a) * 1000.0 for a, b in self.marks]


def run_rollout(batch, frames=None, overrides=None, config="rollout_dit_b", warm_chunks=2,
                device=None):
    """Reference streaming rollout on ``device`` (default: the current GPU): frames/s and
    per-chunk latency (p50 / p99)."""
    if not os.path.isdir(os.path.join(REF, "layers")):
        return _unavailable("reference not installed under baseline/_ref")
    sys.path.insert(0, ROOT)
    from contextlib import nullcontext

    from drivedit_b200.config import get_config

    cfg = get_config(config, overrides)
    r = cfg.rollout
    frames = frames or r.total_frames
    _ref_path()
    from blocks.flow_matching import FlowMatchingConfig, RectifiedFlowSampler

    dev = device or torch.device("cuda", torch.cuda.current_device())
    m = cfg.model
    tpf = m.tokens_per_frame
    torch.manual_seed(0)
    model = build(cfg, dev, max_seq_len=(frames + 8) * tpf).eval()
    amp = (lambda: torch.autocast("cuda", dtype=torch.bfloat16)) if dev.type == "cuda" \
        else nullcontext
    g = torch.Generator(device=dev).manual_seed(1)
    window = r.window_frames * tpf

    def forward_tokens(tok, t, actions, caches, start, keep):
        with amp():
            x, c = model.embed(tok, t, actions)
            new = []
            for blk, cache in zip(model.blocks, caches):
                x, nc = blk(x, kv_cache=cache, cond=c, start_pos=start)
                new.append(nc)
            y = model.out(model.norm(x)).float()
        if keep:
            return y, [{"k": nc["k"][:, -window:], "v": nc["v"][:, -window:]} for nc in new]
        return y, None

    class Predictor:
        """Adapter with the call signature the reference sampler uses."""

        def __init__(self):
            self.caches, self.start, self.actions = None, 0, None

        def __call__(self, z_t, t_batch, mask=None, context=None):
            return forward_tokens(z_t, t_batch, self.actions, self.caches, self.start, False)[0]

    pred = Predictor()
    sampler = RectifiedFlowSampler(pred, FlowMatchingConfig())

    def rollout(n_frames, B):
        ctx = torch.randn(B, r.context_frames, m.latent_channels, m.latent_h, m.latent_w,
                          device=dev, generator=g)
        act = torch.rand(B, n_frames, m.action_dim, device=dev, generator=g) * 2 - 1
        kv_dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        empty = [{"k": torch.zeros(B, 0, m.n_heads, m.d_head, device=dev, dtype=kv_dtype),
                  "v": torch.zeros(B, 0, m.n_heads, m.d_head, device=dev, dtype=kv_dtype)}
                 for _ in model.blocks]
        ones = torch.ones(B, device=dev)
        with torch.no_grad():
            _, caches = forward_tokens(model.patchify(ctx), ones, act[:, :r.context_frames],
                                       empty, 0, True)
        pos = r.context_frames
        timer = _Timer(dev)
        while pos < n_frames:
            nf = min(r.chunk_frames, n_frames - pos)
            s = timer.start()
            z = torch.randn(B, nf * tpf, m.patch_dim, device=dev, generator=g)
            pred.caches, pred.start, pred.actions = caches, pos * tpf, act[:, pos:pos + nf]
            out = sampler.sample(z, r.flow_steps)["final_sample"]
            with torch.no_grad():
                _, caches = forward_tokens(out, ones, act[:, pos:pos + nf], caches, pos * tpf,
                                           True)
            timer.stop(s)
            pos += nf
        return timer.ms()

    try:
        rollout(r.context_frames + warm_chunks * r.chunk_frames, batch)
        chunk_ms = rollout(frames, batch)
    except torch.OutOfMemoryError as exc:
        return _unavailable(f"out of memory in the reference rollout at batch {batch} "
                            f"({str(exc).splitlines()[0][:120]})")
    except Exception as exc:  # noqa: BLE001 - a failing reference path is reported, not fatal
        return _unavailable(f"the reference rollout raised {type(exc).__name__}: "
                            f"{str(exc).splitlines()[0][:160] if str(exc) else ''}")
    return _rollout_summary(chunk_ms, batch, frames - r.context_frames, cfg, impl="reference")


def _rollout_summary(chunk_ms, batch, gen_frames, cfg, impl):
    s = sorted(chunk_ms)

    def pct(q):
        if not s:
            return None
        k = (len(s) - 1) * q / 100.0
        lo, hi = math.floor(k), math.ceil(k)
        return s[lo] + (s[hi] - s[lo]) * (k - lo)

    total_s = sum(chunk_ms) / 1000.0
    return {"impl": impl, "batch": batch, "frames_per_s": round(batch * gen_frames / total_s, 2),
            "p50_chunk_ms": round(pct(50), 3), "p99_chunk_ms": round(pct(99), 3),
            "chunks": len(chunk_ms), "generated_frames": gen_frames,
            "chunk_frames": cfg.rollout.chunk_frames, "flow_steps": cfg.rollout.flow_steps,
            "window_frames": cfg.rollout.window_frames}


def describe_exception(rank):
    """One-line-per-rank error record printed to stderr before a rank exits."""
    return f"[rank {rank}] reference arm failed:\n{traceback.format_exc()}"
