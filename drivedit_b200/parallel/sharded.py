"""Sharded data parallelism for the world models (FSDP's communication pattern).

Every rank holds the full bf16 compute weights (what the forward/backward kernels read),
the full fp32 master copy (what the PyTorch-side conditioning modules read) and a full
fp32 gradient buffer the backward accumulates into; the AdamW moments and the update
itself are sharded ``1/world``. One optimizer step is

    reduce-scatter(grad) -> clip by the global norm -> AdamW(shard) -> all-gather(weights)

which is FSDP's SHARD_GRAD_OP schedule (reference ``training/cuda_optimized.py:571-615``)
with weights kept gathered between steps, because HBM is not the constraint at these
model sizes (DiT-B: 0.5 GB of fp32 master per rank).

``weight_gather=True`` (fused transport) switches the block GEMM weights (attention
QKV / output / linear-branch projections, SwiGLU W13 / W3) to FULL_SHARD's schedule: the
optimizer stores their updated shard only into its own rank's buffers, and each
forward GEMM that consumes one of these weights first all-gathers the peer-owned pieces
into the local buffer from inside the GEMM kernel (``GemmArgs.gb_*`` in
``csrc/gemm/gemm.cu``): the parameter all-gather fused with the first GEMM that reads
it, tile by tile, with no separate collective launch. The backward GEMMs read the
gathered copy. These weights form a contiguous prefix of the flat buffer, so the
optimizer needs one boundary (``local_end``). :meth:`ShardedDataParallel.gather_weights`
materialises the full weights (fp32 and bf16) for checkpointing or inference.

Two transports:

``fused`` (default on CUDA)
    The flat buffers live in CUDA-IPC memory mapped by every rank. The reduce-scatter is
    the optimizer's own read of its shard from every peer's gradient buffer, and the
    all-gather is the optimizer's store of the updated fp32/bf16 shard into every peer's
    buffers (``csrc/comm/comm.cu``); bounded cross-rank flag barriers order the phases
    and carry the squared-norm partials for clipping.
``nccl``
    ``reduce_scatter_tensor`` + local AdamW on the shard + ``all_gather_into_tensor``
    (the baseline; on CPU the same calls run over gloo, which the multi-process tests use).
"""
from __future__ import annotations

import math
import re
from typing import Dict, Optional, Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

from .flat import ALIGN, FlatParamGroup


class SymmetricBuffer:
    """An equally sized CUDA-IPC buffer on every rank with a device table of peer pointers."""

    def __init__(self, nbytes: int, group, device: torch.device):
        from ..ops._ext import ext

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = nbytes
        ptr, handle = ext().ipc_alloc(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptr = ptr
        self.peers = [ptr if r == self.rank else ext().ipc_open(handles[r])
                      for r in range(self.world)]
        self.table = torch.tensor(self.peers, dtype=torch.int64, device=device)
        self.device = device

    def tensor(self, numel: int, dtype: torch.dtype, byte_offset: int = 0) -> torch.Tensor:
        from ..ops._ext import ext

        return ext().tensor_from_ptr(self.ptr + byte_offset, numel, dtype, self.device.index)

    def peer_table(self, byte_offset: int = 0) -> torch.Tensor:
        return self.table + byte_offset

    def close(self):
        from ..ops._ext import ext

        torch.cuda.synchronize(self.device)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                ext().ipc_close(p)
        ext().ipc_free(self.ptr)
        self.peers = []


GATHERED_WEIGHT = re.compile(r"^blocks\.\d+\.(attn\.(qkv|proj|proj_lin)|mlp\.(w13|w3))\.weight$")


class WeightGather:
    """Launch state of one weight's fused all-gather: its flat offset, its address in
    every rank's bf16 buffer, the per-128-row readiness counters and the launch epoch."""

    def __init__(self, engine: "ShardedDataParallel", name: str, param: nn.Parameter):
        off, numel = engine.flat.offsets[name]
        self.name = name
        self.elem0 = off
        self.numel = numel
        self.rank, self.shard = engine.rank, engine.shard_len
        self.peers = [int(p) + 2 * off for p in engine.sym["compute"].peers]
        rows = param.shape[0]
        self.counters = torch.zeros((rows + 127) // 128, dtype=torch.int32, device=engine.device)
        self.epoch = 0

    def launch_args(self, b: torch.Tensor):
        if b.data_ptr() != self.peers[self.rank] or b.numel() != self.numel:
            raise RuntimeError(f"fused weight gather: {self.name} is not the registered view")
        self.epoch += 1
        return self.counters, self.peers, self.rank, self.elem0, self.shard, self.epoch


class ShardedDataParallel:
    """Owns the flat buffers of a model and performs the sharded optimizer step."""

    def __init__(self, model: nn.Module, group=None, device=None, transport: Optional[str] = None,
                 lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.01, grad_clip=1.0,
                 local_params: Optional[Sequence[str]] = None, weight_gather: bool = False,
                 overlap: bool = False):
        """``local_params``: names of rank-local parameters (expert-parallel experts).
        They are neither reduced nor sharded: a local flat group with a full AdamW holds
        them, their squared gradient norm joins the global clipping norm, and the main
        group resolves their compute views (``FlatParamGroup.linked``)."""
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.transport = transport or ("fused" if self.device.type == "cuda" else "nccl")
        self.lr, self.betas, self.eps, self.wd, self.grad_clip = lr, tuple(betas), eps, weight_decay, grad_clip
        named_all = list(model.named_parameters())
        local = set(local_params or [])
        named = [(n, p) for n, p in named_all if n not in local]
        if hasattr(model, "flat_layout"):
            named = model.flat_layout(named)
        self.weight_gather = bool(weight_gather) and self.transport == "fused" and self.world > 1
        if self.weight_gather:  # gathered weights first: a contiguous prefix of the flat buffer
            named = ([(n, p) for n, p in named if GATHERED_WEIGHT.match(n)]
                     + [(n, p) for n, p in named if not GATHERED_WEIGHT.match(n)])
        no_decay = model.no_decay_names() if hasattr(model, "no_decay_names") else []
        pad = ALIGN * self.world * 4
        self.sym = {}
        alloc = None
        if self.transport == "fused":
            numel = _padded_numel(named, no_decay, pad)
            bufs = {}
            for name, dt, es in (("master", torch.float32, 4), ("grad", torch.float32, 4),
                                 ("compute", torch.bfloat16, 2)):
                bufs[name] = SymmetricBuffer(numel * es, self.group, self.device)
            self.sym = bufs
            self.flags = SymmetricBuffer(8 * self.world + 64, self.group, self.device)

            def alloc(name, n, dtype):
                return bufs[name].tensor(n, dtype)
        self.flat = FlatParamGroup(named, self.device, no_decay=no_decay, pad_to=self.world * 4,
                                   allocator=alloc)
        self.local_end = 0
        self.gathers: Dict[int, WeightGather] = {}
        self.local_opt = None
        if local:
            from ..training.optim import FlatAdamW

            lg = FlatParamGroup([(n, p) for n, p in named_all if n in local], self.device,
                                no_decay=no_decay)
            self.local_opt = FlatAdamW(lg, lr, betas, eps, weight_decay, grad_clip)
            self.flat.linked.append(lg)
        n = self.flat.numel
        assert n % (self.world * 4) == 0
        self.shard_len = n // self.world
        self.shard_off = self.rank * self.shard_len
        if self.weight_gather:
            for n, p in named:
                if GATHERED_WEIGHT.match(n):
                    o, k = self.flat.offsets[n]
                    self.local_end = max(self.local_end, o + k)
                    self.gathers[id(p)] = WeightGather(self, n, p)
            self.local_end = (self.local_end + 3) // 4 * 4
            self.flat.gather_for = lambda p: self.gathers.get(id(p))
        # Reduce-scatter overlapped with the backward (fused transport): the flat buffer is
        # cut into buckets (each block's contiguous GEMM weights, plus the remaining
        # ranges) and every rank owns 1/W of every bucket, so each bucket's reduce can run
        # on a side stream as soon as the backward has finished that block on all ranks.
        self.pieces = None
        self._armed = False
        self._done = set()
        self._side = None
        if overlap and self.transport == "fused" and self.world > 1 and not self.weight_gather:
            self.pieces = self._plan_pieces()
            if self.pieces is not None:
                self.shard_len = sum(hi - lo for lo, hi, _, _ in self.pieces)
                self.shard_off = -1  # the shard is the pieces' union, not one range
        self.m = torch.zeros(max(self.shard_len, 4), device=self.device)
        self.v = torch.zeros(max(self.shard_len, 4), device=self.device)
        self.red = torch.zeros(max(self.shard_len, 4), device=self.device)
        self.sumsq = torch.zeros(1, device=self.device)
        self.step_count = 0
        self.epoch = 0
        self.last_grad_norm: Optional[torch.Tensor] = None
        # identical starting weights everywhere
        dist.broadcast(self.flat.master, src=0, group=self.group)
        self.flat.refresh_compute()
        if self.transport == "fused":
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)

    # ------------------------------------------------------------------ overlap
    def _plan_pieces(self):
        """This rank's pieces ``(global lo, global hi, local offset, bucket)``: bucket ``i``
        is the contiguous flat run of block ``i``'s weights (its AdaLN projection, which
        the batched modulation backward writes last, excluded), bucket ``None`` every
        remaining range. Each bucket is cut into ``W`` pieces of a multiple of 4 elements
        (16 bytes); rank ``r`` owns piece ``r`` of every bucket. ``None`` when no block has
        a contiguous run."""
        W, r = self.world, self.rank
        spans: Dict[int, list] = {}
        for name in self.flat.names:
            mm = re.match(r"^blocks\.(\d+)\.", name)
            if mm is None or ".ada." in name or name.endswith("norm1.weight") or name.endswith("norm2.weight"):
                continue
            o, k = self.flat.offsets[name]
            spans.setdefault(int(mm.group(1)), []).append((o, o + k))
        starts = sorted(o for o, _ in self.flat.offsets.values())
        runs = {}
        for i, v in spans.items():
            lo, hi = min(a for a, _ in v), max(b for _, b in v)
            mine = {a for a, _ in v}
            if any(lo <= a < hi and a not in mine for a in starts):  # not contiguous
                continue
            lo, hi = lo // 4 * 4, (hi + 3) // 4 * 4
            runs[i] = (lo, hi)
        if not runs:
            return None
        self.bucket_ids = set(runs)  # identical on every rank (the layout is)
        # the remaining ranges of [0, numel)
        rest, cur = [], 0
        for lo, hi in sorted(runs.values()):
            if lo > cur:
                rest.append((cur, lo))
            cur = max(cur, hi)
        if cur < self.flat.numel:
            rest.append((cur, self.flat.numel))
        buckets = [(i, lo, hi) for i, (lo, hi) in sorted(runs.items())] + [(None, lo, hi) for lo, hi in rest]
        pieces, off = [], 0
        for b, lo, hi in buckets:
            q = ((hi - lo + W - 1) // W + 3) // 4 * 4
            plo, phi = min(hi, lo + r * q), min(hi, lo + (r + 1) * q)
            if phi > plo:
                pieces.append((plo, phi, off, b))
                off += phi - plo
        return pieces

    def arm_overlap(self):
        """Before one backward whose gradients the next ``step`` consumes: each block's
        bucket is reduced as soon as that block's backward is done (``bucket_ready``)."""
        self._armed = self.pieces is not None
        self._done = set()

    def bucket_ready(self, block: int):
        """Called (by the fused engine) right after block ``block``'s backward has been
        enqueued: after every rank got there (bounded barrier on a side stream), reduce
        this rank's piece of the block's bucket by peer loads into the local shard."""
        if not self._armed or block in self._done:
            return
        from ..ops._ext import ext

        if block not in self.bucket_ids:
            return
        mine = [p for p in self.pieces if p[3] == block]  # may be empty: still in the barrier
        main = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(self.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            if not self._done:
                self.sumsq.zero_()
            self._barrier()                               # block `block` is final on every rank
            for lo, hi, off, _ in mine:
                ext().rs_sum_sqnorm(self.sym["grad"].table, self.world, lo, hi - lo, self.red[off:], self.sumsq)
        self._done.add(block)

    # ------------------------------------------------------------------ step
    def zero_grad(self):
        self.flat.zero_grad()

    def step(self):
        self.step_count += 1
        b1, b2 = self.betas
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        scale = 1.0 / self.world  # gradients are summed over ranks; the loss is a mean
        if self.transport == "fused":
            self._step_fused(bc1, bc2, scale)
        else:
            self._step_collective(bc1, bc2, scale)

    def _barrier(self, payload=None):
        from ..ops._ext import ext

        self.epoch += 1
        ext().xrank_barrier(self.flags.table, self.flags.ptr, self.rank, self.world, self.epoch,
                            payload)

    def _step_fused(self, bc1, bc2, scale):
        from ..ops._ext import ext

        pieces = self.pieces
        if pieces is None:  # one contiguous shard
            pieces = [(self.shard_off, self.shard_off + self.shard_len, 0, None)]
        armed = self._armed and self.pieces is not None
        if armed and self._side is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._side)
        # buckets reduced during the backward are done; the rest now
        done = self._done if armed else set()
        if armed:  # every planned bucket took its barrier, in the same order on all ranks
            for b in sorted(self.bucket_ids - done):
                self.bucket_ready(b)
            torch.cuda.current_stream(self.device).wait_stream(self._side)
            done = self._done
        if not done:
            self.sumsq.zero_()
        self._barrier()                                   # every rank's gradients are final
        for lo, hi, off, b in pieces:
            if b is None or b not in done:
                ext().rs_sum_sqnorm(self.sym["grad"].table, self.world, lo, hi - lo, self.red[off:],
                                    self.sumsq)
        if self.local_opt is not None and self.grad_clip > 0:
            self.sumsq += self.local_opt.grad_sq_norm()
        self._barrier(self.sumsq)                         # squared-norm partials exchanged
        pay = self.flags.tensor(self.world, torch.float32, 4 * self.world)
        for lo, hi, off, _ in pieces:
            ext().shard_adamw_allgather(
                self.red[off:], self.flat.master, self.m[off:], self.v[off:], self.sym["master"].table,
                self.sym["compute"].table, self.world, lo, hi - lo,
                self.flat.decay_end, pay if self.grad_clip > 0 else None, float(self.grad_clip),
                self.lr, self.betas[0], self.betas[1], self.eps, self.wd, bc1, bc2, scale,
                self.rank, self.local_end)
        if self.local_opt is not None:
            self._local_step(scale, pay.sum() if self.grad_clip > 0 else None)
        self._barrier()                                   # all peers' stores have landed
        self._armed = False
        self._done = set()

    def _step_collective(self, bc1, bc2, scale):
        g = self.flat.grad
        dist.reduce_scatter_tensor(self.red, g, group=self.group)
        clip = 1.0
        sq = None
        if self.grad_clip > 0:
            sq = self.red.double().pow(2).sum().float().reshape(1)
            if self.local_opt is not None:
                sq = sq + self.local_opt.grad_sq_norm().reshape(1)
            dist.all_reduce(sq, group=self.group)
            norm = sq.sqrt() * scale
            self.last_grad_norm = norm
            clip = torch.clamp(self.grad_clip / (norm + 1e-6), max=1.0)
        lo, hi = self.shard_off, self.shard_off + self.shard_len
        master = self.flat.master[lo:hi]
        gr = self.red * (scale * clip)
        b1, b2 = self.betas
        self.m.mul_(b1).add_(gr, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
        upd = (self.m / bc1) / ((self.v / bc2).sqrt() + self.eps)
        if self.wd:
            d_end = min(max(self.flat.decay_end - lo, 0), self.shard_len)
            master[:d_end].mul_(1 - self.lr * self.wd)
        master.add_(upd, alpha=-self.lr)
        shard = master.clone()
        dist.all_gather_into_tensor(self.flat.master, shard, group=self.group)
        self.flat.refresh_compute()
        if self.local_opt is not None:
            self._local_step(scale, sq.reshape(()) if sq is not None else None)

    def _local_step(self, scale, sq_norm):
        """AdamW on the rank-local parameters with the same step count, gradient scale
        and global clipping norm as the sharded update."""
        self.local_opt.step_count = self.step_count - 1
        self.local_opt.step(grad_scale=scale, sq_norm=sq_norm)

    def gather_weights(self):
        """Weight-sharded mode: copy every rank's shard of the GEMM-gathered weights
        (fp32 master and bf16) into all buffers, so the full weights are resident (before
        ``state_dict`` / checkpointing / inference). Collective: every rank calls it."""
        if not self.weight_gather or self.local_end == 0:
            return
        from ..ops._ext import ext

        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        S = self.shard_len
        for r in range(self.world):
            lo, hi = r * S, min((r + 1) * S, self.local_end)
            if r == self.rank or hi <= lo:
                continue
            for kind, es in (("master", 4), ("compute", 2)):
                src = ext().tensor_from_ptr(self.sym[kind].peers[r] + lo * es, hi - lo,
                                            torch.float32 if es == 4 else torch.bfloat16,
                                            self.device.index)
                (self.flat.master if es == 4 else self.flat.compute)[lo:hi].copy_(src)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def close(self):
        for b in self.sym.values():
            b.close()
        if self.sym:
            self.flags.close()
        self.sym = {}


def _padded_numel(named, no_decay, pad) -> int:
    from .flat import _round

    off = 0
    for _, p in named:
        off = _round(off + p.numel(), ALIGN)
    return _round(off, pad)
