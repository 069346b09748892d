"""Expert parallelism for the MoE FFN: routed experts partitioned over the ranks of an
EP group, tokens moved to the rank that owns their expert and back.

Layout. With ``E`` routed experts and ``W`` ranks, rank ``r`` owns experts
``[r*E/W, (r+1)*E/W)`` (``MoEFFN.w13 / w2``); the shared experts stay replicated
(``w13_shared / w2_shared``) and run on every rank's own tokens. Every rank routes its own
tokens, then the per-expert counts of all ranks form a ``[W, E]`` table that every rank
holds (one small exchange per layer); from it each rank derives, for every (source rank,
expert) block of rows, where it sits in the source's *compact* buffer (its routed rows
sorted by expert, unpadded) and in the owner's grouped-GEMM layout (local experts in
128-row padded segments, sources in rank order inside a segment), so no other metadata
moves.

Transports:

``fused`` (CUDA)
    Rows move through NVLink peer memory from inside our kernels (``csrc/moe/ep.cu``): each
    source *pushes* every token row once to every rank owning one of its experts (P2P
    stores into the owner's symmetric staging rows, with the token's routing for that
    owner), the owner fans the staged rows out into its grouped-GEMM layout with local
    copies, and *pushes* per-token partial sums of its expert outputs into each source's
    symmetric return buffer (P2P stores); backward pushes ``dout`` to the same staging rows
    and ``dx`` partial sums back. Bounded cross-rank flag barriers order the phases; the
    count table itself travels by P2P stores. No NCCL call carries token payload.
``nccl``
    ``all_to_all_single`` of the compact rows plus a local ``ep_copy_rows`` into the
    grouped-GEMM layout (the baseline); on CPU the PyTorch path below runs over gloo.

Reference: the reference has no expert parallelism (``layers/moe.py:372-396`` loops over
all experts locally; ``layers/kernels/moe_kernels.py`` is single-device).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist


def _pad128(x):
    return (np.asarray(x, dtype=np.int64) + 127) // 128 * 128


class ExpertParallel:
    """EP group context: partition of the experts, symmetric buffers, barriers."""

    def __init__(self, group=None, num_experts: int = 8, transport: Optional[str] = None, device=None):
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        assert num_experts % self.world == 0, "experts must divide evenly over the EP ranks"
        self.num_experts = num_experts
        self.local_experts = num_experts // self.world
        dev = torch.device(device) if device is not None else torch.device("cpu")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.transport = transport or ("fused" if self.device.type == "cuda" else "nccl")
        self.n_layers = 0
        self._sym = {}
        self._flags = None
        self.epoch = 0
        self._shared_plans = {}
        self._slot_tables = {}

    def register(self, moe) -> int:
        """A new EP layer; returns its slot (index of its return buffer)."""
        self.n_layers += 1
        return self.n_layers - 1

    def local_range(self) -> Tuple[int, int]:
        return self.rank * self.local_experts, (self.rank + 1) * self.local_experts

    # ------------------------------------------------------------------ symmetric memory
    def sym(self, name: str, nbytes: int):
        """Symmetric buffer ``name`` with at least ``nbytes``; every rank calls this with
        the same size at the same point (growth re-allocates on all ranks together)."""
        from .sharded import SymmetricBuffer

        b = self._sym.get(name)
        if b is None or b.nbytes < nbytes:
            if b is not None:
                b.close()
            b = SymmetricBuffer(int(nbytes), self.group, self.device)
            self._sym[name] = b
        return b

    def slot_table(self, name: str, slot: int, slot_bytes: int) -> torch.Tensor:
        """Peer-pointer table of slot ``slot`` (``slot_bytes`` each) of buffer ``name``."""
        b = self._sym[name]
        key = (name, slot, slot_bytes, b.ptr)
        t = self._slot_tables.get(key)
        if t is None:
            t = b.table + slot * slot_bytes
            self._slot_tables[key] = t
        return t

    def barrier(self):
        from ..ops._ext import ext
        from .sharded import SymmetricBuffer

        if self._flags is None:
            self._flags = SymmetricBuffer(8 * self.world + 64, self.group, self.device)
        self.epoch += 1
        ext().xrank_barrier(self._flags.table, self._flags.ptr, self.rank, self.world, self.epoch, None)

    def close(self):
        for b in self._sym.values():
            b.close()
        if self._flags is not None:
            self._flags.close()
        self._sym, self._flags = {}, None
        self._slot_tables = {}

    # ------------------------------------------------------------------ count table
    def exchange_counts(self, counts: torch.Tensor) -> np.ndarray:
        """``counts [n]`` of this rank (per-expert counts, optionally followed by more
        per-rank integers) -> the ``[W, n]`` table of all ranks, on the host."""
        E = counts.numel()
        if self.transport == "fused":
            from ..ops._ext import ext

            rb = (E * 4 + 15) // 16 * 16
            tab = self.sym("table", self.world * rb)
            src = counts.to(torch.int32)
            if rb != E * 4:
                src = torch.nn.functional.pad(src, (0, rb // 4 - E))
            src = src.contiguous()
            blocks = self._table_blocks()
            ext().ep_copy_rows(None, src.data_ptr(), tab.table, 0, blocks[0], blocks[1], self.world,
                               rb, rb, rb)
            self.barrier()
            out = tab.tensor(self.world * rb // 4, torch.int32).view(self.world, rb // 4)[:, :E]
            return out.cpu().numpy().astype(np.int64)
        c = counts.to(torch.int64).reshape(1, -1)
        if dist.get_backend(self.group) == "nccl" and not c.is_cuda:
            c = c.to(self.device)
        out = torch.empty(self.world, E, dtype=torch.int64, device=c.device)
        dist.all_gather_into_tensor(out, c.contiguous(), group=self.group)
        return out.cpu().numpy()

    def _table_blocks(self):
        if getattr(self, "_tblocks", None) is None:
            b = torch.tensor([[0, 0, p, self.rank] for p in range(self.world)], dtype=torch.int32)
            self._tblocks = (b.to(self.device), torch.arange(self.world, dtype=torch.int32,
                                                             device=self.device))
        return self._tblocks

    def shared_plan(self, N: int, ns: int):
        """Grouped-GEMM tables for the ``ns`` shared experts over ``N`` local tokens."""
        key = (N, ns)
        if key not in self._shared_plans:
            from ..ops._ext import ext

            mt = ns * ((N + 127) // 128)
            dummy = torch.zeros(1, dtype=torch.int32, device=self.device)
            p = ext().moe_plan(dummy, 0, ns, N, mt)
            self._shared_plans[key] = (p, mt)
        return self._shared_plans[key]


# ----------------------------------------------------------------------------- plan
class EpPlan:
    """Movement plan of one layer, derived from the ``[W, E]`` count table.

    ``compact_start[s, e]``: first row of expert ``e`` in source ``s``'s compact buffer.
    ``block_start[s, e]``: first row of source ``s``'s block of expert ``e`` in the owner's
    grouped-GEMM layout (segments of the owner's local experts, padded to 128 rows).
    ``recv_start[s, e]``: the same block in the owner's source-major receive buffer of the
    ``nccl`` transport (rows of source 0, then source 1, ...).
    """

    def __init__(self, ep: ExpertParallel, table: np.ndarray):
        W, El, E = ep.world, ep.local_experts, ep.num_experts
        r = ep.rank
        table = np.asarray(table, dtype=np.int64)
        self.table = table
        lo, hi = ep.local_range()
        self.lo, self.hi = lo, hi
        tot = table.sum(0)                                                   # [E] rows per expert
        padded = _pad128(tot).reshape(W, El)
        seg = (np.cumsum(padded, 1) - padded).reshape(E)                     # segment start per expert
        self.block_start = seg[None, :] + (np.cumsum(table, 0) - table)      # [W, E]
        self.compact_start = np.cumsum(table, 1) - table                     # [W, E]
        mine = table[:, lo:hi]                                               # [W, El] rows to me
        flat = mine.reshape(-1)
        self.recv_start = (np.cumsum(flat) - flat).reshape(W, El)
        self.local_counts = tot[lo:hi]                                       # [El]
        self.owner_rows = int(padded[r].sum())
        self.owner_mtiles = self.owner_rows // 128
        self.n_routed = int(table[r].sum())                                  # my compact rows
        self.send_splits = table[r].reshape(W, El).sum(1).tolist()           # rows to each owner
        self.recv_splits = mine.sum(1).tolist()                              # rows from each source
        self.n_recv = int(mine.sum())

    def packet(self, ep: ExpertParallel, N: int, ns: int, k: int):
        """One int32 host array with everything the device needs for this layer:
        pull / push block lists (+ prefix sums), the owner's local counts, and the
        source-side dispatch segments (compact starts, counts, cursor), in that order."""
        W, El, E = ep.world, ep.local_experts, ep.num_experts
        lo, hi = self.lo, self.hi
        n = self.table[:, lo:hi].reshape(-1)
        s_idx = np.repeat(np.arange(W), El)
        cs = self.compact_start[:, lo:hi].reshape(-1)
        bs = self.block_start[:, lo:hi].reshape(-1)
        rs = self.recv_start.reshape(-1)
        keep = n > 0
        prefix = np.cumsum(n[keep]) - n[keep]
        zero = np.zeros_like(s_idx)
        if ep.transport == "fused":
            pull = np.stack([s_idx, cs, zero, bs], 1)[keep]         # peer compact -> my layout
            push = np.stack([zero, bs, s_idx, cs], 1)[keep]         # my layout -> peer compact
        else:
            pull = np.stack([zero, rs, zero, bs], 1)[keep]          # recv buffer -> my layout
            push = np.stack([zero, bs, zero, rs], 1)[keep]          # my layout -> send-back buffer
        nb = int(keep.sum())
        mine = self.table[ep.rank]
        pad_n = (N + 127) // 128 * 128
        seg_start = np.concatenate([self.compact_start[ep.rank], np.arange(ns) * pad_n])
        seg_count = np.concatenate([mine, np.full(ns, N)])
        parts = [pull.reshape(-1), prefix, push.reshape(-1), prefix, self.local_counts,
                 seg_start, seg_count, np.zeros(E + ns)]
        arr = np.concatenate([np.asarray(p, dtype=np.int64) for p in parts]).astype(np.int32)
        sizes = [4 * nb, nb, 4 * nb, nb, El, E + ns, E + ns, E + ns]
        return arr, sizes, nb


def upload_packet(arr: np.ndarray, sizes: List[int], device):
    """One host->device copy of the packet; returns device views in ``sizes`` order."""
    t = torch.from_numpy(arr)
    if device.type == "cuda":
        t = t.pin_memory().to(device, non_blocking=True)
    out, o = [], 0
    for n in sizes:
        out.append(t[o:o + n])
        o += n
    return out


def ep_move(blocks, prefix, total, row_bytes, *, src_table=None, src=None, dst_table=None, dst=None,
            src_ld=None, dst_ld=None):
    """Row-block copy (``ep_copy_rows``) with either side a peer table or a local tensor."""
    from ..ops._ext import ext

    if total == 0:
        return
    sp = src.data_ptr() if src is not None else 0
    dp = dst.data_ptr() if dst is not None else 0
    ext().ep_copy_rows(src_table, sp, dst_table, dp, blocks.view(-1, 4), prefix, total, row_bytes,
                       src_ld or row_bytes, dst_ld or row_bytes)


# ----------------------------------------------------------------------------- PyTorch path
def ep_experts_forward_torch(moe, xf: torch.Tensor, weights: torch.Tensor, experts: torch.Tensor):
    """Routed-expert output ``[N, D]`` (fp32) for tokens ``xf`` routed to global
    expert ids ``experts [N, k]`` with weights ``[N, k]``, plus the ``[W, E]`` count table.
    Differentiable end to end (the exchange is ``all_to_all_single`` with autograd)."""
    from torch.distributed.nn.functional import all_to_all_single

    ep: ExpertParallel = moe.ep
    N, D = xf.shape
    k = experts.shape[1]
    E, El = ep.num_experts, ep.local_experts
    flat_e = experts.reshape(-1)
    counts = torch.bincount(flat_e, minlength=E)
    table = ep.exchange_counts(counts)
    plan = EpPlan(ep, table)
    order = torch.argsort(flat_e, stable=True)                         # compact order
    x_sorted = xf[order // k].contiguous()
    x_recv = all_to_all_single(torch.empty(plan.n_recv, D, dtype=xf.dtype, device=xf.device),
                               x_sorted, plan.recv_splits, plan.send_splits, group=ep.group)
    # rows arrive source-major, local experts in order inside each source
    y_recv = torch.zeros(plan.n_recv, D, dtype=torch.float32, device=xf.device)
    for j in range(El):
        idx = [np.arange(plan.recv_start[s, j], plan.recv_start[s, j] + plan.table[s, plan.lo + j])
               for s in range(ep.world)]
        idx = torch.as_tensor(np.concatenate(idx), dtype=torch.long, device=xf.device)
        if idx.numel():
            y_recv = y_recv.index_add(0, idx, moe._expert(j, x_recv[idx]).float())
    y_sorted = all_to_all_single(torch.empty(N * k, D, dtype=torch.float32, device=xf.device),
                                 y_recv, plan.send_splits, plan.recv_splits, group=ep.group)
    y_flat = torch.zeros_like(y_sorted).index_copy(0, order, y_sorted)  # (token, slot) order
    out = (y_flat.view(N, k, D) * weights.unsqueeze(-1).float()).sum(1)
    return out, table
