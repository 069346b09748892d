"""Tensor parallelism (with sequence-parallel activations) for streaming rollout of the
world model, one process per GPU.

Layout on ``W`` ranks: the token rows of a chunk are sharded (rank r holds rows
``[r M/W, (r+1) M/W)`` of the residual stream); attention heads and the SwiGLU hidden units
are split (heads padded with zero weights up to a multiple of ``W``, e.g. 12 -> 16 on 8
ranks); the KV cache holds only the rank's heads. Per block::

    h1 = adaln_rmsnorm(x_shard)                           local rows
    qkv = all_gather(h1) @ Wqkv_r^T  (+ RoPE)             AG -> GEMM
    o = attention(q_r, K_r, V_r)                          local heads, cached window
    x1 = x_shard + reduce_scatter(o @ Wproj_r^T)          GEMM -> RS
    h2 = adaln_rmsnorm(x1)
    a = swiglu(all_gather(h2) @ W13_r^T)                  AG -> GEMM
    x2 = x1 + reduce_scatter(a @ W3_r^T)                  GEMM -> RS

Small chunks (at most ``replicate_rows_max`` token rows, e.g. a 4-frame chunk at batch 1)
use plain tensor parallelism instead: every rank holds all rows of the residual stream
(AdaLN and the head run on all rows on every rank), the QKV and SwiGLU GEMMs read the
local rows with the rank's column shard of the weights (no all-gather), and the output and
down projections end in an all-reduce: each rank's GEMM writes its partial into its own
peer-readable buffer, one barrier, and ``tp_allreduce_sum`` adds every rank's partial
(P2P loads, fixed rank order, so all ranks hold identical rows) and the residual. That is
two barriers per block instead of four, no gather copies, and every AdaLN modulation of
the forward comes from one GEMM; the bytes crossing NVLink per all-reduce are a few MB at
batch 1, so latency, not bandwidth, sets the cost.

Transports:

``fused``
    The all-gather reads the peers' row shards in peer memory: for narrow GEMMs (one
    column tile per rank) inside the GEMM, whose TMA producer loads the A rows of peer p
    straight out of p's shard (``csrc/gemm/gemm.cu``, per-peer tensor maps, no multicast);
    for wider ones a P2P-load kernel pulls each peer's rows across NVLink once on a side
    stream while the GEMM runs on the rank's own rows (a remote A tile re-read by several
    column tiles would cross NVLink each time). The reduce-scatter happens inside the GEMM: its epilogue
    stores every output tile into the owning rank's receive slot (P2P stores), so the
    transfer overlaps the remaining tiles; the owner then sums its ``W`` slots with the
    residual (``tp_sum_rows``). Bounded cross-rank flag barriers order the phases.
``nccl``
    ``all_gather_into_tensor`` before and ``reduce_scatter_tensor`` after the plain GEMMs.

The reference has no tensor parallelism (its rollout is single-GPU,
``inference/rollout.py:158-492``).
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.distributed as dist


def _head_perm(H: int, W: int):
    """Padded head count and, per rank, its heads (``None`` marks a zero padding head)."""
    Hp = (H + W - 1) // W * W
    per = Hp // W
    return Hp, [[h if h < H else None for h in range(r * per, (r + 1) * per)] for r in range(W)]


class TPLayerWeights:
    def __init__(self, blk, rank: int, W: int, cfg, dtype):
        d, Dh, H = cfg.d_model, cfg.d_head, cfg.n_heads
        Hp, heads = _head_perm(H, W)
        mine = heads[rank]
        self.heads = len(mine)
        dl = self.heads * Dh
        wqkv = blk.attn.qkv.weight.detach().to(dtype)
        wproj = blk.attn.proj.weight.detach().to(dtype)
        q = torch.zeros(3 * dl, d, dtype=dtype, device=wqkv.device)
        p = torch.zeros(d, dl, dtype=dtype, device=wqkv.device)
        for j, h in enumerate(mine):
            if h is None:
                continue
            for s in range(3):
                q[s * dl + j * Dh:s * dl + (j + 1) * Dh] = wqkv[s * d + h * Dh:s * d + (h + 1) * Dh]
            p[:, j * Dh:(j + 1) * Dh] = wproj[:, h * Dh:(h + 1) * Dh]
        self.wqkv, self.wproj = q.contiguous(), p.contiguous()
        w13 = blk.mlp.w13.weight.detach().to(dtype)           # [2F, d], gate/value in groups of 32
        w3 = blk.mlp.w3.weight.detach().to(dtype)             # [d, F]
        F = w3.shape[1]
        if F % (32 * W):
            raise ValueError(f"SwiGLU width {F} does not split into 32-column groups over {W} ranks")
        f0, f1 = rank * F // W, (rank + 1) * F // W
        self.w13 = w13[2 * f0:2 * f1].contiguous()
        self.w3 = w3[:, f0:f1].contiguous()
        self.norm1 = blk.norm1.weight.detach()
        self.norm2 = blk.norm2.weight.detach()
        self.ada = blk.ada


class TPKVCache:
    """Per-layer K/V windows of this rank's heads (the layout of ``LayerKVCache``)."""

    def __init__(self, n_layers, B, window_frames, chunk_frames, tpf, d_local, device, dtype):
        from ..models.world_dit import LayerKVCache

        cap = (2 * window_frames + chunk_frames) * tpf
        self.layers = [LayerKVCache(B, cap, d_local, window_frames * tpf, device, dtype) for _ in range(n_layers)]
        self.frames = 0
        self.tpf = tpf

    def reserve(self, n_tokens: int) -> int:
        return [c.reserve(n_tokens) for c in self.layers][0]

    def commit(self, n_frames: int):
        for c in self.layers:
            c.commit(n_frames * self.tpf)
        self.frames += n_frames


class TensorParallelWorldDiT:
    """Inference-only tensor-parallel view of a :class:`WorldDiT` (same weights on every
    rank before sharding). Plugs into :class:`~drivedit_b200.inference.rollout.StreamingRollout`
    through ``make_kv_cache`` / ``forward_cached_chunk``."""

    def __init__(self, model, group=None, transport: Optional[str] = None, dtype=torch.bfloat16,
                 ag_tma_max_n: int = 256, replicate_rows_max: int = 4096):
        """``ag_tma_max_n``: widest per-rank GEMM (columns) whose all-gather runs inside the
        GEMM as peer TMA loads; wider ones pull the rows once and overlap.
        ``replicate_rows_max``: chunks of at most this many token rows run with the
        residual stream replicated on every rank and all-reduces (see the module notes)."""
        self.model = model
        self.cfg = model.cfg
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = next(model.parameters()).device
        self.transport = transport or ("fused" if self.device.type == "cuda" else "nccl")
        self.dtype = dtype
        self.ag_tma_max_n = ag_tma_max_n
        self.replicate_rows_max = replicate_rows_max
        self._ping = 0
        self._mods_w = None
        self.layers = [TPLayerWeights(b, self.rank, self.world, self.cfg, dtype) for b in model.blocks]
        self.heads_local = self.layers[0].heads
        self.d_local = self.heads_local * self.cfg.d_head
        self._sym = {}
        self._flags = None
        self.epoch = 0

    def parameters(self):
        return self.model.parameters()

    # ---------------------------------------------------------------- symmetric memory
    def _buf(self, name, nbytes):
        from .sharded import SymmetricBuffer

        b = self._sym.get(name)
        if b is None or b.nbytes < nbytes:
            if b is not None:
                b.close()
            b = SymmetricBuffer(int(nbytes), self.group, self.device)
            self._sym[name] = b
        return b

    def _barrier(self):
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

    # ---------------------------------------------------------------- rollout hooks
    def make_kv_cache(self, B, window_frames, chunk_frames, device, dtype):
        return TPKVCache(len(self.layers), B, window_frames, chunk_frames, self.cfg.tokens_per_frame,
                         self.d_local, device, dtype)

    @torch.no_grad()
    def forward_cached_chunk(self, x_t, t, actions, cache: TPKVCache, commit: bool, extra_cond=None):
        if self.device.type != "cuda":
            raise RuntimeError("tensor-parallel rollout runs on the CUDA kernels")
        rows = x_t.shape[0] * x_t.shape[1] * self.cfg.tokens_per_frame
        if rows <= self.replicate_rows_max:
            return self._forward_replicated(x_t, t, actions, cache, commit, extra_cond)
        return self._forward(x_t, t, actions, cache, commit, extra_cond)

    # ---------------------------------------------------------------- replicated rows
    def _all_mods(self, c2):
        """Every block's AdaLN modulation and the head's for the chunk's frames in one
        GEMM (bf16 operands, fp32 accumulation and bias): per-block views of
        ``[frames, n_mod x d]`` and the head's ``[frames, 2 d]``."""
        from ..ops.gemm import gemm

        if self._mods_w is None:
            lins = [lw.ada for lw in self.layers] + [self.model.final_ada]
            ws = [lin.weight.detach() for lin in lins]
            bs = [lin.bias.detach() for lin in lins]
            self._mods_w = (torch.cat(ws).to(torch.bfloat16).contiguous(), torch.cat(bs).float().contiguous(),
                            ws[0].shape[0])
        w, b, per = self._mods_w
        mods = gemm(c2.to(torch.bfloat16).contiguous(), w, epi="f32", bias=b)
        L = len(self.layers)
        return [mods[:, i * per:(i + 1) * per] for i in range(L)], mods[:, L * per:]

    def _allreduce_gemm(self, a, w, residual):
        """``residual + all_reduce(a @ w^T)``: the GEMM writes this rank's partial into its
        peer-readable buffer (two buffers used in turn: a rank writes a buffer again only
        after the next collective's barrier, which every peer reaches after its sum of the
        buffer's previous contents), one barrier, then the peer-load sum."""
        from ..ops._ext import ext
        from ..ops.gemm import gemm

        M, N = a.shape[0], w.shape[0]
        if self.transport == "fused":
            self._ping ^= 1
            buf = self._buf(f"part{self._ping}", M * N * 2)
            part = buf.tensor(M * N, torch.bfloat16).view(M, N)
            gemm(a, w, part)
            self._barrier()                              # every rank's partial is complete
            return ext().tp_allreduce_sum(buf.table, self.world, M * N, part, residual)
        part = gemm(a, w)
        dist.all_reduce(part, group=self.group)
        return part + residual

    def _forward_replicated(self, x_t, t, actions, cache, commit, extra_cond):
        from ..models.world_dit import patchify, unpatchify
        from ..ops._ext import ext
        from ..ops.fused import adaln_rmsnorm
        from ..ops.gemm import gemm

        m, cfg = self.model, self.cfg
        B, Fc, C, H, W_ = x_t.shape
        d, Dh = cfg.d_model, cfg.d_head
        dl, Hl = self.d_local, self.heads_local
        tok = patchify(x_t, cfg.patch).reshape(-1, cfg.patch_dim).to(torch.bfloat16).contiguous()
        M = tok.shape[0]
        T = M // B
        tpf = T // Fc
        x = gemm(tok, m.patch_embed.weight.detach().to(torch.bfloat16), bias=m.patch_embed.bias.detach().float())
        c2 = m.condition(t, actions, extra_cond).reshape(B * Fc, d)
        mods, fm = self._all_mods(c2)
        tab = m.rope.table(Fc, cache.frames).to(x.device)
        row = cache.reserve(T)
        scale = 1.0 / math.sqrt(Dh)
        for lw, lc, mod in zip(self.layers, cache.layers, mods):
            h1, _ = adaln_rmsnorm(x, lw.norm1, mod, 0, d, tpf)
            qkv = gemm(h1, lw.wqkv, epi="rope", rope_tab=tab, rope_cols=2 * dl, rope_rows_per_seq=T,
                       rope_head_dim=Dh)
            q3 = qkv.view(B, T, 3 * dl)
            lc.k[:, row:row + T].copy_(q3[:, :, dl:2 * dl])
            lc.v[:, row:row + T].copy_(q3[:, :, 2 * dl:])
            cap = lc.k.shape[1]
            k2 = lc.k.view(B * cap, dl)[lc.start:]
            v2 = lc.v.view(B * cap, dl)[lc.start:]
            S = row + T - lc.start
            o = torch.empty(M, dl, device=x.device, dtype=torch.bfloat16)
            ext().attn_fwd(qkv, k2, v2, o, None, 0, 0, 0, 0, B, Hl, T, S, T, cap, 1, tpf,
                           lc.pos0 + row, lc.pos0 + lc.start, scale, None, None, None)
            x1 = self._allreduce_gemm(o, lw.wproj, x)
            h2, _ = adaln_rmsnorm(x1, lw.norm2, mod, 2 * d, 3 * d, tpf)
            gu = torch.empty(M, lw.w13.shape[0], device=x.device, dtype=torch.bfloat16)
            a = torch.empty(M, lw.w13.shape[0] // 2, device=x.device, dtype=torch.bfloat16)
            gemm(h2, lw.w13, gu, epi="swiglu", out2=a)
            x = self._allreduce_gemm(a, lw.w3, x1)
        if commit:
            cache.commit(Fc)
        h, _ = adaln_rmsnorm(x, m.final_norm.weight.detach(), fm, 0, d, tpf, cfg.norm_eps)
        out = gemm(h, m.out_proj.weight.detach().to(torch.bfloat16), bias=m.out_proj.bias.detach().float())
        return unpatchify(out.view(B, T, cfg.patch_dim), Fc, C, H, W_, cfg.patch)

    # ---------------------------------------------------------------- collectives
    def _gather_gemm(self, h_shard, h_sym, w, rows, M, epi="bf16", **kw):
        """``all_gather(h) @ w^T``. Fused transport: with at most one 256-column tile per
        rank the GEMM reads the peers' rows itself (TMA loads of peer memory); otherwise a
        copy kernel on a side stream pulls every peer's rows across NVLink once while the
        GEMM runs on this rank's own rows, and the GEMMs over the peers' rows follow (a
        tile of A read by several column tiles would otherwise cross NVLink several times,
        since peer reads are not cached in this GPU's L2)."""
        from ..ops._ext import ext
        from ..ops.gemm import EPI, gemm

        N = w.shape[0]
        sw = epi == "swiglu"
        if self.transport == "fused":
            out = torch.empty(M, N, device=self.device, dtype=torch.bfloat16)
            out2 = torch.empty(M, N // 2, device=self.device, dtype=torch.bfloat16) if sw else None
            T = kw.get("rope_rows_per_seq", 1)
            if N <= self.ag_tma_max_n or self.world == 1:
                ext().gemm_tp(h_sym, w, out, EPI[epi], M, list(self._h_peers), rows, None, 0, 0, 0, out2,
                              kw.get("rope_tab"), kw.get("rope_cols", 0), T, 0, kw.get("rope_head_dim", 64))
                return (out, out2) if sw else out
            W, r = self.world, self.rank
            K = h_sym.shape[1]
            full = self._local("hfull", M, K)
            main = torch.cuda.current_stream()
            side = self._side_stream()
            side.wait_stream(main)
            with torch.cuda.stream(side):
                self._pull_rows(full, K, rows)
                ev = torch.cuda.Event()
                ev.record(side)
            r0 = r * rows

            def part(a, lo, hi):
                if hi <= lo:
                    return
                kw2 = {}
                if epi == "rope":
                    kw2 = dict(rope_tab=kw["rope_tab"], rope_cols=kw["rope_cols"], rope_rows_per_seq=T,
                               rope_pos_offset=lo % T, rope_head_dim=kw.get("rope_head_dim", 64))
                if sw:
                    gemm(a, w, out[lo:hi], epi="swiglu", out2=out2[lo:hi])
                else:
                    gemm(a, w, out[lo:hi], epi=epi, **kw2)

            part(h_sym, r0, r0 + rows)                   # own rows while the peers' rows arrive
            main.wait_event(ev)
            part(full[:r0], 0, r0)
            part(full[r0 + rows:], r0 + rows, M)
            full.record_stream(main)
            return (out, out2) if sw else out
        full = torch.empty(M, h_shard.shape[1], device=self.device, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(full, h_shard.contiguous(), group=self.group)
        if sw:
            out = torch.empty(M, N, device=self.device, dtype=torch.bfloat16)
            a = torch.empty(M, N // 2, device=self.device, dtype=torch.bfloat16)
            gemm(full, w, out, epi="swiglu", out2=a)
            return out, a
        return gemm(full, w, epi=epi, **kw)

    def _local(self, name, rows, cols):
        t = getattr(self, "_locals", {}).get(name)
        if t is None or t.shape != (rows, cols):
            t = torch.empty(rows, cols, device=self.device, dtype=torch.bfloat16)
            self._locals = {**getattr(self, "_locals", {}), name: t}
        return t

    def _side_stream(self):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(self.device)
        return self._side

    def _pull_rows(self, full, K, rows):
        """Every peer's row shard -> its rows of ``full`` (one P2P-load kernel)."""
        from ..ops._ext import ext

        key = (rows, K)
        if getattr(self, "_pull_key", None) != key:
            peers = [p for p in range(self.world) if p != self.rank]
            self._pull_blocks = torch.tensor([[p, 0, 0, p * rows] for p in peers], dtype=torch.int32,
                                             device=self.device)
            self._pull_prefix = torch.arange(0, len(peers) * rows, rows, dtype=torch.int32, device=self.device)
            self._pull_key = key
        hb = self._sym["h"]
        ext().ep_copy_rows(hb.table, 0, None, full.data_ptr(), self._pull_blocks, self._pull_prefix,
                           (self.world - 1) * rows, K * 2, K * 2, K * 2)

    def _gemm_scatter(self, a, w, rows, residual):
        """``residual + reduce_scatter(a @ w^T)`` for this rank's rows."""
        from ..ops._ext import ext
        from ..ops.gemm import EPI, gemm

        M, N = a.shape[0], w.shape[0]
        if self.transport == "fused":
            recv = self._buf("recv", self.world * rows * N * 2)
            ext().gemm_tp(a, w, None, EPI["bf16"], M, [], 0, recv.table, rows, self.rank, N, None, None, 0, 1, 0,
                          64)
            self._barrier()                              # every rank's partial rows have landed
            return ext().tp_sum_rows(recv.tensor(self.world * rows * N, torch.bfloat16).view(-1, N),
                                     self.world, rows, residual)
        part = gemm(a, w)
        out = torch.empty(rows, N, device=self.device, dtype=torch.bfloat16)
        dist.reduce_scatter_tensor(out, part, group=self.group)
        return out + residual

    def _publish(self, h, rows):
        """Row shard ``h`` into the peer-readable buffer (fused transport)."""
        if self.transport != "fused":
            return h, h
        d = h.shape[1]
        hb = self._buf("h", rows * max(d, 1) * 2)
        view = hb.tensor(rows * d, torch.bfloat16).view(rows, d)
        view.copy_(h)
        self._h_peers = [int(p) for p in hb.peers]
        self._barrier()                                  # every rank's shard is complete
        return h, view

    def _forward(self, x_t, t, actions, cache, commit, extra_cond):
        from ..models.world_dit import patchify, unpatchify
        from ..ops._ext import ext
        from ..ops.fused import adaln_rmsnorm
        from ..ops.gemm import gemm

        m, cfg = self.model, self.cfg
        W, r = self.world, self.rank
        B, Fc, C, H, W_ = x_t.shape
        d, Dh = cfg.d_model, cfg.d_head
        dl, Hl = self.d_local, self.heads_local
        tok = patchify(x_t, cfg.patch).reshape(-1, cfg.patch_dim).to(torch.bfloat16).contiguous()
        M = tok.shape[0]
        T = M // B
        tpf = T // Fc
        if M % (128 * W):
            raise ValueError(f"{M} token rows do not split into 128-row tiles over {W} ranks")
        rows = M // W
        if not (rows % tpf == 0 or tpf % rows == 0):
            raise ValueError("row shards must nest in frames")
        r0 = r * rows
        g0 = r0 // tpf
        wpe = m.patch_embed.weight.detach().to(torch.bfloat16)
        x = gemm(tok[r0:r0 + rows].contiguous(), wpe, bias=m.patch_embed.bias.detach().float())
        c2 = m.condition(t, actions, extra_cond).reshape(B * Fc, d)
        tab = m.rope.table(Fc, cache.frames).to(x.device)
        row = cache.reserve(T)
        scale = 1.0 / math.sqrt(Dh)
        for lw, lc in zip(self.layers, cache.layers):
            mod = lw.ada(c2)[g0:]
            h1, _ = adaln_rmsnorm(x, lw.norm1, mod, 0, d, tpf)
            h1, h1s = self._publish(h1, rows)
            qkv = self._gather_gemm(h1, h1s, lw.wqkv, rows, M, epi="rope", rope_tab=tab, rope_cols=2 * dl,
                                    rope_rows_per_seq=T, rope_head_dim=Dh)
            q3 = qkv.view(B, T, 3 * dl)
            lc.k[:, row:row + T].copy_(q3[:, :, dl:2 * dl])
            lc.v[:, row:row + T].copy_(q3[:, :, 2 * dl:])
            cap = lc.k.shape[1]
            k2 = lc.k.view(B * cap, dl)[lc.start:]
            v2 = lc.v.view(B * cap, dl)[lc.start:]
            S = row + T - lc.start
            o = torch.empty(M, dl, device=x.device, dtype=torch.bfloat16)
            ext().attn_fwd(qkv, k2, v2, o, None, 0, 0, 0, 0, B, Hl, T, S, T, cap, 1, tpf,
                           lc.pos0 + row, lc.pos0 + lc.start, scale, None, None, None)
            x1 = self._gemm_scatter(o, lw.wproj, rows, x)
            h2, _ = adaln_rmsnorm(x1, lw.norm2, mod, 2 * d, 3 * d, tpf)
            h2, h2s = self._publish(h2, rows)
            _, a = self._gather_gemm(h2, h2s, lw.w13, rows, M, epi="swiglu")
            x = self._gemm_scatter(a, lw.w3, rows, x1)
        if commit:
            cache.commit(Fc)
        fm = m.final_ada(c2)[g0:]
        h, _ = adaln_rmsnorm(x, m.final_norm.weight.detach(), fm, 0, d, tpf, cfg.norm_eps)
        out_sh = gemm(h, m.out_proj.weight.detach().to(torch.bfloat16), bias=m.out_proj.bias.detach().float())
        out = torch.empty(M, out_sh.shape[1], device=x.device, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(out, out_sh.contiguous(), group=self.group)
        return unpatchify(out.view(B, T, cfg.patch_dim), Fc, C, H, W_, cfg.patch)
