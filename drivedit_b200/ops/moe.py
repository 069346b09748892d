"""Fused MoE FFN on sm_100a: routing -> dispatch -> grouped tcgen05 GEMMs -> combine.

Forward (``N`` tokens, ``E`` routed + ``ns`` shared experts, top-``k``):
  logits = h Wr^T                            gemm.cu (fp32 out)
  route: softmax(+bias), top-k, renormalise, shared gates, counts, prob sums   moe.cu
  plan: 128-row padded expert segments + grouped-GEMM tile tables (device side: no
        host synchronisation on expert counts)
  dispatch: token rows -> expert segments     moe.cu
  gu, a = grouped GEMM(x_perm, W13[e]) with the SwiGLU epilogue
  y     = grouped GEMM(a, W2[e])
  out   = residual + sum_j w_j y[slot(t, j)]  moe.cu (combine)
Backward: combine backward (dy, d weights) -> grouped GEMM with the dSwiGLU epilogue ->
grouped weight-gradient GEMMs reducing over each expert's segment (fp32 into the flat
gradient buffer) -> grouped dgrad -> gather-sum to tokens; router gradients (softmax /
top-k renormalisation / shared gates / aux loss) through ``[N, E]`` PyTorch ops and two
small GEMMs.

Reference semantics: layers/moe.py:73-424.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from ._ext import ext
from .gemm import EPI, gemm


def _max_mtiles(N: int, E: int, k: int, ns: int) -> int:
    return (N * k + 127) // 128 + E + ns * ((N + 127) // 128)


def moe_ffn_forward(h: torch.Tensor, residual: torch.Tensor, moe, W):
    """Returns (out, aux_loss_value, saved) for ``h [N, d]`` bf16."""
    N, d = h.shape
    E, k, ns = moe.num_experts, moe.top_k, moe.num_shared_experts
    Fh = moe.expert_dim
    Ep = E + ns
    logits = gemm(h, W(moe.router_weight), epi="f32")
    idx, w, sw, probs, counts, psum = ext().moe_route(logits, moe.expert_bias, E, k, ns, True)
    mt = _max_mtiles(N, E, k, ns)
    seg_start, seg_count, t_exp, t_row, total, kstart, kend, cursor = ext().moe_plan(
        counts, E, ns, N, mt)
    rows = mt * 128
    xp = torch.empty(rows, d, device=h.device, dtype=torch.bfloat16)
    slot_of = ext().moe_dispatch(h, idx, seg_start, seg_count, cursor, xp, E, ns)
    w13 = W(moe.w13)        # [Ep, 2F, d]
    w2 = W(moe.w2)          # [Ep, d, F]
    gu = torch.empty(rows, 2 * Fh, device=h.device, dtype=torch.bfloat16)
    act = torch.empty(rows, Fh, device=h.device, dtype=torch.bfloat16)
    tables = (t_exp, t_row, total, kstart, kend, mt)
    ext().gemm_grouped(xp, w13, gu, EPI["swiglu"], False, 1, *tables, None, act)
    y = torch.empty(rows, d, device=h.device, dtype=torch.bfloat16)
    ext().gemm_grouped(act, w2, y, EPI["bf16"], False, 1, *tables, None, None)
    out = ext().moe_combine(w, sw, slot_of, y, residual, ns)
    f = counts.float() / (N * k)
    P = psum / N
    aux = E * (f * P).sum()
    moe.update_bias(counts, N)
    saved = dict(h=h, idx=idx, w=w, sw=sw, probs=probs, f=f, slot_of=slot_of, xp=xp, gu=gu,
                 act=act, y=y, tables=tables)
    return out, aux, saved


def moe_ffn_backward(dout: torch.Tensor, d_aux, moe, W, sv) -> torch.Tensor:
    """Gradient w.r.t. the FFN input ``h``; accumulates the expert / router weight
    gradients into their flat-buffer ``.grad`` views. ``dout`` is the gradient of the
    block output (the residual path is handled by the caller)."""
    h = sv["h"]
    N, d = h.shape
    E, k, ns = moe.num_experts, moe.top_k, moe.num_shared_experts
    Fh = moe.expert_dim
    Ep = E + ns
    tables = sv["tables"]
    dy, dw = ext().moe_combine_bwd(sv["w"], sv["sw"], sv["slot_of"], sv["y"], dout, ns)
    rows = dy.shape[0]
    w13, w2 = W(moe.w13), W(moe.w2)
    dgu = torch.empty(rows, 2 * Fh, device=h.device, dtype=torch.bfloat16)
    ext().gemm_grouped(dy, w2, dgu, EPI["dswiglu"], True, 1, *tables, sv["gu"], None)
    g_w2 = moe.w2.grad.view(Ep * d, Fh)
    ext().gemm_grouped(dy, sv["act"], g_w2, EPI["f32_acc"], True, 2, *tables, None, None)
    dxp = torch.empty(rows, d, device=h.device, dtype=torch.bfloat16)
    ext().gemm_grouped(dgu, w13, dxp, EPI["bf16"], True, 1, *tables, None, None)
    g_w13 = moe.w13.grad.view(Ep * 2 * Fh, d)
    ext().gemm_grouped(dgu, sv["xp"], g_w13, EPI["f32_acc"], True, 2, *tables, None, None)
    dh = ext().moe_unpermute(dxp, sv["slot_of"], N)
    dlog = router_dlogits(sv["probs"], sv["idx"], sv["w"], sv["sw"], dw, d_aux, sv["f"],
                          E, k, ns, moe.e_pad)
    dlog = dlog.to(torch.bfloat16)
    gemm(dlog, h, moe.router_weight.grad, epi="f32_acc", a_t=True, b_t=True)
    gemm(dlog, W(moe.router_weight), dh, b_t=True, residual=dh)
    return dh


def router_dlogits(p, idx, w, sw, dw, d_aux, f, E: int, k: int, ns: int, e_pad: int):
    """Gradient of the loss w.r.t. the router logits ``[N, e_pad]`` (fp32).

    ``dw [N, k+ns]`` is the gradient w.r.t. the combine weights (renormalised top-k
    gates, then shared gates). The routed part goes back through the top-k
    renormalisation ``w_j = p_j / sum_top p`` and ``p = softmax(logits + bias)``; the aux
    load-balance loss ``E * sum_e f_e mean_n p_ne`` adds ``d_aux * E/N * f`` to ``dp``
    (``f`` is a count share, not differentiated); shared gates are a plain softmax.
    """
    N = p.shape[0]
    idx = idx.long()
    dwr = dw[:, :k].float()
    stop = torch.gather(p, 1, idx).sum(-1, keepdim=True)
    dptop = (dwr - (dwr * w).sum(-1, keepdim=True)) / (stop + 1e-8)
    dp = torch.zeros_like(p).scatter_(1, idx, dptop)
    if d_aux is not None:  # a 0-dim device tensor: no host synchronisation
        dp = dp + d_aux.float() * (E / N) * f[None, :]
    dz = p * (dp - (p * dp).sum(-1, keepdim=True))
    dlog = torch.zeros(N, e_pad, device=p.device, dtype=torch.float32)
    dlog[:, :E] = dz
    if ns:
        g = sw[:, :ns].float()
        dws = dw[:, k:].float()
        dlog[:, E:E + ns] = g * (dws - (g * dws).sum(-1, keepdim=True))
    return dlog


# ----------------------------------------------------------------------------- expert parallel
def _grouped_ffn(x, w13, w2, tables, Fh):
    rows, d = x.shape
    gu = torch.empty(rows, 2 * Fh, device=x.device, dtype=torch.bfloat16)
    act = torch.empty(rows, Fh, device=x.device, dtype=torch.bfloat16)
    ext().gemm_grouped(x, w13, gu, EPI["swiglu"], False, 1, *tables, None, act)
    y = torch.empty(rows, d, device=x.device, dtype=torch.bfloat16)
    ext().gemm_grouped(act, w2, y, EPI["bf16"], False, 1, *tables, None, None)
    return gu, act, y


def _grouped_ffn_bwd(dy, x, gu, act, w13, w2, g13, g2, tables, Fh):
    """dx of the grouped SwiGLU FFN; weight gradients accumulate into ``g13 / g2``."""
    rows, d = dy.shape
    dgu = torch.empty(rows, 2 * Fh, device=dy.device, dtype=torch.bfloat16)
    ext().gemm_grouped(dy, w2, dgu, EPI["dswiglu"], True, 1, *tables, gu, None)
    ext().gemm_grouped(dy, act, g2, EPI["f32_acc"], True, 2, *tables, None, None)
    dx = torch.empty(rows, d, device=dy.device, dtype=torch.bfloat16)
    ext().gemm_grouped(dgu, w13, dx, EPI["bf16"], True, 1, *tables, None, None)
    ext().gemm_grouped(dgu, x, g13, EPI["f32_acc"], True, 2, *tables, None, None)
    return dx


def _route(h, moe, W):
    E, k, ns = moe.num_experts, moe.top_k, moe.num_shared_experts
    logits = gemm(h, W(moe.router_weight), epi="f32")
    return ext().moe_route(logits, moe.expert_bias, E, k, ns, True)


def _shared_forward(h, moe, W, ep):
    """Shared experts on the local tokens: dispatch into their 128-row segments and the
    grouped SwiGLU FFN. Returns (slot_of [N, ns], xs, gu, act, y, tables) or Nones."""
    ns = moe.num_shared_experts
    if not ns:
        return None, None, None, None, None, None
    N, d = h.shape
    sp, mt_s = ep.shared_plan(N, ns)
    xs = torch.empty(mt_s * 128, d, device=h.device, dtype=torch.bfloat16)
    none = torch.empty(N, 0, device=h.device, dtype=torch.int32)
    slot_s = ext().moe_dispatch(h, none, sp[0], sp[1], sp[7], xs, 0, ns)
    tables = (sp[2], sp[3], sp[4], sp[5], sp[6], mt_s)
    gu, act, y = _grouped_ffn(xs, W(moe.w13_shared), W(moe.w2_shared), tables, moe.expert_dim)
    return slot_s, xs, gu, act, y, tables


def _shared_backward(dout, moe, W, sv):
    """(dw_shared [N, ns], dx rows of the shared segments) for the local tokens."""
    ns = moe.num_shared_experts
    N, d = dout.shape
    if not ns:
        return torch.empty(N, 0, device=dout.device), None
    w0 = torch.empty(N, 0, device=dout.device, dtype=torch.float32)
    dys, dws = ext().moe_combine_bwd(w0, sv["sw"], sv["slot_s"], sv["y_s"], dout, ns)
    Fh = moe.expert_dim
    dxs = _grouped_ffn_bwd(dys, sv["xs"], sv["gu_s"], sv["act_s"], W(moe.w13_shared), W(moe.w2_shared),
                           moe.w13_shared.grad.view(ns * 2 * Fh, d), moe.w2_shared.grad.view(ns * d, Fh),
                           sv["tables_s"], Fh)
    return dws, dxs


def _router_backward(h, dw, d_aux, dh, moe, W, sv):
    E, k, ns = moe.num_experts, moe.top_k, moe.num_shared_experts
    dlog = router_dlogits(sv["probs"], sv["idx"], sv["w"], sv["sw"], dw, d_aux, sv["f"],
                          E, k, ns, moe.e_pad)
    dlog = dlog.to(torch.bfloat16)
    gemm(dlog, h, moe.router_weight.grad, epi="f32_acc", a_t=True, b_t=True)
    gemm(dlog, W(moe.router_weight), dh, b_t=True, residual=dh)
    return dh


def _finish_forward(moe, ep, counts, psum, table, N):
    E, k = moe.num_experts, moe.top_k
    f = counts.float() / (N * k)
    aux = E * (f * (psum / N)).sum()
    gcounts = torch.from_numpy(table.sum(0)).to(counts.device, non_blocking=True)
    moe.update_bias(gcounts, N * ep.world)
    return f, aux


def _owner_plan(ep, plan, N, device):
    """Owner-layout tables of this rank's local experts (counts from the table)."""
    lcounts = torch.from_numpy(plan.local_counts.astype("int32")).to(device, non_blocking=True)
    rp = ext().moe_plan(lcounts, ep.local_experts, 0, N, max(plan.owner_mtiles, 1))
    return rp, (rp[2], rp[3], rp[4], rp[5], rp[6], plan.owner_mtiles)


def moe_ffn_forward_ep(h: torch.Tensor, residual: torch.Tensor, moe, W):
    """Expert-parallel form of :func:`moe_ffn_forward` (``moe.ep`` set): the
    ``fused`` transport moves rows over NVLink peer memory, ``nccl`` with all-to-all."""
    if moe.ep.transport == "fused":
        return _ep_forward_fused(h, residual, moe, W)
    return _ep_forward_nccl(h, residual, moe, W)


def moe_ffn_backward_ep(dout: torch.Tensor, d_aux, moe, W, sv) -> torch.Tensor:
    if moe.ep.transport == "fused":
        return _ep_backward_fused(dout, d_aux, moe, W, sv)
    return _ep_backward_nccl(dout, d_aux, moe, W, sv)


# ---- fused transport: owner-driven, one row per (token, owner rank) each way
# Optional stage timing for benchmarks: when EP_TRACE is a list, CUDA events are appended
# as (stage, event) at the stage boundaries of the fused forward / backward.
EP_TRACE = None


def _mark(stage: str):
    if EP_TRACE is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        EP_TRACE.append((stage, ev))


def _ep_forward_fused(h, residual, moe, W):
    """route -> every source pushes each token row once to every rank owning one of its
    experts (``ep_push_rows``: P2P stores into the owner's staging rows, with the token's
    routing for that owner) -> count table (one barrier and host sync; the pushes have
    landed) -> each owner fans its staged rows out into its expert segments
    (``ep_owner_fanout``, local copies) -> local experts' grouped GEMMs -> per-token
    partial sums over the owner's experts stored into the sources' return buffers
    (``ep_owner_scatter_sum``; the shared experts' GEMMs run meanwhile) -> barrier ->
    ``ep_source_reduce``: residual + the owners' partials + gated shared experts."""
    from ..parallel.expert import EpPlan

    ep = moe.ep
    N, d = h.shape
    E, k, ns, Fh = moe.num_experts, moe.top_k, moe.num_shared_experts, moe.expert_dim
    Wd = ep.world
    El = ep.local_experts
    lo = ep.rank * El
    cap = Wd * N
    _mark("fwd.start")
    idx, w, sw, probs, counts, psum = _route(h, moe, W)
    _mark("fwd.route")
    stage = ep.sym("stage", cap * d * 2)
    smeta = ep.sym("smeta", cap * (1 + 2 * k) * 4)
    ocnt = torch.zeros(Wd, device=h.device, dtype=torch.int32)
    pos = torch.empty(N, Wd, device=h.device, dtype=torch.int32)
    ext().ep_push_rows(idx, w, h, stage.table, smeta.table, ocnt, pos, Wd, ep.rank, El)
    _mark("fwd.push")
    full = ep.exchange_counts(torch.cat([counts.to(torch.int32), ocnt]))  # barrier: pushes landed
    table = full[:, :E]
    _mark("fwd.counts")
    if not (table.sum(1) == N * k).all():
        raise RuntimeError("expert parallelism needs the same number of tokens on every rank")
    plan = EpPlan(ep, table)
    rp, tables_r = _owner_plan(ep, plan, N, h.device)
    uniq = full[:, E + ep.rank]                   # rows each source pushed to me
    prefix_h = np.concatenate([[0], np.cumsum(uniq)]).astype(np.int32)
    total = int(prefix_h[-1])
    prefix = torch.from_numpy(prefix_h).to(h.device, non_blocking=True)
    meta = torch.empty(max(total, 1), 2 + k, device=h.device, dtype=torch.int32)
    meta_w = torch.empty(max(total, 1), k, device=h.device, dtype=torch.float32)
    urow = torch.empty(max(total, 1), device=h.device, dtype=torch.int32)
    n_uniq = torch.zeros(1, device=h.device, dtype=torch.int32)
    xr = torch.empty(max(plan.owner_rows, 1), d, device=h.device, dtype=torch.bfloat16)
    _mark("fwd.plan")
    ext().ep_owner_fanout(stage.ptr, smeta.ptr, prefix, total, Wd, N, k, d, lo, El, rp[0], rp[7], xr, meta,
                          meta_w, urow, n_uniq)
    _mark("fwd.gather")
    gu_r = act_r = None
    y_r = xr
    if plan.owner_rows:
        ext().moe_zero_pad(rp[0], rp[1], xr)
        gu_r, act_r, y_r = _grouped_ffn(xr, W(moe.w13), W(moe.w2), tables_r, Fh)
    _mark("fwd.experts")
    ret = ep.sym("ret", cap * d * 2)
    # owner-side arguments (the three peer tables are unused by these kernels)
    base = (stage.table, stage.table, stage.table, Wd, ep.rank, N, k, d, lo, El, rp[0], rp[7], meta, meta_w,
            n_uniq)
    ext().ep_owner_scatter_sum(*base, y_r, True, ret.table)
    _mark("fwd.scatter")
    slot_s, xs, gu_s, act_s, y_s, tables_s = _shared_forward(h, moe, W, ep)
    _mark("fwd.shared")
    ep.barrier()                                  # every owner's partial rows have landed
    _mark("fwd.barrier")
    out = ext().ep_source_reduce(idx, ret.tensor(cap * d, torch.bfloat16).view(cap, d), El, residual,
                                 sw if ns else None, slot_s, y_s)
    _mark("fwd.reduce")
    f, aux = _finish_forward(moe, ep, counts, psum, table, N)
    saved = dict(h=h, idx=idx, w=w, sw=sw, probs=probs, f=f, plan=plan, owner=base[3:], rp=rp,
                 tables_r=tables_r, xr=xr, gu_r=gu_r, act_r=act_r, y_r=y_r, slot_s=slot_s, xs=xs,
                 gu_s=gu_s, act_s=act_s, y_s=y_s, tables_s=tables_s, pos=pos, urow=urow)
    return out, aux, saved


def _ep_backward_fused(dout, d_aux, moe, W, sv):
    """every source pushes its dout rows to the owners' staging rows of the forward
    (``ep_push_rows`` in gradient mode) -> barrier -> each owner reads them locally, writes
    ``dy = w dout`` into its segments and stores ``dw = dout . y`` into the source
    (``ep_owner_grad_gather``) -> local experts' backward GEMMs -> per-token sums of ``dx``
    over the owner's experts pushed back -> barrier -> sources add them up."""
    ep = moe.ep
    h = sv["h"]
    N, d = h.shape
    k, ns, Fh = moe.top_k, moe.num_shared_experts, moe.expert_dim
    El = ep.local_experts
    plan = sv["plan"]
    Wd = ep.world
    cap = Wd * N
    _mark("bwd.start")
    dstage = ep.sym("dstage", cap * d * 2)
    ext().ep_push_rows(sv["idx"], None, dout, dstage.table, None, None, sv["pos"], Wd, ep.rank, El)
    _mark("bwd.push")
    dwb = ep.sym("dw", N * k * 4)
    dws, dxs = _shared_backward(dout, moe, W, sv)
    _mark("bwd.shared")
    ep.barrier()                                  # every rank's dout rows have landed
    _mark("bwd.barrier1")
    owner = (dstage.table, dstage.table, dstage.table) + sv["owner"]
    dyr = torch.empty(max(plan.owner_rows, 1), d, device=h.device, dtype=torch.bfloat16)
    ext().ep_owner_grad_gather(*owner, sv["y_r"], dyr, dwb.table, local_rows=dstage.ptr, urow=sv["urow"])
    _mark("bwd.gather")
    dxr = dyr
    if plan.owner_rows:
        ext().moe_zero_pad(sv["rp"][0], sv["rp"][1], dyr)
        dxr = _grouped_ffn_bwd(dyr, sv["xr"], sv["gu_r"], sv["act_r"], W(moe.w13), W(moe.w2),
                               moe.w13.grad.view(El * 2 * Fh, d), moe.w2.grad.view(El * d, Fh),
                               sv["tables_r"], Fh)
    _mark("bwd.experts")
    dret = ep.sym("dret", cap * d * 2)
    ext().ep_owner_scatter_sum(*owner, dxr, False, dret.table)
    _mark("bwd.scatter")
    ep.barrier()                                  # every dx partial and dw value has landed
    _mark("bwd.barrier2")
    dh = ext().ep_source_reduce(sv["idx"], dret.tensor(cap * d, torch.bfloat16).view(cap, d), El,
                                None, None, sv["slot_s"], dxs)
    _mark("bwd.reduce")
    dw = torch.cat([dwb.tensor(N * k, torch.float32).view(N, k), dws], 1)
    return _router_backward(h, dw, d_aux, dh, moe, W, sv)


# ---- nccl transport: compact rows sorted by expert, all_to_all, local re-layout
def _ep_forward_nccl(h, residual, moe, W):
    import torch.distributed as dist

    from ..parallel.expert import EpPlan, ep_move, upload_packet

    ep = moe.ep
    N, d = h.shape
    E, k, ns, Fh = moe.num_experts, moe.top_k, moe.num_shared_experts, moe.expert_dim
    El = ep.local_experts
    idx, w, sw, probs, counts, psum = _route(h, moe, W)
    table = ep.exchange_counts(counts)
    plan = EpPlan(ep, table)
    arr, sizes, nb = plan.packet(ep, N, ns, k)
    pull_b, pull_p, push_b, push_p, lcounts, seg_start, seg_count, cursor = upload_packet(
        arr, sizes, h.device)
    rb = 2 * d
    send = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
    # routed rows only (compact, sorted by expert); shared experts go their own way
    slot_of = ext().moe_dispatch(h, idx, seg_start[:E], seg_count[:E], cursor[:E], send, E, 0, None, False)
    recv = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
    dist.all_to_all_single(recv[:plan.n_recv], send[:N * k], plan.recv_splits, plan.send_splits,
                           group=ep.group)
    xr = torch.empty(max(plan.owner_rows, 1), d, device=h.device, dtype=torch.bfloat16)
    ep_move(pull_b, pull_p, plan.n_recv, rb, src=recv, dst=xr)
    rp, tables_r = _owner_plan(ep, plan, N, h.device)
    gu_r = act_r = None
    y_r = xr
    if plan.owner_rows:
        ext().moe_zero_pad(rp[0], rp[1], xr)
        gu_r, act_r, y_r = _grouped_ffn(xr, W(moe.w13), W(moe.w2), tables_r, Fh)
    stage = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
    ep_move(push_b, push_p, plan.n_recv, rb, src=y_r, dst=stage)
    yret = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
    dist.all_to_all_single(yret[:N * k], stage[:plan.n_recv], plan.send_splits, plan.recv_splits,
                           group=ep.group)
    slot_s, xs, gu_s, act_s, y_s, tables_s = _shared_forward(h, moe, W, ep)
    if ns:   # routed slots index yret, shared slots index y_s
        slot_all = torch.cat([slot_of, slot_s], 1).contiguous()
        out = ext().moe_combine(w, sw, slot_all, yret, residual, ns, y_s)
    else:
        out = ext().moe_combine(w, sw, slot_of, yret, residual, 0)
    f, aux = _finish_forward(moe, ep, counts, psum, table, N)
    saved = dict(h=h, idx=idx, w=w, sw=sw, probs=probs, f=f, slot_of=slot_of, plan=plan,
                 pull=(pull_b, pull_p), push=(push_b, push_p), xr=xr, gu_r=gu_r, act_r=act_r,
                 rp=rp, tables_r=tables_r, yret=yret, slot_s=slot_s, xs=xs, gu_s=gu_s, act_s=act_s,
                 y_s=y_s, tables_s=tables_s)
    return out, aux, saved


def _ep_backward_nccl(dout, d_aux, moe, W, sv):
    import torch.distributed as dist

    from ..parallel.expert import ep_move

    ep = moe.ep
    h = sv["h"]
    N, d = h.shape
    E, k, ns, Fh = moe.num_experts, moe.top_k, moe.num_shared_experts, moe.expert_dim
    El = ep.local_experts
    plan, rb = sv["plan"], 2 * d
    dy_c, dw_r = ext().moe_combine_bwd(sv["w"], sv["sw"], sv["slot_of"], sv["yret"], dout, 0)
    recv = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
    dist.all_to_all_single(recv[:plan.n_recv], dy_c[:N * k], plan.recv_splits, plan.send_splits,
                           group=ep.group)
    dyr = torch.empty(max(plan.owner_rows, 1), d, device=h.device, dtype=torch.bfloat16)
    ep_move(*sv["pull"], plan.n_recv, rb, src=recv, dst=dyr)
    dxr = dyr
    if plan.owner_rows:
        ext().moe_zero_pad(sv["rp"][0], sv["rp"][1], dyr)
        dxr = _grouped_ffn_bwd(dyr, sv["xr"], sv["gu_r"], sv["act_r"], W(moe.w13), W(moe.w2),
                               moe.w13.grad.view(El * 2 * Fh, d), moe.w2.grad.view(El * d, Fh),
                               sv["tables_r"], Fh)
    stage = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
    ep_move(*sv["push"], plan.n_recv, rb, src=dxr, dst=stage)
    dret = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
    dist.all_to_all_single(dret[:N * k], stage[:plan.n_recv], plan.send_splits, plan.recv_splits,
                           group=ep.group)
    dws, dxs = _shared_backward(dout, moe, W, sv)
    if ns:   # routed slots index dret, shared slots index dxs
        dh = ext().moe_unpermute(dret, torch.cat([sv["slot_of"], sv["slot_s"]], 1).contiguous(), N, dxs, k)
    else:
        dh = ext().moe_unpermute(dret, sv["slot_of"], N)
    dw = torch.cat([dw_r, dws], 1)
    return _router_backward(h, dw, d_aux, dh, moe, W, sv)
