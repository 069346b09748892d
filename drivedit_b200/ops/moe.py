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


def moe_ffn_forward_ep(h: torch.Tensor, residual: torch.Tensor, moe, W):
    """Expert-parallel form of :func:`moe_ffn_forward` (``moe.ep`` set).

    route (local) -> count table exchange -> compact dispatch of the routed rows into the
    send buffer (shared-expert rows into the local shared layout) -> owner pull into the
    grouped-GEMM layout -> local experts' grouped GEMMs -> push of the outputs into the
    sources' return buffers (the shared experts' GEMMs run meanwhile) -> combine.
    """
    import torch.distributed as dist

    from ..parallel.expert import EpPlan, ep_move, upload_packet

    ep = moe.ep
    N, d = h.shape
    E, k, ns, Fh = moe.num_experts, moe.top_k, moe.num_shared_experts, moe.expert_dim
    El = ep.local_experts
    fused = ep.transport == "fused"
    logits = gemm(h, W(moe.router_weight), epi="f32")
    idx, w, sw, probs, counts, psum = ext().moe_route(logits, moe.expert_bias, E, k, ns, True)
    table = ep.exchange_counts(counts)                       # host: [W, E]
    plan = EpPlan(ep, table)
    arr, sizes, nb = plan.packet(ep, N, ns, k)
    pull_b, pull_p, push_b, push_p, lcounts, seg_start, seg_count, cursor = upload_packet(
        arr, sizes, h.device)
    rb = 2 * d
    cap = int(table.sum(1).max())                            # same on every rank
    assert plan.n_routed == N * k
    xs = None
    if ns:
        sp, mt_s = ep.shared_plan(N, ns)
        xs = torch.empty(mt_s * 128, d, device=h.device, dtype=torch.bfloat16)
    if fused:
        sbuf = ep.sym("send", cap * rb)
        send = sbuf.tensor(cap * d, torch.bfloat16).view(cap, d)
    else:
        send = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
    slot_of = ext().moe_dispatch(h, idx, seg_start, seg_count, cursor, send, E, ns, xs, False)
    # ---- dispatch: the owner gathers its experts' rows from every source
    xr = torch.empty(max(plan.owner_rows, 1), d, device=h.device, dtype=torch.bfloat16)
    if fused:
        ep.barrier()                                         # every send buffer is complete
        ep_move(pull_b, pull_p, plan.n_recv, rb, src_table=sbuf.table, dst=xr)
    else:
        recv = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
        dist.all_to_all_single(recv[:plan.n_recv], send[:N * k], plan.recv_splits, plan.send_splits,
                               group=ep.group)
        ep_move(pull_b, pull_p, plan.n_recv, rb, src=recv, dst=xr)
    rp = ext().moe_plan(lcounts, El, 0, N, max(plan.owner_mtiles, 1))
    seg_r = (rp[0], rp[1])
    tables_r = (rp[2], rp[3], rp[4], rp[5], rp[6], plan.owner_mtiles)
    w13, w2 = W(moe.w13), W(moe.w2)
    gu_r = act_r = None
    y_r = xr
    if plan.owner_rows:
        ext().moe_zero_pad(seg_r[0], seg_r[1], xr)
        gu_r, act_r, y_r = _grouped_ffn(xr, w13, w2, tables_r, Fh)
    # ---- combine side: outputs back to the sources' compact return buffers
    if fused:
        rbuf = ep.sym("ret", ep.n_layers * cap * rb)
        ret_tab = ep.slot_table("ret", moe.ep_slot, cap * rb)
        ep_move(push_b, push_p, plan.n_recv, rb, src=y_r, dst_table=ret_tab)
        yret = rbuf.tensor(cap * d, torch.bfloat16, moe.ep_slot * cap * rb).view(cap, d)
    else:
        stage = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
        ep_move(push_b, push_p, plan.n_recv, rb, src=y_r, dst=stage)
        yret = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
        dist.all_to_all_single(yret[:N * k], stage[:plan.n_recv], plan.send_splits, plan.recv_splits,
                               group=ep.group)
    gu_s = act_s = y_s = None
    if ns:   # shared experts on the local tokens while the peers finish
        tables_s = (sp[2], sp[3], sp[4], sp[5], sp[6], mt_s)
        gu_s, act_s, y_s = _grouped_ffn(xs, W(moe.w13_shared), W(moe.w2_shared), tables_s, Fh)
    if fused:
        ep.barrier()                                         # every return row has landed
    out = ext().moe_combine(w, sw, slot_of, yret, residual, ns, y_s)
    f = counts.float() / (N * k)
    aux = E * (f * (psum / N)).sum()
    gcounts = torch.from_numpy(table.sum(0)).to(h.device, non_blocking=True)
    moe.update_bias(gcounts, N * ep.world)
    saved = dict(h=h, idx=idx, w=w, sw=sw, probs=probs, f=f, slot_of=slot_of, plan=plan,
                 pull=(pull_b, pull_p), push=(push_b, push_p), cap=cap, xr=xr, gu_r=gu_r,
                 act_r=act_r, seg_r=seg_r, tables_r=tables_r, yret=yret, xs=xs, gu_s=gu_s,
                 act_s=act_s, y_s=y_s, tables_s=tables_s if ns else None)
    return out, aux, saved


def moe_ffn_backward_ep(dout: torch.Tensor, d_aux, moe, W, sv) -> torch.Tensor:
    """Backward of :func:`moe_ffn_forward_ep`: ``dy`` rows travel to the experts' owners
    (pull), the local experts' backward GEMMs run there, ``dx`` rows travel back (push)."""
    import torch.distributed as dist

    from ..parallel.expert import ep_move

    ep = moe.ep
    h = sv["h"]
    N, d = h.shape
    E, k, ns, Fh = moe.num_experts, moe.top_k, moe.num_shared_experts, moe.expert_dim
    El = ep.local_experts
    fused = ep.transport == "fused"
    plan, cap, rb = sv["plan"], sv["cap"], 2 * d
    if fused:
        dsb = ep.sym("dsend", cap * rb)
        dsend = dsb.tensor(cap * d, torch.bfloat16).view(cap, d)
    else:
        dsend = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
    res = ext().moe_combine_bwd(sv["w"], sv["sw"], sv["slot_of"], sv["yret"], dout, ns, sv["y_s"],
                                dsend, None)
    dw = res[1]
    dys = res[2] if ns else None
    dyr = torch.empty(max(plan.owner_rows, 1), d, device=h.device, dtype=torch.bfloat16)
    pull_b, pull_p = sv["pull"]
    if fused:
        ep.barrier()                                         # every dy row is written
        ep_move(pull_b, pull_p, plan.n_recv, rb, src_table=dsb.table, dst=dyr)
    else:
        recv = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
        dist.all_to_all_single(recv[:plan.n_recv], dsend[:N * k], plan.recv_splits, plan.send_splits,
                               group=ep.group)
        ep_move(pull_b, pull_p, plan.n_recv, rb, src=recv, dst=dyr)
    dxr = dyr
    if plan.owner_rows:
        ext().moe_zero_pad(sv["seg_r"][0], sv["seg_r"][1], dyr)
        dxr = _grouped_ffn_bwd(dyr, sv["xr"], sv["gu_r"], sv["act_r"], W(moe.w13), W(moe.w2),
                               moe.w13.grad.view(El * 2 * Fh, d), moe.w2.grad.view(El * d, Fh),
                               sv["tables_r"], Fh)
    push_b, push_p = sv["push"]
    if fused:
        drb = ep.sym("dret", cap * rb)
        ep_move(push_b, push_p, plan.n_recv, rb, src=dxr, dst_table=drb.table)
        dret = drb.tensor(cap * d, torch.bfloat16).view(cap, d)
    else:
        stage = torch.empty(max(plan.n_recv, 1), d, device=h.device, dtype=torch.bfloat16)
        ep_move(push_b, push_p, plan.n_recv, rb, src=dxr, dst=stage)
        dret = torch.empty(max(N * k, 1), d, device=h.device, dtype=torch.bfloat16)
        dist.all_to_all_single(dret[:N * k], stage[:plan.n_recv], plan.send_splits, plan.recv_splits,
                               group=ep.group)
    dxs = None
    if ns:
        dxs = _grouped_ffn_bwd(dys, sv["xs"], sv["gu_s"], sv["act_s"], W(moe.w13_shared),
                               W(moe.w2_shared), moe.w13_shared.grad.view(ns * 2 * Fh, d),
                               moe.w2_shared.grad.view(ns * d, Fh), sv["tables_s"], Fh)
    if fused:
        ep.barrier()                                         # every dx row has landed
    dh = ext().moe_unpermute(dret, sv["slot_of"], N, dxs, k)
    dlog = router_dlogits(sv["probs"], sv["idx"], sv["w"], sv["sw"], dw, d_aux, sv["f"],
                          E, k, ns, moe.e_pad)
    dlog = dlog.to(torch.bfloat16)
    gemm(dlog, h, moe.router_weight.grad, epi="f32_acc", a_t=True, b_t=True)
    gemm(dlog, W(moe.router_weight), dh, b_t=True, residual=dh)
    return dh
