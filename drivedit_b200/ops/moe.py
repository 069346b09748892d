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
