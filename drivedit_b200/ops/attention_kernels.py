"""Launch wrappers for the tcgen05 attention kernels (``csrc/attn``) and the SLA plan.

Dense modes call the flash kernels directly on the ``[M, 3d]`` qkv buffer (no
transposes: q, k, v of head h sit at columns ``64h``, ``d + 64h``, ``2d + 64h``).

SLA (``attn_mode == "sla"``):
  1. routing (:func:`sla_plan`): mean-pooled q/k per 64-token block, block scores,
     frame-causal validity, top-k selection with the diagonal forced; then the
     forward pair lists (per 128-query tile, the union of its two query blocks'
     selections paired two 64-key blocks at a time, with 4-bit half masks) and the
     backward transpose lists (per 128-key tile, the query blocks that selected it,
     paired two at a time into 128-query units);
  2. block-sparse softmax: the same forward/backward kernels in list mode;
  3. linear branch over the allowed-but-unselected blocks (elu+1 feature map),
     computed as block KV states combined by the (valid & ~selected) block matrix.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from ..layers.sla import SLAConfig, block_valid_mask, n_selected, sla_linear_reference
from ._ext import ext

CAUSAL = {"none": 0, "frame": 1, "token": 2}


class SLAPlan:
    def __init__(self, sel, valid, pair_blocks, pair_mask, pair_count, kv_qtiles, kv_qmask,
                 kv_count):
        self.sel, self.valid = sel, valid
        self.pair_blocks, self.pair_mask, self.pair_count = pair_blocks, pair_mask, pair_count
        self.kv_qtiles, self.kv_qmask, self.kv_count = kv_qtiles, kv_qmask, kv_count


def sla_route_blocks(q: torch.Tensor, k: torch.Tensor, B: int, T: int, H: int, bs: int,
                     frac: float, tpf: Optional[int], causal_token: bool, always_diag: bool):
    """``q``/``k`` are ``[B, T, H, 64]`` views; returns (sel [B,H,nb,nb], valid [nb,nb])."""
    nb = T // bs
    qm = q.unflatten(1, (nb, bs)).float().mean(2)         # [B, nb, H, D]
    km = k.unflatten(1, (nb, bs)).float().mean(2)
    score = torch.einsum("bqhd,bkhd->bhqk", qm, km) / math.sqrt(q.shape[-1])
    valid = block_valid_mask(nb, nb, bs, tpf, causal_token, q.device)
    score = score.masked_fill(~valid, float("-inf"))
    if always_diag:
        idx = torch.arange(nb, device=q.device)
        score[:, :, idx, idx] = float("inf")
    kk = min(n_selected(nb, frac), nb)
    top = score.topk(kk, dim=-1).indices
    sel = torch.zeros(score.shape, dtype=torch.bool, device=q.device).scatter_(-1, top, True)
    return sel & valid, valid, kk


def sla_plan(q, k, B, T, H, cfg, tpf: Optional[int], causal: str) -> SLAPlan:
    bs = cfg.block_size
    assert bs == 64, "the sparse kernels pair 64-key blocks"
    assert T % 128 == 0, "SLA kernels need sequence lengths that are multiples of 128"
    sel, valid, kk = sla_route_blocks(q, k, B, T, H, bs, cfg.topk_frac,
                                      tpf if causal == "frame" else None, causal == "token",
                                      cfg.always_diag)
    nb = T // bs
    nt = nb // 2
    dev = q.device
    ar = torch.arange(nb, device=dev)
    # ---- forward lists: per query tile, union of its two query blocks' selections
    lo, hi = sel[:, :, 0::2], sel[:, :, 1::2]                       # [B,H,nt,nb]
    union = lo | hi
    order = torch.argsort(torch.where(union, ar, ar + nb), dim=-1)  # selected first, ascending
    cnt = union.sum(-1)                                             # [B,H,nt]
    max_pairs = max(1, min(nb, 2 * kk) // 2 + (min(nb, 2 * kk) % 2))
    o = order[..., : 2 * max_pairs]
    if o.shape[-1] < 2 * max_pairs:
        o = torch.cat([o, o[..., :1].expand(*o.shape[:-1], 2 * max_pairs - o.shape[-1])], -1)
    b0, b1 = o[..., 0::2], o[..., 1::2]
    p = torch.arange(max_pairs, device=dev)
    v0 = (2 * p) < cnt[..., None]
    v1 = (2 * p + 1) < cnt[..., None]
    b1 = torch.where(v1, b1, b0)
    g = lambda m, bb: torch.gather(m, -1, bb)
    bits = ((g(lo, b0) & v0).to(torch.uint8)
            | ((g(lo, b1) & v1).to(torch.uint8) << 1)
            | ((g(hi, b0) & v0).to(torch.uint8) << 2)
            | ((g(hi, b1) & v1).to(torch.uint8) << 3))
    pair_blocks = (b0 | (b1 << 16)).to(torch.int32).reshape(B * H * nt, max_pairs).contiguous()
    pair_mask = bits.reshape(B * H * nt, max_pairs).contiguous()
    pair_count = ((cnt + 1) // 2).to(torch.int32).reshape(-1).contiguous()
    # ---- backward lists: per key tile (blocks 2t, 2t+1), the query blocks that selected
    # either key block, ascending, paired two at a time (qa | qb << 16; an odd last
    # block is paired with itself and its second half masked off)
    sk = sel.view(B, H, nb, nt, 2)                                  # [B,H,q,kt,khalf]
    kb = (sk[..., 0].to(torch.uint8) | (sk[..., 1].to(torch.uint8) << 1)).transpose(-1, -2)
    any_t = kb != 0                                                 # [B,H,kt,q]
    order_t = torch.argsort(torch.where(any_t, ar, ar + nb), dim=-1)
    cnt_t = any_t.sum(-1)                                           # [B,H,kt]
    qa, qb = order_t[..., 0::2], order_t[..., 1::2]                 # [B,H,kt,nt]
    pt = torch.arange(nt, device=dev)
    va = (2 * pt) < cnt_t[..., None]
    vb = (2 * pt + 1) < cnt_t[..., None]
    qb = torch.where(vb, qb, qa)
    ma = torch.where(va, torch.gather(kb, -1, qa), torch.zeros_like(qa, dtype=torch.uint8))
    mb = torch.where(vb, torch.gather(kb, -1, qb), torch.zeros_like(qb, dtype=torch.uint8))
    kv_count = ((cnt_t + 1) // 2).to(torch.int32).reshape(-1).contiguous()
    kv_qtiles = (qa | (qb << 16)).to(torch.int32).reshape(B * H * nt, nt).contiguous()
    kv_qmask = (ma | (mb << 2)).to(torch.uint8).reshape(B * H * nt, nt).contiguous()
    return SLAPlan(sel, valid, pair_blocks, pair_mask, pair_count, kv_qtiles, kv_qmask, kv_count)


class SLAKernelPlan:
    """Routing outputs of the ``sla_route`` kernel plus the linear-branch state."""

    def __init__(self, wlin, pair_blocks, pair_mask, pair_count, kv_qtiles, kv_qmask, kv_count):
        self.wlin = wlin
        self.pair_blocks, self.pair_mask, self.pair_count = pair_blocks, pair_mask, pair_count
        self.kv_qtiles, self.kv_qmask, self.kv_count = kv_qtiles, kv_qmask, kv_count
        self.state = None
        self.den = None


def sla_plan_kernel(qkv: torch.Tensor, B: int, T: int, H: int, cfg, tpf: int, causal: str,
                    sel_bits: bool = False) -> SLAKernelPlan:
    """Routing on the device: block means, scores, top-k, lists (``csrc/attn/sla.cu``)."""
    assert cfg.block_size == 64 and T % 128 == 0
    nb = T // 64
    nt = nb // 2
    dev = qkv.device
    qm = torch.empty(B * H * T, device=dev, dtype=torch.float32)
    km = torch.empty(B * H * T, device=dev, dtype=torch.float32)
    ext().sla_pool(qkv, qm, km, B, T, H)
    kk = min(n_selected(nb, cfg.topk_frac), nb)
    max_pairs = max(1, kk)
    BH = B * H
    wlin = torch.empty(BH, nb, nb, device=dev, dtype=torch.bfloat16)
    pb = torch.empty(BH * nt, max_pairs, device=dev, dtype=torch.int32)
    pm = torch.empty(BH * nt, max_pairs, device=dev, dtype=torch.uint8)
    pc = torch.empty(BH * nt, device=dev, dtype=torch.int32)
    kq = torch.empty(BH * nt, nt, device=dev, dtype=torch.int32)
    km_ = torch.empty(BH * nt, nt, device=dev, dtype=torch.uint8)
    kc = torch.empty(BH * nt, device=dev, dtype=torch.int32)
    code = {"none": 0, "frame": 1, "token": 2}[causal]
    bpf = max(1, tpf // 64) if causal == "frame" else 1
    sb = torch.empty(BH * nb * ((nb + 31) // 32), device=dev, dtype=torch.int32) if sel_bits else None
    ext().sla_route(qm, km, BH, nb, kk, code, bpf, bool(cfg.always_diag), wlin, pb, pm, pc, kq,
                    km_, kc, sb)
    plan = SLAKernelPlan(wlin, pb, pm, pc, kq, km_, kc)
    plan.sel_bits = sb
    return plan


def sla_linear_fwd_kernel(qkv, plan: SLAKernelPlan, B, T, H, eps=1e-6):
    nb = T // 64
    d = H * 64
    dev = qkv.device
    kvz = torch.empty(B * H, nb, 4160, device=dev, dtype=torch.bfloat16)
    ext().sla_kv_state(qkv, kvz, B, T, H)
    state = torch.empty(B * H * nb, 4160, device=dev, dtype=torch.float32)
    ext().gemm_batched(plan.wlin, kvz, state, 1, False, True)
    o_lin = torch.empty(B * T, d, device=dev, dtype=torch.bfloat16)
    den = torch.empty(B * H * T, device=dev, dtype=torch.float32)
    ext().sla_lin_out(qkv, state, o_lin, den, B, T, H, eps)
    plan.state, plan.den = state, den
    return o_lin


def sla_linear_bwd_kernel(qkv, o_lin, do_lin, plan: SLAKernelPlan, dqkv, B, T, H):
    nb = T // 64
    dev = qkv.device
    dsz = torch.empty(B * H, nb, 4160, device=dev, dtype=torch.bfloat16)
    ext().sla_lin_bwd_q(qkv, plan.state, o_lin, do_lin, plan.den, dsz, dqkv, B, T, H)
    dkvz = torch.empty(B * H * nb, 4160, device=dev, dtype=torch.float32)
    ext().gemm_batched(plan.wlin, dsz, dkvz, 1, True, True)
    ext().sla_lin_bwd_kv(qkv, dkvz, dqkv, B, T, H)


def _heads(qkv, bc):
    B, T, H = bc.B, bc.T, bc.H
    v = qkv.view(B, T, 3, H, 64)
    return v[:, :, 0], v[:, :, 1], v[:, :, 2]


def attention_fwd_kernel(qkv: torch.Tensor, bc):
    B, T, H, d = bc.B, bc.T, bc.H, bc.d
    assert bc.Dh == 64, "the attention kernels are written for d_head = 64"
    M = qkv.shape[0]
    o = torch.empty(M, d, device=qkv.device, dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device=qkv.device, dtype=torch.float32)
    scale = 1.0 / math.sqrt(bc.Dh)
    causal = CAUSAL[bc.causal]
    plan = None
    o_lin = None
    lists = (None, None, None)
    if bc.attn_mode == "sla":
        plan = sla_plan_kernel(qkv, B, T, H, bc.sla_cfg, bc.tpf, bc.causal)
        lists = (plan.pair_blocks, plan.pair_mask, plan.pair_count)
        o_lin = sla_linear_fwd_kernel(qkv, plan, B, T, H)
        plan.o_lin = o_lin
    ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, causal, bc.tpf,
                   0, 0, scale, *lists)
    return o, o_lin, lse, plan


def attention_bwd_kernel(qkv, o, lse, do, do_lin, plan, bc):
    B, T, H, d = bc.B, bc.T, bc.H, bc.d
    M = qkv.shape[0]
    dev = qkv.device
    delta = torch.empty(B * H * T, device=dev, dtype=torch.float32)
    ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
    dq_acc = torch.zeros(M, d, device=dev, dtype=torch.float32)
    dqkv = torch.empty(M, 3 * d, device=dev, dtype=torch.bfloat16)
    lists = (None, None, None)
    if plan is not None:
        lists = (plan.kv_qtiles, plan.kv_qmask, plan.kv_count)
    ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, dqkv, dqkv, 0, d, 2 * d, 0, 0, d,
                   2 * d, B, H, T, T, T, T, CAUSAL[bc.causal], bc.tpf, 0, 0,
                   1.0 / math.sqrt(bc.Dh), *lists, 0)
    ext().attn_dq_finalize(dq_acc, dqkv, 0, H, None, T, 0)
    if plan is not None and do_lin is not None:
        sla_linear_bwd_kernel(qkv, plan.o_lin, do_lin, plan, dqkv, B, T, H)
    return dqkv


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: str = "none",
                    tokens_per_frame: int = 1, q_pos_offset: int = 0, kv_pos_offset: int = 0,
                    scale: Optional[float] = None):
    """Forward-only flash attention on ``[B, T, H, 64]`` bf16 tensors (any strides whose
    last two dims are contiguous ``H x 64``); returns ``(o [B, T, H, 64], lse [B, H, T])``."""
    B, T, H, D = q.shape
    S = k.shape[1]
    assert D == 64
    q2 = q.reshape(B * T, H * D) if q.is_contiguous() else q.contiguous().reshape(B * T, H * D)
    k2 = k.reshape(B * S, H * D) if k.is_contiguous() else k.contiguous().reshape(B * S, H * D)
    v2 = v.reshape(B * S, H * D) if v.is_contiguous() else v.contiguous().reshape(B * S, H * D)
    o = torch.empty(B * T, H * D, device=q.device, dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device=q.device, dtype=torch.float32)
    ext().attn_fwd(q2, k2, v2, o, lse, 0, 0, 0, 0, B, H, T, S, T, S, CAUSAL[causal],
                   tokens_per_frame, q_pos_offset, kv_pos_offset,
                   scale if scale is not None else 1.0 / math.sqrt(D), None, None, None)
    return o.view(B, T, H, D), lse.view(B, H, T)


def packed_self_attention(qkv: torch.Tensor, B: int, T: int, H: int, causal: str = "none",
                          tokens_per_frame: int = 1, scale: Optional[float] = None) -> torch.Tensor:
    """Forward-only attention over a packed ``qkv [B*T, 3*H*64]`` bf16 projection (q, k, v
    column blocks, heads contiguous within each); any ``T`` (the last tile is masked).
    Returns ``o [B*T, H*64]``."""
    d = H * 64
    assert qkv.shape == (B * T, 3 * d) and qkv.is_contiguous()
    o = torch.empty(B * T, d, device=qkv.device, dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device=qkv.device, dtype=torch.float32)
    ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, CAUSAL[causal],
                   tokens_per_frame, 0, 0, scale if scale is not None else 0.125, None, None, None)
    return o
