"""Kernel micro-benchmarks (CUDA-event timing after warm-up, L2 flushed between runs).

``python -m drivedit_b200.ops.bench_kernels gemm`` times the tcgen05 GEMM at the DiT-B
training shapes (8 x 8192 tokens, d=768) next to ``torch.matmul`` (cuBLAS) and prints
one JSON line per shape with TFLOP/s.
"""
from __future__ import annotations

import argparse
import json

import torch

L2_FLUSH_BYTES = 256 << 20


def _timeit(fn, iters=20, warmup=5, flush=True):
    buf = torch.empty(L2_FLUSH_BYTES // 4, device="cuda", dtype=torch.float32)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            buf.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


GEMM_SHAPES = [
    # (name, M, N, K, a_t, b_t, epi)
    ("qkv_fwd", 65536, 2304, 768, False, False, "bf16"),
    ("w13_fwd_swiglu", 65536, 6144, 768, False, False, "swiglu"),
    ("w2_fwd", 65536, 768, 3072, False, False, "bf16"),
    ("w2_dgrad_dswiglu", 65536, 3072, 768, False, True, "dswiglu"),
    ("w13_dgrad", 65536, 768, 6144, False, True, "bf16"),
    ("w13_wgrad", 6144, 768, 65536, True, True, "f32_acc"),
    ("square_8192", 8192, 8192, 8192, False, False, "bf16"),
]


def bench_gemm(iters: int = 20, shapes=None):
    from .gemm import gemm

    for name, M, N, K, a_t, b_t, epi in GEMM_SHAPES:
        if shapes and name not in shapes:
            continue
        a = torch.randn(*((K, M) if a_t else (M, K)), device="cuda", dtype=torch.bfloat16)
        b = torch.randn(*((K, N) if b_t else (N, K)), device="cuda", dtype=torch.bfloat16)
        kw = {}
        if epi == "dswiglu":
            kw["residual"] = torch.randn(M, 2 * N, device="cuda", dtype=torch.bfloat16)
        out = None
        if epi == "f32_acc":
            out = torch.zeros(M, N, device="cuda", dtype=torch.float32)
        ms = _timeit(lambda: gemm(a, b, out, epi=epi, a_t=a_t, b_t=b_t, **kw), iters)
        A = a.t() if a_t else a
        B = b.t() if b_t else b
        ms_ref = _timeit(lambda: torch.matmul(A, B.t()), iters)
        flops = 2.0 * M * N * K
        print(json.dumps({
            "kernel": "gemm_tc", "shape": name, "M": M, "N": N, "K": K, "epi": epi,
            "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
            "cublas_ms": round(ms_ref, 4), "cublas_tflops": round(flops / ms_ref / 1e9, 1),
        }), flush=True)
        del a, b, out, kw


def bench_attn(iters: int = 10, B: int = 8, H: int = 12, T: int = 8192, tpf: int = 512,
               dbg: int = 0, trace: bool = False):
    """Frame-causal flash attention fwd and bwd at the DiT-B training shape."""
    import math

    from ._ext import ext

    d = H * 64
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.5).bfloat16()
    o = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device="cuda")
    do = torch.randn(B * T, d, device="cuda").bfloat16()
    delta = torch.empty(B * H * T, device="cuda")
    dq_acc = torch.zeros(B * T, d, device="cuda")
    dqkv = torch.empty(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
    sc = 1 / 8.0

    def fwd():
        ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, 1, tpf, 0, 0, sc,
                       None, None, None)

    def bwd():
        ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
        dq_acc.zero_()
        ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, dqkv, dqkv, 0, d, 2 * d, 0, 0, d,
                       2 * d, B, H, T, T, T, T, 1, tpf, 0, 0, sc, None, None, None, dbg)
        ext().attn_dq_finalize(dq_acc, dqkv, 0, H, None, T, 0)

    fwd()
    # visible (query, key) pairs under frame-causal masking
    frames = T // tpf
    pairs = B * H * tpf * tpf * frames * (frames + 1) / 2
    f_fwd = 4.0 * pairs * 64
    f_bwd = 10.0 * pairs * 64
    ms_f = _timeit(fwd, iters)
    ms_b = _timeit(bwd, iters)
    print(json.dumps({"kernel": "attn_fwd", "B": B, "H": H, "T": T, "tpf": tpf, "ms": round(ms_f, 3),
                      "tflops": round(f_fwd / ms_f / 1e9, 1)}), flush=True)
    print(json.dumps({"kernel": "attn_bwd", "B": B, "H": H, "T": T, "tpf": tpf, "ms": round(ms_b, 3),
                      "tflops": round(f_bwd / ms_b / 1e9, 1), "debug_flags": dbg}), flush=True)
    if trace:
        _attn_trace(fwd, qkv, o, do, lse, delta, dq_acc, dqkv, B, H, T, tpf, sc)


def bench_sla_attn(iters: int = 10, B: int = 8, H: int = 12, T: int = 8192, tpf: int = 512,
                   small: bool = False):
    """SLA block-sparse softmax attention (top 12.5 % of 64x64 blocks, frame-causal) at
    the DiT-B training shape: routing, sparse forward and sparse backward timed
    separately. Effective TFLOP/s count only the selected (query block, key block) pairs
    (4 * 64 * 64 * 64 flops per pair forward, 10x backward), so the figure shows how
    much of the work the kernels spend on selected pairs."""
    import math

    from ..layers.sla import SLAConfig
    from ._ext import ext
    from .attention_kernels import sla_plan_kernel

    if small:
        B = 2
    d = H * 64
    torch.manual_seed(0)
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.5).bfloat16()
    o = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device="cuda")
    do = torch.randn(B * T, d, device="cuda").bfloat16()
    delta = torch.empty(B * H * T, device="cuda")
    dq_acc = torch.zeros(B * T, d, device="cuda")
    dqkv = torch.empty(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
    cfg = SLAConfig(block_size=64, topk_frac=0.125, causal="frame", tokens_per_frame=tpf)
    sc = 1.0 / math.sqrt(64)
    plan = sla_plan_kernel(qkv, B, T, H, cfg, tpf, "frame", sel_bits=True)
    lists = (plan.pair_blocks, plan.pair_mask, plan.pair_count)
    tlists = (plan.kv_qtiles, plan.kv_qmask, plan.kv_count)
    # selected pairs: popcount of the 4-bit quadrant masks of the listed pairs
    counts = plan.pair_count.long()
    mask = plan.pair_mask.long()
    live = torch.arange(mask.shape[1], device="cuda")[None, :] < counts[:, None]
    bits = sum(((mask >> i) & 1) for i in range(4)) * live
    selected = float(bits.sum())
    computed = float(counts.sum()) * 4  # 128 x 128 tiles = 4 block pairs each
    computed_bwd = float(plan.kv_count.long().sum()) * 4  # 128-key x 128-query units

    def route():
        sla_plan_kernel(qkv, B, T, H, cfg, tpf, "frame")

    def fwd():
        ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, 1, tpf, 0, 0, sc,
                       *lists)

    def bwd():
        ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
        dq_acc.zero_()
        ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, dqkv, dqkv, 0, d, 2 * d, 0, 0, d,
                       2 * d, B, H, T, T, T, T, 1, tpf, 0, 0, sc, *tlists, 0)
        ext().attn_dq_finalize(dq_acc, dqkv, 0, H, None, T, 0)

    fwd()
    f_pair = 64.0 * 64 * 64
    ms_r, ms_f, ms_b = _timeit(route, iters), _timeit(fwd, iters), _timeit(bwd, iters)
    print(json.dumps({"kernel": "sla_route", "B": B, "H": H, "T": T, "ms": round(ms_r, 3)}), flush=True)
    for name, ms, mult, comp in (("sla_attn_fwd", ms_f, 4.0, computed),
                                 ("sla_attn_bwd", ms_b, 10.0, computed_bwd)):
        print(json.dumps({"kernel": name, "B": B, "H": H, "T": T, "ms": round(ms, 3),
                          "selected_pairs": int(selected), "computed_pairs": int(comp),
                          "tflops_selected": round(mult * f_pair * selected / ms / 1e9, 1),
                          "tflops_computed": round(mult * f_pair * comp / ms / 1e9, 1)}),
              flush=True)


def _attn_trace(fwd, qkv, o, do, lse, delta, dq_acc, dqkv, B, H, T, tpf, sc):
    """clock64 events of one heavy CTA per kernel (cycles from the CTA's first event):
    forward roles producer / MMA / softmax, backward producer / MMA / softmax / dQ."""
    from ._ext import ext

    d = H * 64
    buf = torch.zeros(3 * 8 * 64, dtype=torch.int64, device="cuda")
    ext().attn_fwd_set_trace(buf, 0)
    fwd()
    torch.cuda.synchronize()
    ext().attn_fwd_set_trace(None, 0)
    _print_trace("attn_fwd", buf.view(3, 8, 64).cpu(), ["producer", "mma", "softmax"])
    tb = torch.zeros(4 * 8 * 64, dtype=torch.int64, device="cuda")
    ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
    dq_acc.zero_()
    ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, dqkv, dqkv, 0, d, 2 * d, 0, 0, d,
                   2 * d, B, H, T, T, T, T, 1, tpf, 0, 0, sc, None, None, None, 0, trace=tb, trace_cta=0)
    torch.cuda.synchronize()
    _print_trace("attn_bwd", tb.view(4, 8, 64).cpu(), ["producer", "mma", "softmax", "dq"])


def _print_trace(name, t, roles):
    nz = t[t != 0]
    if nz.numel() == 0:
        print(json.dumps({"trace": name, "empty": True}), flush=True)
        return
    t0 = int(nz.min())
    out = {}
    for r, role in enumerate(roles):
        for ev in range(8):
            row = t[r, ev]
            if (row != 0).any():
                out[f"{role}.{ev}"] = [int(x) - t0 if int(x) else None for x in row[:24]]
    print(json.dumps({"trace": name, "cycles_from_first_event": out}), flush=True)


def bench_sla_linear(iters: int = 10, B: int = 4, H: int = 12, T: int = 8192):
    """The four per-block kernels of the SLA linear branch at the DiT-B shape (state and
    state gradients random; the batched GEMM between them is not timed here)."""
    from ._ext import ext

    d = H * 64
    nb = T // 64
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.5).bfloat16()
    kvz = torch.empty(B * H * nb * 4160, device="cuda", dtype=torch.bfloat16)
    state = torch.rand(B * H * nb, 4160, device="cuda") + 0.1
    o = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    den = torch.empty(B * H * T, device="cuda")
    do = torch.randn(B * T, d, device="cuda").bfloat16()
    dsz = torch.empty(B * H * nb * 4160, device="cuda", dtype=torch.bfloat16)
    dqkv = torch.zeros(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
    dkvz = torch.randn(B * H * nb, 4160, device="cuda") * 0.01
    runs = {
        "sla_kv_state": lambda: ext().sla_kv_state(qkv, kvz, B, T, H),
        "sla_lin_out": lambda: ext().sla_lin_out(qkv, state, o, den, B, T, H, 1e-6),
        "sla_lin_bwd_q": lambda: ext().sla_lin_bwd_q(qkv, state, o, do, den, dsz, dqkv, B, T, H),
        "sla_lin_bwd_kv": lambda: ext().sla_lin_bwd_kv(qkv, dkvz, dqkv, B, T, H),
    }
    for name, fn in runs.items():
        fn()
        ms = _timeit(fn, iters)
        print(json.dumps({"kernel": name, "B": B, "H": H, "T": T, "ms": round(ms, 4)}), flush=True)


def bench_norm(iters: int = 20, M: int = 65536, D: int = 768, tpf: int = 512):
    """AdaLN-RMSNorm forward and backward at the DiT-B shape (8 x 8192 tokens, d=768,
    512 tokens per frame), with achieved DRAM bandwidth over the bytes each must move."""
    from .fused import adaln_rmsnorm, adaln_rmsnorm_bwd

    G = M // tpf
    x = torch.randn(M, D, device="cuda").bfloat16()
    w = 1 + 0.1 * torch.randn(D, device="cuda")
    mod = 0.2 * torch.randn(G, 6 * D, device="cuda")
    dh = torch.randn(M, D, device="cuda").bfloat16()
    dres = torch.randn(M, D, device="cuda").bfloat16()
    dmod = torch.zeros_like(mod)
    dw = torch.zeros_like(w)
    h, r = adaln_rmsnorm(x, w, mod, 0, D, tpf)
    row = M * D * 2
    for name, fn, nbytes in (
            ("adaln_fwd", lambda: adaln_rmsnorm(x, w, mod, 0, D, tpf), 2 * row),
            ("adaln_bwd", lambda: adaln_rmsnorm_bwd(dh, x, r, w, mod, 0, D, tpf, dmod, dw, dres),
             4 * row)):
        ms = _timeit(fn, iters)
        print(json.dumps({"kernel": name, "M": M, "D": D, "ms": round(ms, 4),
                          "GB_s": round(nbytes / ms / 1e6, 1)}), flush=True)


def bench_conv3d(iters: int = 10):
    """VAE causal 3x3x3 convolutions at 8 frames of 256x512 RGB (encoder level 0,
    128 ch, and level 2, 512 ch at 65x129), stride-2 downsample, vs cuDNN."""
    import torch.nn.functional as F

    from .conv3d import causal_conv3d

    shapes = [("enc_l0_res", 1, 128, 128, 8, 256, 512, (3, 3, 3), (1, 1, 1)),
              ("enc_l2_res", 1, 512, 512, 2, 65, 129, (3, 3, 3), (1, 1, 1)),
              ("enc_down0", 1, 128, 128, 8, 256, 512, (4, 4, 4), (2, 2, 2))]
    for name, B, Cin, Cout, T, H, W, k, st in shapes:
        x = torch.randn(B, Cin, T, H, W, device="cuda").bfloat16()
        x = x.contiguous(memory_format=torch.channels_last_3d)
        w = torch.randn(Cout, Cin, *k, device="cuda") * 0.02
        b = torch.zeros(Cout, device="cuda")
        y = causal_conv3d(x, w, b, st)
        ms = _timeit(lambda: causal_conv3d(x, w, b, st), iters)
        wb = w.bfloat16().contiguous(memory_format=torch.channels_last_3d)
        xp = F.pad(x, (0, 0, 0, 0, k[0] - 1, 0))
        ms_ref = _timeit(lambda: F.conv3d(xp, wb, None, st, (0, k[1] // 2, k[2] // 2)), iters)
        flops = 2.0 * y.numel() * Cin * k[0] * k[1] * k[2]
        print(json.dumps({"kernel": "conv3d_tc", "shape": name, "ms": round(ms, 4),
                          "tflops": round(flops / ms / 1e9, 1), "cudnn_ms": round(ms_ref, 4),
                          "cudnn_tflops": round(flops / ms_ref / 1e9, 1)}), flush=True)


def bench_groupnorm(iters: int = 10, small: bool = False):
    """VAE GroupNorm(32) + SiLU forward and backward (channels-last) at the encoder's
    level-0 activation (8 frames x 128 ch x 256x512, 268 MB bf16), vs PyTorch's GroupNorm
    + SiLU. Roofline: the forward reads x once for statistics and once to normalise and
    writes y; the backward reads dy and x and writes dx."""
    import torch.nn.functional as F

    from .conv3d import group_norm_silu

    B, C, T, H, W = (1, 128, 2, 128, 256) if small else (1, 128, 8, 256, 512)
    x = torch.randn(B, C, T, H, W, device="cuda").bfloat16().contiguous(
        memory_format=torch.channels_last_3d).requires_grad_(True)
    w = torch.ones(C, device="cuda", requires_grad=True)
    b = torch.zeros(C, device="cuda", requires_grad=True)
    dy = torch.randn(B, C, T, H, W, device="cuda").bfloat16().contiguous(
        memory_format=torch.channels_last_3d)
    nbytes = x.numel() * 2
    y = group_norm_silu(x, 32, w, b)
    ms_f = _timeit(lambda: group_norm_silu(x, 32, w, b), iters)
    ms_b = _timeit(lambda: torch.autograd.grad(group_norm_silu(x, 32, w, b), (x,), dy), iters)
    wb, bb = w.detach().bfloat16(), b.detach().bfloat16()
    ms_rf = _timeit(lambda: F.silu(F.group_norm(x, 32, wb, bb)), iters)
    print(json.dumps({"kernel": "groupnorm_silu_fwd", "shape": [B, C, T, H, W], "ms": round(ms_f, 4),
                      "gbs": round(3 * nbytes / ms_f / 1e6, 1), "torch_ms": round(ms_rf, 4)}), flush=True)
    print(json.dumps({"kernel": "groupnorm_silu_fwd+bwd", "ms": round(ms_b, 4),
                      "gbs_bwd_only": round(6 * nbytes / max(ms_b - ms_f, 1e-6) / 1e6, 1)}), flush=True)
    del y


def bench_kv_attn(iters: int = 20, small: bool = False):
    """Rollout chunk attention over the rolling KV cache at the DiT-B rollout shape:
    a 4-frame chunk (2048 queries) against the 32-frame window plus the chunk
    (18432 keys), frame-causal with absolute offsets, 12 heads, batch 1 and 16. Roofline:
    the K/V window bytes read (the FLOPs are small at batch 1)."""
    import math

    from ._ext import ext

    H, tpf = 12, 512
    d = H * 64
    Tq, S = 4 * tpf, 36 * tpf
    for B in ((1,) if small else (1, 16)):
        q = (torch.randn(B * Tq, d, device="cuda") * 0.5).bfloat16()
        kv = (torch.randn(B * S, 2 * d, device="cuda") * 0.5).bfloat16()
        o = torch.empty(B * Tq, d, device="cuda", dtype=torch.bfloat16)
        pos = S - Tq  # the chunk is the newest 4 frames of the window

        def fwd():
            ext().attn_fwd(q, kv, kv, o, None, 0, 0, d, 0, B, H, Tq, S, Tq, S, 1, tpf, pos, 0,
                           1.0 / math.sqrt(64), None, None, None)

        fwd()
        ms = _timeit(fwd, iters)
        kv_bytes = 2 * B * S * d * 2
        flops = 4.0 * B * H * Tq * S * 64
        print(json.dumps({"kernel": "attn_fwd_kvcache", "B": B, "Tq": Tq, "S": S, "ms": round(ms, 4),
                          "tflops": round(flops / ms / 1e9, 1),
                          "kv_gbs": round(kv_bytes / ms / 1e6, 1)}), flush=True)


def bench_moe_gemm(iters: int = 10, N: int = 32768, d: int = 1024, E: int = 64, k: int = 6,
                   F: int = 512, ns: int = 2, small: bool = False):
    """Grouped (MoE) SwiGLU and down GEMMs of one MoE-DiT-L layer on one GPU (random
    router, skewed counts), vs one cuBLAS matmul per expert over the same rows."""
    from ..layers.mlp import pack_swiglu
    from ._ext import ext
    from .gemm import EPI

    if small:
        N = 8192
    torch.manual_seed(0)
    h = (torch.randn(N, d, device="cuda") * 0.5).bfloat16()
    logits = torch.randn(N, E + ns, device="cuda") * 2.0  # routed, then shared-gate logits
    idx, w, sw, probs, counts, psum = ext().moe_route(logits, torch.zeros(E, device="cuda"), E, k, ns, True)
    mt = (N * k + 127) // 128 + E + ns * ((N + 127) // 128)
    plan = ext().moe_plan(counts, E, ns, N, mt)
    rows = mt * 128
    xp = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    ext().moe_dispatch(h, idx, plan[0], plan[1], plan[7], xp, E, ns)
    Ep = E + ns
    w13 = (torch.randn(Ep, 2 * F, d, device="cuda") * 0.02).bfloat16()
    w2 = (torch.randn(Ep, d, F, device="cuda") * 0.02).bfloat16()
    gu = torch.empty(rows, 2 * F, device="cuda", dtype=torch.bfloat16)
    act = torch.empty(rows, F, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    tables = (plan[2], plan[3], plan[4], plan[5], plan[6], mt)

    def ours():
        ext().gemm_grouped(xp, w13, gu, EPI["swiglu"], False, 1, *tables, None, act)
        ext().gemm_grouped(act, w2, y, EPI["bf16"], False, 1, *tables, None, None)

    seg = plan[0].cpu().tolist()
    cnt = plan[1].cpu().tolist()

    def per_expert():
        for e in range(Ep):
            if cnt[e]:
                xs = xp[seg[e]:seg[e] + cnt[e]]
                g = xs @ w13[e].t()
                a = torch.nn.functional.silu(g[:, :F]) * g[:, F:]
                y[seg[e]:seg[e] + cnt[e]] = a @ w2[e].t()

    ours()
    ms = _timeit(ours, iters)
    ms_ref = _timeit(per_expert, max(3, iters // 2))
    routed_rows = float(sum(cnt))
    flops = 2.0 * routed_rows * d * (2 * F) + 2.0 * routed_rows * F * d
    print(json.dumps({"kernel": "gemm_grouped (swiglu + down)", "tokens": N, "experts": E, "top_k": k,
                      "shared": ns, "rows": int(routed_rows), "max_rows_per_expert": int(max(cnt[:E])),
                      "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                      "cublas_loop_ms": round(ms_ref, 4),
                      "cublas_loop_tflops": round(flops / ms_ref / 1e9, 1)}), flush=True)


def bench_ep(iters: int = 5, d: int = 1024, E: int = 64, k: int = 6, F: int = 512, ns: int = 2,
             N: int = 32768, transport: str = "fused"):
    """Expert-parallel MoE layer on all ranks of a torchrun job (one per GPU): device time
    of each stage of the forward and backward (max over ranks), and the NVLink bytes of
    the row movement next to the 770 GB/s per-direction peer-copy reference.
    Defaults: the MoE-DiT-L layer (d 1024, 64 experts of width 512, top-6, 2 shared) on
    4 x 8192 tokens per rank."""
    import datetime
    import os

    import torch.distributed as dist

    from . import moe as moe_ops
    from ..layers.moe import MoEFFN
    from ..parallel.expert import ExpertParallel
    from ..parallel.flat import FlatParamGroup

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    torch.manual_seed(0)
    moe = MoEFFN(d, E, k, F, ns).cuda()
    ep = ExpertParallel(num_experts=E, transport=transport, device="cuda")
    moe.shard_experts(ep)
    main_g = FlatParamGroup([(n, p) for n, p in moe.named_parameters() if n not in ("w13", "w2")])
    main_g.linked.append(FlatParamGroup([("w13", moe.w13), ("w2", moe.w2)]))
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    h = torch.randn(N, d, device="cuda", generator=g).to(torch.bfloat16)
    r = torch.randn(N, d, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(N, d, device="cuda", generator=g).to(torch.bfloat16)
    one = torch.ones((), device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")

    def step():
        out, aux, sv = moe_ops.moe_ffn_forward_ep(h, r, moe, main_g.compute_view)
        moe_ops.moe_ffn_backward_ep(dout, one, moe, main_g.compute_view, sv)
        return sv

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    stages = {}
    totals = []
    for _ in range(iters):
        flush.zero_()
        dist.barrier()
        moe_ops.EP_TRACE = []
        s0 = torch.cuda.Event(enable_timing=True)
        s0.record()
        sv = step()
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.cuda.synchronize()
        tr, moe_ops.EP_TRACE = moe_ops.EP_TRACE, None
        totals.append(s0.elapsed_time(e0))
        for (a, ea), (b, eb) in zip(tr[:-1], tr[1:]):
            if a.split(".")[0] == b.split(".")[0]:
                stages.setdefault(b, []).append(ea.elapsed_time(eb))
    # rows peers pushed to this rank in the last forward (NVLink inbound); as many go back
    meta = sv.get("owner")[9] if transport == "fused" else None
    remote_rows = 0
    if meta is not None:
        nu = int(sv["owner"][11].item())
        remote_rows = int((meta[:nu, 0] != rank).sum())
    med = {kk: sorted(v)[len(v) // 2] for kk, v in stages.items()}
    t = torch.tensor([sorted(totals)[len(totals) // 2]] + [med[kk] for kk in sorted(med)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    rr = torch.tensor([float(remote_rows)], device="cuda")
    dist.all_reduce(rr, op=dist.ReduceOp.MAX)
    if rank == 0:
        keys = sorted(med)
        res = {"what": "ep_layer", "transport": transport, "world": W, "N_per_rank": N, "d": d, "experts": E,
               "top_k": k, "ms_fwd_bwd": round(float(t[0]), 3),
               "stage_ms_max_over_ranks": {kk: round(float(v), 3) for kk, v in zip(keys, t[1:].tolist())},
               "remote_rows_per_direction_max": int(rr.item())}
        if transport == "fused":
            mb = rr.item() * d * 2 / 1e6
            res["nvlink_mb_per_phase"] = round(mb, 1)
            # P2P-store phases: row pushes to the owners, partial sums back to the sources
            for st in ("fwd.push", "fwd.scatter", "bwd.push", "bwd.scatter"):
                ms = res["stage_ms_max_over_ranks"].get(st)
                if ms:
                    gbs = mb / ms
                    res[f"{st}_GBps"] = round(gbs, 1)
                    res[f"{st}_frac_of_770"] = round(gbs / 770.0, 3)
        print(json.dumps(res), flush=True)
    ep.close()
    dist.barrier()


def bench_optim(iters: int = 10, numel: int = 130_000_000, transport: str = "fused"):
    """Sharded optimizer step on every rank of a torchrun job (reduce-scatter of the fp32
    gradients + global-norm clip + AdamW on the shard + all-gather of fp32 and bf16
    weights) for a flat buffer of ``numel`` parameters (DiT-B has ~130M); device time max
    over ranks and the bytes that cross NVLink per rank next to the 770 GB/s reference."""
    import datetime
    import os

    import torch.distributed as dist
    import torch.nn as nn

    from ..parallel.sharded import ShardedDataParallel

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    rank, W = dist.get_rank(), dist.get_world_size()
    rows = numel // 4096
    net = nn.Module()
    net.w = nn.Parameter(torch.randn(rows, 4096, device="cuda") * 0.02)
    eng = ShardedDataParallel(net, transport=transport, lr=1e-4, weight_decay=0.01, grad_clip=1.0)
    eng.flat.grad.normal_()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        dist.barrier()
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        eng.step()
        e0.record()
        torch.cuda.synchronize()
        ts.append(s0.elapsed_time(e0))
    t = torch.tensor([sorted(ts)[len(ts) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    n = eng.flat.numel
    # per rank: read (W-1)/W of the fp32 gradient from peers, write (W-1)/W of fp32 master
    # + bf16 compute into peers
    mb_in = n * 4 * (W - 1) / W / 1e6
    mb_out = n * 6 * (W - 1) / W / 1e6
    if rank == 0:
        ms = float(t.item())
        print(json.dumps({"what": "sharded_optimizer_step", "transport": transport, "world": W, "numel": n,
                          "ms": round(ms, 3), "nvlink_in_mb": round(mb_in, 1), "nvlink_out_mb": round(mb_out, 1),
                          "roofline_ms_at_770": round(max(mb_in, mb_out) / 770.0, 3),
                          "frac_of_roofline": round(max(mb_in, mb_out) / 770.0 / ms, 3)}), flush=True)
    eng.close()
    dist.barrier()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("what", nargs="*", default=["gemm"], help="gemm attn sla_attn sla norm conv3d ep optim")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--small", action="store_true", help="small attention case (for ncu)")
    p.add_argument("--B", type=int, default=8, help="attention batch")
    p.add_argument("--trace", action="store_true", help="attention: clock64 trace of one CTA per kernel")
    p.add_argument("--shape", nargs="*", help="gemm shapes to run (names in GEMM_SHAPES)")
    p.add_argument("--transport", default="fused", help="ep: fused | nccl")
    args = p.parse_args()
    for w in args.what:
        if w == "attn" and args.small:
            bench_attn(args.iters, B=1, H=2, T=8192)
        elif w == "attn":
            bench_attn(args.iters, B=args.B, trace=args.trace)
        elif w == "attn_nodq":  # timing experiment: backward without the dQ reductions
            bench_attn(args.iters, dbg=1)
        elif w == "sla":
            bench_sla_linear(args.iters, B=args.B if args.B != 8 else 4)
        elif w == "gemm":
            bench_gemm(args.iters, args.shape)
        elif w == "ep":
            bench_ep(args.iters, transport=args.transport)
        elif w == "optim":
            bench_optim(args.iters, transport=args.transport)
        elif w in ("groupnorm", "kv_attn", "moe_gemm", "sla_attn"):
            globals()[f"bench_{w}"](args.iters, small=args.small)
        else:
            globals()[f"bench_{w}"](args.iters)
    from ._ext import check_device_status

    check_device_status()


if __name__ == "__main__":
    main()
