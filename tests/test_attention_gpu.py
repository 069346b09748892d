"""tcgen05 flash attention (fwd + bwd, dense masks and SLA lists) vs PyTorch fp32."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _mask(T, S, causal, tpf, q_off=0, kv_off=0, device="cuda"):
    qa = torch.arange(T, device=device)[:, None] + q_off
    ka = torch.arange(S, device=device)[None, :] + kv_off
    if causal == "frame":
        return (ka // tpf) <= (qa // tpf)
    if causal == "token":
        return ka <= qa
    return torch.ones(T, S, dtype=torch.bool, device=device)


def _ref(q, k, v, mask):
    s = torch.einsum("bthd,bshd->bhts", q.float(), k.float()) / 8.0
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse[..., None]).nan_to_num(0.0)
    return torch.einsum("bhts,bshd->bthd", p, v.float()), lse


@pytest.mark.parametrize("causal,T,tpf", [("frame", 1024, 256), ("token", 512, 1), ("none", 384, 1),
                                          ("frame", 256, 64)])
def test_flash_fwd_bwd_dense(causal, T, tpf):
    from drivedit_b200.ops._ext import ext
    from drivedit_b200.ops.attention_kernels import CAUSAL
    B, H, D = 2, 3, 64
    d = H * D
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.7).bfloat16()
    o = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device="cuda")
    ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, CAUSAL[causal], tpf,
                   0, 0, 1 / 8.0, None, None, None)
    v5 = qkv.view(B, T, 3, H, D)
    q, k, v = [v5[:, :, i].float().requires_grad_(True) for i in range(3)]
    mask = _mask(T, T, causal, tpf)
    ro, rlse = _ref(q, k, v, mask)
    assert _rel(o.view(B, T, H, D), ro) < 2e-2
    assert ((lse.view(B, H, T) * math.log(2) - rlse).abs().max() < 2e-2)
    # backward
    do = torch.randn(B * T, d, device="cuda").bfloat16()
    ro.backward(do.view(B, T, H, D).float())
    delta = torch.empty(B * H * T, device="cuda")
    ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
    dq_acc = torch.zeros(B * T, d, device="cuda")
    dqkv = torch.zeros(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
    ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, dqkv, dqkv, 0, d, 2 * d, 0, 0, d,
                   2 * d, B, H, T, T, T, T, CAUSAL[causal], tpf, 0, 0, 1 / 8.0, None, None, None, 0)
    ext().attn_dq_finalize(dq_acc, dqkv, 0, H, None, T, 0)
    g = dqkv.view(B, T, 3, H, D)
    assert _rel(g[:, :, 0], q.grad) < 3e-2
    assert _rel(g[:, :, 1], k.grad) < 3e-2
    assert _rel(g[:, :, 2], v.grad) < 3e-2


def test_flash_kv_cache_offsets():
    """Queries = the last 2 frames (absolute frames 6-7) over a cache holding frames 2-7."""
    from drivedit_b200.ops.attention_kernels import flash_attention
    B, H, D, tpf = 1, 2, 64, 128
    q = torch.randn(B, 2 * tpf, H, D, device="cuda").bfloat16()
    k = torch.randn(B, 6 * tpf, H, D, device="cuda").bfloat16()
    v = torch.randn(B, 6 * tpf, H, D, device="cuda").bfloat16()
    o, lse = flash_attention(q, k, v, "frame", tpf, q_pos_offset=6 * tpf, kv_pos_offset=2 * tpf)
    mask = _mask(2 * tpf, 6 * tpf, "frame", tpf, 6 * tpf, 2 * tpf)
    ro, _ = _ref(q, k, v, mask)
    assert _rel(o, ro) < 2e-2


@pytest.mark.parametrize("splits", [1, 2, 3, 0])
def test_flash_kv_cache_split_kv(splits):
    """Rollout-shaped KV-cache attention (a 4-frame chunk over a longer window, few
    heads) with the key range split over 1, 2 or 3 CTAs per query tile (0: the launch's
    own choice) and merged by log-sum-exp: output and lse match the fp32 reference."""
    from drivedit_b200.ops._ext import ext
    from drivedit_b200.ops.attention_kernels import flash_attention
    B, H, D, tpf = 1, 2, 64, 256
    Tq, S = 4 * tpf, 12 * tpf          # chunk = the newest 4 of 12 frames
    q = torch.randn(B, Tq, H, D, device="cuda").bfloat16()
    k = torch.randn(B, S, H, D, device="cuda").bfloat16()
    v = torch.randn(B, S, H, D, device="cuda").bfloat16()
    prev = ext().attn_fwd_set_kv_splits(splits)
    try:
        o, lse = flash_attention(q, k, v, "frame", tpf, q_pos_offset=S - Tq, kv_pos_offset=0)
    finally:
        ext().attn_fwd_set_kv_splits(prev)
    mask = _mask(Tq, S, "frame", tpf, S - Tq, 0)
    ro, rlse = _ref(q, k, v, mask)
    assert _rel(o, ro) < 2e-2
    # the kernels' lse is in the log2 domain of the scaled scores
    assert (lse.float() - rlse * 1.4426950408889634).abs().max().item() < 2e-2


def test_sla_sparse_fwd_bwd_matches_masked_reference():
    from drivedit_b200.config import SLAParams
    from drivedit_b200.layers.sla import expand_block_mask
    from drivedit_b200.ops._ext import ext
    from drivedit_b200.ops.attention_kernels import sla_plan
    B, H, D, T, tpf = 2, 2, 64, 1024, 256
    d = H * D
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.7).bfloat16()
    v5 = qkv.view(B, T, 3, H, D)
    plan = sla_plan(v5[:, :, 0], v5[:, :, 1], B, T, H, SLAParams(64, 0.25, True), tpf, "frame")
    o = torch.empty(B * T, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device="cuda")
    ext().attn_fwd(qkv, qkv, qkv, o, lse, 0, d, 2 * d, 0, B, H, T, T, T, T, 1, tpf, 0, 0, 1 / 8.0,
                   plan.pair_blocks, plan.pair_mask, plan.pair_count)
    q, k, v = [v5[:, :, i].float().requires_grad_(True) for i in range(3)]
    mask = expand_block_mask(plan.sel, 64)
    ro, _ = _ref(q, k, v, mask)
    assert _rel(o.view(B, T, H, D), ro) < 2e-2
    do = torch.randn(B * T, d, device="cuda").bfloat16()
    ro.backward(do.view(B, T, H, D).float())
    delta = torch.empty(B * H * T, device="cuda")
    ext().attn_delta(o, do, delta, 0, 0, B, H, T, T)
    dq_acc = torch.zeros(B * T, d, device="cuda")
    dqkv = torch.zeros(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
    ext().attn_bwd(qkv, qkv, qkv, o, do, lse, delta, dq_acc, dqkv, dqkv, 0, d, 2 * d, 0, 0, d, 2 * d,
                   B, H, T, T, T, T, 1, tpf, 0, 0, 1 / 8.0, plan.kv_qtiles, plan.kv_qmask,
                   plan.kv_count, 0)
    ext().attn_dq_finalize(dq_acc, dqkv, 0, H, None, T, 0)
    g = dqkv.view(B, T, 3, H, D)
    assert _rel(g[:, :, 0], q.grad) < 3e-2
    assert _rel(g[:, :, 1], k.grad) < 3e-2
    assert _rel(g[:, :, 2], v.grad) < 3e-2


def test_attention_status_clean():
    from drivedit_b200.ops._ext import device_status
    torch.cuda.synchronize()
    assert device_status() == 0
