"""SLA routing and linear-branch kernels vs the PyTorch fp32 oracle."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _sel_from_bits(bits, B, H, nb):
    words = (nb + 31) // 32
    w = bits.view(B, H, nb, words).to(torch.int64) & 0xFFFFFFFF
    j = torch.arange(nb, device=bits.device)
    return ((w[..., j // 32] >> (j % 32)) & 1).bool()


@pytest.mark.parametrize("T,tpf", [(2048, 512), (1024, 256), (512, 256)])
def test_route_kernel_matches_torch(T, tpf):
    from drivedit_b200.config import SLAParams
    from drivedit_b200.ops.attention_kernels import sla_plan_kernel, sla_route_blocks
    B, H = 2, 3
    d = H * 64
    qkv = torch.randn(B * T, 3 * d, device="cuda").bfloat16()
    cfg = SLAParams(64, 0.125, True)
    plan = sla_plan_kernel(qkv, B, T, H, cfg, tpf, "frame", sel_bits=True)
    v = qkv.view(B, T, 3, H, 64)
    sel_ref, valid, kk = sla_route_blocks(v[:, :, 0], v[:, :, 1], B, T, H, 64, 0.125, tpf, False, True)
    nb = T // 64
    sel = _sel_from_bits(plan.sel_bits, B, H, nb)
    mismatch = (sel != sel_ref).float().mean().item()
    assert mismatch < 0.01, mismatch
    # W = valid & ~sel
    w = plan.wlin.view(B, H, nb, nb).bool()
    assert torch.equal(w, valid[None, None] & ~sel)
    # list consistency: every selected (q-block, k-block) appears in the forward pairs
    nt = nb // 2
    pb = plan.pair_blocks.view(B, H, nt, -1).cpu()
    pm = plan.pair_mask.view(B, H, nt, -1).cpu()
    pc = plan.pair_count.view(B, H, nt).cpu()
    rebuilt = torch.zeros(B, H, nb, nb, dtype=torch.bool)
    for b in range(B):
        for h in range(H):
            for t in range(nt):
                for p in range(int(pc[b, h, t])):
                    b0, b1 = int(pb[b, h, t, p]) & 0xFFFF, int(pb[b, h, t, p]) >> 16
                    m = int(pm[b, h, t, p])
                    for qh in range(2):
                        for kh, blk in enumerate((b0, b1)):
                            if (m >> (qh * 2 + kh)) & 1:
                                rebuilt[b, h, 2 * t + qh, blk] = True
    assert torch.equal(rebuilt, sel.cpu())
    from test_sla_lists_cpu import rebuild_from_kv_lists
    assert torch.equal(rebuild_from_kv_lists(plan.kv_qtiles.cpu(), plan.kv_qmask.cpu(),
                                             plan.kv_count.cpu(), B, H, nb), sel.cpu())


def test_linear_branch_kernels_match_reference():
    from drivedit_b200.config import SLAParams
    from drivedit_b200.layers.sla import sla_linear_reference
    from drivedit_b200.ops.attention_kernels import (sla_linear_bwd_kernel, sla_linear_fwd_kernel,
                                                     sla_plan_kernel)
    B, H, T, tpf = 2, 2, 1024, 256
    d = H * 64
    qkv = (torch.randn(B * T, 3 * d, device="cuda") * 0.5).bfloat16()
    plan = sla_plan_kernel(qkv, B, T, H, SLAParams(64, 0.25, True), tpf, "frame", sel_bits=True)
    o_lin = sla_linear_fwd_kernel(qkv, plan, B, T, H)
    nb = T // 64
    lin = plan.wlin.view(B, H, nb, nb).bool()
    v = qkv.view(B, T, 3, H, 64)
    q, k, vv = [v[:, :, i].float().requires_grad_(True) for i in range(3)]
    ref = sla_linear_reference(q, k, vv, lin, 64)
    assert _rel(o_lin.view(B, T, H, 64), ref) < 3e-2
    do = torch.randn(B * T, d, device="cuda").bfloat16()
    ref.backward(do.view(B, T, H, 64).float())
    dqkv = torch.zeros(B * T, 3 * d, device="cuda", dtype=torch.bfloat16)
    sla_linear_bwd_kernel(qkv, o_lin, do, plan, dqkv, B, T, H)
    g = dqkv.view(B, T, 3, H, 64)
    assert _rel(g[:, :, 0], q.grad) < 5e-2
    assert _rel(g[:, :, 1], k.grad) < 5e-2
    assert _rel(g[:, :, 2], vv.grad) < 5e-2


def test_batched_gemm():
    from drivedit_b200.ops._ext import ext
    a = torch.randn(6, 128, 256, device="cuda").bfloat16()
    b = torch.randn(6, 256, 4160, device="cuda").bfloat16()   # [batch][K][N]
    d = torch.empty(6 * 128, 4160, device="cuda")
    ext().gemm_batched(a, b, d, 1, False, True)
    ref = torch.bmm(a.float(), b.float()).reshape(6 * 128, 4160)
    assert _rel(d, ref) < 1e-2
    at = torch.randn(6, 256, 128, device="cuda").bfloat16()   # A stored [K][M]
    d2 = torch.empty(6 * 128, 4160, device="cuda")
    ext().gemm_batched(at, b, d2, 1, True, True)
    ref2 = torch.bmm(at.float().transpose(1, 2), b.float()).reshape(6 * 128, 4160)
    assert _rel(d2, ref2) < 1e-2
