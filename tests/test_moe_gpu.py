"""Fused MoE FFN (routing, dispatch, grouped tcgen05 GEMMs, combine) vs the PyTorch path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _frob(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_grouped_gemm_matches_per_expert():
    from drivedit_b200.ops._ext import ext
    from drivedit_b200.ops.gemm import EPI
    torch.manual_seed(0)
    E, d, F, N, k, ns = 8, 256, 128, 300, 2, 1
    logits = torch.randn(N, 32, device="cuda")
    idx, w, sw, probs, counts, psum = ext().moe_route(logits, None, E, k, ns, True)
    mt = (N * k + 127) // 128 + E + ns * ((N + 127) // 128)
    seg_start, seg_count, t_exp, t_row, total, kst, ken, cur = ext().moe_plan(counts, E, ns, N, mt)
    x = torch.randn(N, d, device="cuda").bfloat16()
    xp = torch.empty(mt * 128, d, device="cuda", dtype=torch.bfloat16)
    slot_of = ext().moe_dispatch(x, idx, seg_start, seg_count, cur, xp, E, ns)
    Wt = (torch.randn(E + ns, F, d, device="cuda") * 0.05).bfloat16()
    y = torch.empty(mt * 128, F, device="cuda", dtype=torch.bfloat16)
    ext().gemm_grouped(xp, Wt, y, EPI["bf16"], False, 1, t_exp, t_row, total, kst, ken, mt, None, None)
    ss, sc = seg_start.cpu(), seg_count.cpu()
    for e in range(E + ns):
        r0, c = int(ss[e]), int(sc[e])
        if c == 0:
            continue
        ref = xp[r0:r0 + c].float() @ Wt[e].float().t()
        assert _rel(y[r0:r0 + c], ref) < 2e-2, e
    # weight gradient over segments: D[e] = xp[seg]^T y[seg]
    g = torch.zeros((E + ns) * d, F, device="cuda")
    ext().gemm_grouped(xp, y, g, EPI["f32_acc"], True, 2, t_exp, t_row, total, kst, ken, mt, None, None)
    for e in range(E + ns):
        r0, c = int(ss[e]), int(sc[e])
        ref = xp[r0:r0 + c].float().t() @ y[r0:r0 + c].float()
        assert _rel(g[e * d:(e + 1) * d], ref) < 2e-2, e


def test_moe_world_model_fused_matches_torch():
    from drivedit_b200.config import get_config
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.parallel.flat import FlatParamGroup
    torch.manual_seed(0)
    cfg = get_config("tiny", ["model.n_layers=2", "model.latent_h=32", "model.latent_w=32",
                              "train.frames=2", "model.mlp_hidden=0"])
    from drivedit_b200.config import MoEParams
    cfg.model.moe = MoEParams(num_experts=8, top_k=2, expert_dim=128, num_shared=2, aux_loss_weight=0.01)
    m_ref = WorldDiT(cfg.model).cuda()
    with torch.no_grad():
        for n, p in m_ref.named_parameters():
            if p.abs().sum() == 0 and "router_weight" not in n:
                p.normal_(0, 0.02)
            if "router_weight" in n:  # wider logits: few near-ties between the two paths
                p.mul_(10.0)
    m = WorldDiT(cfg.model).cuda()
    m.load_state_dict(m_ref.state_dict())
    group = FlatParamGroup(m.named_parameters(), "cuda")
    m.enable_fused(group=group)
    x = torch.randn(2, 2, 16, 32, 32, device="cuda")
    t = torch.rand(2, device="cuda")
    a = torch.rand(2, 2, 2, device="cuda")
    m_ref.train(); m.train()
    v_ref, aux_ref = m_ref(x, t, a, return_aux=True)
    v, aux = m(x.bfloat16(), t, a, return_aux=True)
    assert _frob(v, v_ref) < 3e-2
    assert abs(float(aux) - float(aux_ref)) < 1e-3 * max(1.0, abs(float(aux_ref)))
    dv = torch.randn_like(v_ref)
    (v_ref.float() * dv).sum().add(aux_ref).backward()
    group.zero_grad()
    (v.float() * dv).sum().add(aux).backward()
    torch.cuda.synchronize()
    ref = dict(m_ref.named_parameters())
    bad = {}
    for n, p in m.named_parameters():
        g = ref[n].grad
        if g is None or g.abs().max() == 0:
            continue
        # Frobenius-relative: a bf16 rounding that flips one token's k-th expert moves
        # that token's gradients only. Router gradients pass through the top-k
        # renormalisation and softmax Jacobians (two differences of near-equal terms):
        # the same MoE layer run entirely in bf16 PyTorch is ~11% (Frobenius) away from
        # fp32 there, so the router weight and the norm feeding it get a wider bound.
        r = _frob(p.grad, g)
        tol = 0.2 if ("router_weight" in n or "norm2" in n) else 5e-2
        if r > tol:
            bad[n] = r
    assert not bad, bad
