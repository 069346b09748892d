"""MoE layer semantics on CPU: routing, experts, aux loss, bias balancing, reference
checkpoint keys, and the hand-written router gradient used by the fused backward."""
import torch
import torch.nn.functional as F

from drivedit_b200.layers.mlp import split_gu
from drivedit_b200.layers.moe import MoEFFN, aux_load_balance_loss
from drivedit_b200.ops.moe import router_dlogits


def _naive(moe, x):
    w, e, p, g = moe.route(x)
    out = torch.zeros_like(x)
    for n in range(x.shape[0]):
        for j in range(moe.top_k):
            out[n] += w[n, j] * moe._expert(int(e[n, j]), x[n:n + 1])[0]
        for s in range(moe.num_shared_experts):
            out[n] += g[n, s] * moe._expert(moe.num_experts + s, x[n:n + 1])[0]
    return out


def test_moe_forward_matches_per_token_loop():
    torch.manual_seed(0)
    moe = MoEFFN(32, num_experts=6, top_k=2, expert_dim=32, num_shared_experts=1).eval()
    x = torch.randn(40, 32)
    y = moe(x).output if hasattr(moe(x), "output") else moe(x)[0]
    assert torch.allclose(y, _naive(moe, x), atol=1e-5)


def test_router_dlogits_matches_autograd():
    torch.manual_seed(1)
    N, E, k, ns, e_pad = 50, 8, 3, 2, 32
    logits = torch.randn(N, e_pad, dtype=torch.float64) * 2
    logits[:, E + ns:] = 0
    logits.requires_grad_(True)
    bias = torch.randn(E, dtype=torch.float64) * 0.1
    p = F.softmax(logits[:, :E] + bias, -1)
    wt, idx = torch.topk(p, k, -1)
    w = wt / (wt.sum(-1, keepdim=True) + 1e-8)
    g = F.softmax(logits[:, E:E + ns], -1)
    counts = torch.bincount(idx.reshape(-1), minlength=E).double()
    f = counts / (N * k)
    A, Bs = torch.randn(N, k, dtype=torch.float64), torch.randn(N, ns, dtype=torch.float64)
    d_aux = torch.tensor(0.37, dtype=torch.float64)
    loss = (w * A).sum() + (g * Bs).sum() + d_aux * E * (f * p.mean(0)).sum()
    loss.backward()
    dw = torch.cat([A, Bs], -1)
    got = router_dlogits(p.detach(), idx, w.detach(), g.detach(), dw, d_aux, f, E, k, ns, e_pad)
    assert torch.allclose(got.double(), logits.grad, atol=1e-5)


def test_aux_loss_uniform_is_one_and_bias_balances():
    E = 4
    p = torch.full((8, E), 1.0 / E)
    e = torch.arange(8).remainder(E)[:, None]
    aux, counts = aux_load_balance_loss(p, e, E)
    assert abs(float(aux) - 1.0) < 1e-6 and counts.tolist() == [2.0] * 4
    moe = MoEFFN(16, num_experts=E, top_k=1, expert_dim=32, bias_update_speed=0.1).train()
    moe.update_bias(torch.tensor([8.0, 0, 0, 0]), 8)
    assert moe.expert_bias[0] < 0 and (moe.expert_bias[1:] > 0).all()


def test_reference_key_roundtrip():
    torch.manual_seed(2)
    a = MoEFFN(32, num_experts=4, top_k=2, expert_dim=32, num_shared_experts=1)
    sd = a.reference_state_dict()
    assert "experts.0.w_gate.weight" in sd and "shared_experts.0.w_out.weight" in sd
    b = MoEFFN(32, num_experts=4, top_k=2, expert_dim=32, num_shared_experts=1)
    b.load_state_dict(sd)
    for n, p in a.named_parameters():
        assert torch.equal(p, dict(b.named_parameters())[n]), n
    gu = torch.randn(3, 64)
    g, u = split_gu(gu)
    assert g.shape == u.shape == (3, 32)
