"""Sanitizer substitutes: the deterministic MoE permutation (stable (expert, token)
order, bit-identical expert gradients run to run) and the bounds-checked index kernels
(a corrupt routing table is reported in the status word instead of faulting). The bad
indices used here still address allocated memory, so even an unchecked kernel could
not fault."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _moe(seed=0):
    from drivedit_b200.layers.moe import MoEFFN

    torch.manual_seed(seed)
    return MoEFFN(256, num_experts=16, top_k=4, expert_dim=128, num_shared_experts=1).cuda()


def test_deterministic_dispatch_is_a_stable_sort():
    from drivedit_b200.ops import debug
    from drivedit_b200.ops._ext import ext

    torch.manual_seed(1)
    N, E, k, ns, d = 3000, 16, 4, 1, 256
    h = torch.randn(N, d, device="cuda").bfloat16()
    logits = torch.randn(N, E + ns, device="cuda")  # routed, then shared-gate logits
    idx, w, sw, probs, counts, psum = ext().moe_route(logits, torch.zeros(E, device="cuda"), E, k, ns, True)
    mt = (N * k + 127) // 128 + E + ns * ((N + 127) // 128)
    plan = ext().moe_plan(counts, E, ns, N, mt)
    xp = torch.empty(mt * 128, d, device="cuda", dtype=torch.bfloat16)
    with debug.deterministic():
        slot = ext().moe_dispatch(h, idx, plan[0], plan[1], plan[7], xp, E, ns).cpu()
    seg = plan[0].cpu()
    flat = idx.cpu().reshape(-1).long()
    order = torch.argsort(flat * (N * k) + torch.arange(N * k), stable=True)  # (expert, token, route)
    want = torch.empty(N * k, dtype=torch.long)
    pos = torch.zeros(E, dtype=torch.long)
    for i in order.tolist():
        e = int(flat[i])
        want[i] = int(seg[e]) + int(pos[e])
        pos[e] += 1
    assert torch.equal(slot[:, :k].reshape(-1).long(), want)
    # the rows landed where the slots say
    t = torch.arange(N).repeat_interleave(k)
    assert torch.equal(xp.cpu()[want], h.cpu()[t])


def test_deterministic_moe_gradients_repeat_bit_for_bit():
    from drivedit_b200.ops import debug
    from drivedit_b200.parallel.flat import FlatParamGroup

    x = torch.randn(4096, 256, device="cuda").bfloat16()
    grads = []
    with debug.deterministic():
        for _ in range(2):
            moe = _moe()
            g = FlatParamGroup(moe.named_parameters(), "cuda")
            from drivedit_b200.ops.moe import moe_ffn_backward, moe_ffn_forward

            out, aux, sv = moe_ffn_forward(x, x, moe, g.compute_view)
            moe_ffn_backward(torch.ones_like(out), torch.ones((), device="cuda"), moe,
                             g.compute_view, sv)
            torch.cuda.synchronize()
            grads.append(g.grad.clone())
    assert torch.equal(grads[0], grads[1])


def test_bounds_mode_reports_a_bad_expert_id_and_a_bad_slot():
    from drivedit_b200.ops import debug
    from drivedit_b200.ops._ext import ext, reset_device_status

    reset_device_status()
    N, E, k, ns, d = 512, 8, 2, 1, 128
    h = torch.randn(N, d, device="cuda").bfloat16()
    logits = torch.randn(N, E + ns, device="cuda")
    idx, w, sw, probs, counts, psum = ext().moe_route(logits, torch.zeros(E, device="cuda"), E, k, ns, True)
    mt = (N * k + 127) // 128 + E + ns * ((N + 127) // 128)
    plan = ext().moe_plan(counts, E, ns, N, mt)
    xp = torch.zeros(mt * 128, d, device="cuda", dtype=torch.bfloat16)
    bad = idx.clone()
    bad[7, 1] = E          # one past the routed experts (still inside the E + ns tables)
    with debug.check_bounds():
        slot = ext().moe_dispatch(h, bad, plan[0], plan[1], plan[7], xp, E, ns)
        torch.cuda.synchronize()
        assert int(ext().read_status()) == debug.BAD_INDEX_STATUS
        assert debug.bad_index() == E and int(slot[7, 1]) == -1
        reset_device_status()
        # a slot past y's rows; y is a view of a larger buffer, so the read stays allocated
        big = torch.zeros(mt * 128 + 256, d, device="cuda", dtype=torch.bfloat16)
        y = big[:mt * 128]
        good = ext().moe_dispatch(h, idx, plan[0], plan[1], plan[7], xp, E, ns)
        good[3, 0] = mt * 128 + 5
        ext().moe_combine(w, sw, good, y, None, ns)
        torch.cuda.synchronize()
        assert int(ext().read_status()) == debug.BAD_INDEX_STATUS
        assert debug.bad_index() == mt * 128 + 5
    reset_device_status()
    assert not debug.is_checking_bounds()
