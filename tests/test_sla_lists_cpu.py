"""SLA work lists built by the PyTorch planner (``ops.attention_kernels.sla_plan``): the
forward pair lists and the backward query-block pair lists cover exactly the selected
(query block, key block) pairs, and the backward lists carry no query block that selected
neither key block of a tile."""
import torch


def rebuild_from_kv_lists(kv_qtiles, kv_qmask, kv_count, B, H, nb):
    """Selection matrix [B, H, nb, nb] implied by the backward lists."""
    nt = nb // 2
    qp = kv_qtiles.view(B, H, nt, -1)
    qm = kv_qmask.view(B, H, nt, -1)
    qc = kv_count.view(B, H, nt)
    out = torch.zeros(B, H, nb, nb, dtype=torch.bool)
    for b in range(B):
        for h in range(H):
            for t in range(nt):
                for u in range(int(qc[b, h, t])):
                    pair, m = int(qp[b, h, t, u]), int(qm[b, h, t, u])
                    for qh, blk in enumerate((pair & 0xFFFF, pair >> 16)):
                        for kh in range(2):
                            if (m >> (qh * 2 + kh)) & 1:
                                assert not out[b, h, blk, 2 * t + kh], "pair listed twice"
                                out[b, h, blk, 2 * t + kh] = True
    return out


def test_sla_plan_lists_cover_selection():
    from drivedit_b200.config import SLAParams
    from drivedit_b200.ops.attention_kernels import sla_plan
    torch.manual_seed(0)
    B, H, T, tpf = 2, 3, 1024, 256
    q, k = torch.randn(B, T, H, 64), torch.randn(B, T, H, 64)
    plan = sla_plan(q, k, B, T, H, SLAParams(64, 0.25, True), tpf, "frame")
    nb = T // 64
    nt = nb // 2
    sel = plan.sel
    assert torch.equal(rebuild_from_kv_lists(plan.kv_qtiles, plan.kv_qmask, plan.kv_count,
                                             B, H, nb), sel)
    # one unit per two query blocks that selected a key block of the tile
    per_tile = sel.view(B, H, nb, nt, 2).any(-1).sum(2)                # [B,H,kt]
    assert torch.equal(plan.kv_count.view(B, H, nt), ((per_tile + 1) // 2).int())
    # forward lists rebuild the selection too
    pb = plan.pair_blocks.view(B, H, nt, -1)
    pm = plan.pair_mask.view(B, H, nt, -1)
    pc = plan.pair_count.view(B, H, nt)
    fwd = torch.zeros_like(sel)
    for b in range(B):
        for h in range(H):
            for t in range(nt):
                for p in range(int(pc[b, h, t])):
                    b0, b1 = int(pb[b, h, t, p]) & 0xFFFF, int(pb[b, h, t, p]) >> 16
                    m = int(pm[b, h, t, p])
                    for qh in range(2):
                        for kh, blk in enumerate((b0, b1)):
                            if (m >> (qh * 2 + kh)) & 1:
                                fwd[b, h, 2 * t + qh, blk] = True
    assert torch.equal(fwd, sel)
