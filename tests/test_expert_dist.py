"""Expert parallelism on CPU: the movement plan's index arithmetic (simulated copies over
3 ranks), the MoE FFN's expert-parallel forward/backward over 2 gloo ranks against one
process holding every expert, and one fsdp_ep training step against plain fsdp."""
import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.dist


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _np(obj):
    """Tensors -> numpy so results survive the worker's exit (no shared-memory handles)."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().numpy().copy()
    if isinstance(obj, dict):
        return {k: _np(v) for k, v in obj.items()}
    return obj


def _t(obj):
    if isinstance(obj, np.ndarray):
        return torch.from_numpy(obj)
    if isinstance(obj, dict):
        return {k: _t(v) for k, v in obj.items()}
    return obj


def _run(fn, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return {r: _t(v) for r, v in out}


# ----------------------------------------------------------------------------- plan
@pytest.mark.parametrize("transport", ["fused", "nccl"])
def test_plan_moves_every_row_to_its_owner_and_back(transport):
    """Simulate the pull/push block copies of every rank with numpy buffers."""
    from drivedit_b200.parallel.expert import EpPlan

    W, E, k, ns = 3, 6, 2, 1
    rng = np.random.default_rng(0)
    N = [5, 7, 4]
    table = np.zeros((W, E), np.int64)
    routes = []
    for s in range(W):
        e = np.stack([rng.choice(E, k, replace=False) for _ in range(N[s])])
        routes.append(e)
        table[s] = np.bincount(e.reshape(-1), minlength=E)
    # source compact buffers: row value = (src, expert, token)
    compact = []
    for s in range(W):
        flat = routes[s].reshape(-1)
        order = np.argsort(flat, kind="stable")
        compact.append(np.stack([np.full(len(order), s), flat[order], order // k], 1))
    ret = [np.full_like(c, -1) for c in compact]
    for r in range(W):
        ep = SimpleNamespace(world=W, rank=r, num_experts=E, local_experts=E // W, transport=transport,
                             local_range=lambda r=r: (r * (E // W), (r + 1) * (E // W)))
        plan = EpPlan(ep, table)
        arr, sizes, nb = plan.packet(ep, N[r], ns, k)
        parts = np.split(arr, np.cumsum(sizes)[:-1])
        pull = parts[0].reshape(-1, 4)
        prefix = parts[1]
        push = parts[2].reshape(-1, 4)
        rows = np.diff(np.append(prefix, plan.n_recv))
        owner = np.full((plan.owner_rows, 3), -1)
        if transport == "fused":
            for (sr, srow, _, drow), n in zip(pull, rows):
                owner[drow:drow + n] = compact[sr][srow:srow + n]
        else:   # source-major receive buffer first (what all_to_all delivers)
            recv = np.concatenate([compact[s][plan.compact_start[s, plan.lo]:
                                              plan.compact_start[s, plan.lo] + plan.recv_splits[s]]
                                   for s in range(W)])
            for (_, srow, _, drow), n in zip(pull, rows):
                owner[drow:drow + n] = recv[srow:srow + n]
        # every row of my segments belongs to my expert of that segment; padding stays -1
        lc = plan.local_counts
        seg = np.concatenate([[0], np.cumsum((lc + 127) // 128 * 128)])
        for j in range(E // W):
            blk = owner[seg[j]:seg[j] + lc[j]]
            assert (blk[:, 1] == plan.lo + j).all()
            assert (owner[seg[j] + lc[j]:seg[j + 1]] == -1).all()
        assert (owner[:, 0] >= 0).sum() == plan.n_recv
        # push back (identity expert): sources get their rows at their compact positions
        if transport == "fused":
            for (_, srow, dr, drow), n in zip(push, rows):
                ret[dr][drow:drow + n] = owner[srow:srow + n]
        else:
            stage = np.full((plan.n_recv, 3), -1)
            for (_, srow, _, drow), n in zip(push, rows):
                stage[drow:drow + n] = owner[srow:srow + n]
            o = 0
            for s in range(W):
                c0 = plan.compact_start[s, plan.lo]
                ret[s][c0:c0 + plan.recv_splits[s]] = stage[o:o + plan.recv_splits[s]]
                o += plan.recv_splits[s]
        # dispatch segments of this source: compact starts, then shared segments
        seg_start = parts[5]
        assert (seg_start[:E] == plan.compact_start[r]).all()
        assert seg_start[E] == 0 and parts[6][E] == N[r]
    for s in range(W):
        assert (ret[s] == compact[s]).all()


# ----------------------------------------------------------------------------- MoE FFN
def _moe():
    from drivedit_b200.layers.moe import MoEFFN

    torch.manual_seed(0)
    return MoEFFN(32, num_experts=4, top_k=2, expert_dim=32, num_shared_experts=1)


def _xg(rank):
    g = torch.Generator().manual_seed(10 + rank)
    return torch.randn(12, 32, generator=g), torch.randn(12, 32, generator=g)


def _moe_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from drivedit_b200.parallel.expert import ExpertParallel

    moe = _moe()
    ep = ExpertParallel(num_experts=4)
    moe.shard_experts(ep)
    x, g = _xg(rank)
    y = moe(x).output
    (y * g).sum().backward()
    q.put((rank, _np({"y": y.detach(), "w13": moe.w13.grad.clone(), "w2": moe.w2.grad.clone(),
                  "w13s": moe.w13_shared.grad.clone(), "router": moe.router_weight.grad.clone(),
                  "counts": moe.last_counts.clone(), "lo": ep.local_range()[0]})))
    dist.destroy_process_group()


def test_moe_expert_parallel_matches_single_process():
    world = 2
    got = _run(_moe_worker, world)
    E = 4
    full = _moe()
    ys, grads13, grads2 = [], torch.zeros_like(full.w13), torch.zeros_like(full.w2)
    per_rank = []
    total_counts = 0
    for r in range(world):
        full.zero_grad()
        x, g = _xg(r)
        y = full(x).output
        (y * g).sum().backward()
        ys.append(y.detach())
        grads13 += full.w13.grad
        grads2 += full.w2.grad
        per_rank.append((full.w13.grad[E:].clone(), full.router_weight.grad.clone()))
        total_counts = total_counts + full.last_counts
    for r in range(world):
        o = got[r]
        lo = o["lo"]
        torch.testing.assert_close(o["y"], ys[r], rtol=1e-5, atol=1e-6)
        # routed experts: gradient summed over every source's tokens
        torch.testing.assert_close(o["w13"], grads13[lo:lo + 2], rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(o["w2"], grads2[lo:lo + 2], rtol=1e-4, atol=1e-6)
        # replicated parts: this rank's own gradient
        torch.testing.assert_close(o["w13s"], per_rank[r][0], rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(o["router"], per_rank[r][1], rtol=1e-4, atol=1e-6)
        # the bias update sees the global counts on every rank
        assert torch.equal(o["counts"].long(), total_counts.long())


# ----------------------------------------------------------------------------- trainer
def _cfg(parallel):
    from drivedit_b200.config.presets import Config, ModelConfig, MoEParams, TrainConfig

    m = ModelConfig(n_layers=2, d_model=32, n_heads=2, mlp_hidden=64, latent_channels=4,
                    latent_h=8, latent_w=8, moe=MoEParams(num_experts=4, top_k=2, expert_dim=32,
                                                          num_shared=1, aux_loss_weight=0.01))
    return Config(model=m, train=TrainConfig(batch_per_gpu=1, frames=2, lr=1e-2, parallel=parallel))


def _train_worker(rank, world, port, q, parallel):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from drivedit_b200.data import make_batch
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.training.trainer import WorldModelTrainer

    cfg = _cfg(parallel)
    torch.manual_seed(0)
    model = WorldDiT(cfg.model)
    tr = WorldModelTrainer(model, cfg.train, "cpu", process_group=dist.group.WORLD)
    batch = make_batch(cfg, generator=torch.Generator().manual_seed(100 + rank))
    loss = tr.train_step(batch)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    q.put((rank, _np({"loss": float(loss), "sd": sd,
                      "lo": tr.ep.local_range()[0] if tr.ep is not None else 0})))
    dist.destroy_process_group()


def test_fsdp_ep_step_matches_fsdp():
    world = 2
    ep = _run(_train_worker, world, "fsdp_ep")
    ref = _run(_train_worker, world, "fsdp")
    E = 4
    for r in range(world):
        assert abs(ep[r]["loss"] - ref[r]["loss"]) < 1e-5
        sd, rsd, lo = ep[r]["sd"], ref[r]["sd"], ep[r]["lo"]
        for name, v in sd.items():
            if name.endswith("moe.w13") or name.endswith("moe.w2"):
                want = rsd[name][lo:lo + E // world]
            elif name.endswith("moe.w13_shared"):
                want = rsd[name.replace("w13_shared", "w13")][E:]
            elif name.endswith("moe.w2_shared"):
                want = rsd[name.replace("w2_shared", "w2")][E:]
            elif "expert_bias" in name or "expert_load_ema" in name:
                continue   # EP balances on global counts, plain fsdp on local ones
            else:
                want = rsd[name]
            torch.testing.assert_close(v, want, rtol=1e-4, atol=1e-6, msg=name)
