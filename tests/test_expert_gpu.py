"""Expert-parallel MoE on the GPU kernels.

* one rank (one GPU): the expert-parallel kernel path (owner gather of token rows from
  the peer-mapped buffers, owner-side partial sums, shared experts apart) reproduces the
  single-device MoE kernel path on the same weights;
* two ranks (two GPUs): one fsdp_ep training step with the peer-memory transport matches
  the NCCL all-to-all transport and plain fsdp (every expert on every rank).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _np(obj):
    if isinstance(obj, torch.Tensor):
        return obj.detach().float().cpu().numpy().copy()
    if isinstance(obj, dict):
        return {k: _np(v) for k, v in obj.items()}
    return obj


def _collect(q, procs, n, timeout):
    """``n`` results from ``q``; fails fast when a worker died instead of waiting."""
    import queue
    import time

    out, t0 = [], time.monotonic()
    while len(out) < n:
        try:
            out.append(q.get(timeout=5))
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead, f"worker exited with {dead}"
            assert time.monotonic() - t0 < timeout, "workers timed out"
    return out


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _cfg(parallel, fused=True):
    from drivedit_b200.config.presets import Config, ModelConfig, MoEParams, TrainConfig

    m = ModelConfig(n_layers=2, d_model=256, n_heads=4, mlp_hidden=512, latent_channels=16,
                    latent_h=16, latent_w=32, moe=MoEParams(num_experts=8, top_k=2, expert_dim=256,
                                                            num_shared=1, aux_loss_weight=0.01))
    return Config(model=m, train=TrainConfig(batch_per_gpu=2, frames=4, lr=1e-3, dtype="bf16",
                                             parallel=parallel, fused_collectives=fused))


# ----------------------------------------------------------------------------- one GPU
def _one_rank_worker(rank, world, port, q):
    _init(rank, world, port)
    from drivedit_b200.layers.moe import MoEFFN
    from drivedit_b200.ops._ext import check_device_status
    from drivedit_b200.ops.moe import moe_ffn_backward, moe_ffn_backward_ep, moe_ffn_forward, moe_ffn_forward_ep
    from drivedit_b200.parallel.expert import ExpertParallel
    from drivedit_b200.parallel.flat import FlatParamGroup

    d, E, k, F, ns, N = 256, 8, 2, 256, 2, 1000
    res = {}
    for mode in ("local", "ep"):
        torch.manual_seed(0)
        moe = MoEFFN(d, E, k, F, ns).cuda()
        if mode == "ep":
            ep = ExpertParallel(num_experts=E, transport="fused", device="cuda")
            moe.shard_experts(ep)
            main = FlatParamGroup([(n, p) for n, p in moe.named_parameters() if n not in ("w13", "w2")])
            main.linked.append(FlatParamGroup([("w13", moe.w13), ("w2", moe.w2)]))
            grp = main
        else:
            grp = FlatParamGroup(moe.named_parameters())
        grp.zero_grad()
        g = torch.Generator(device="cuda").manual_seed(1)
        h = torch.randn(N, d, device="cuda", generator=g).to(torch.bfloat16)
        r = torch.randn(N, d, device="cuda", generator=g).to(torch.bfloat16)
        dout = torch.randn(N, d, device="cuda", generator=g).to(torch.bfloat16)
        fwd, bwd = (moe_ffn_forward, moe_ffn_backward) if mode == "local" else (moe_ffn_forward_ep,
                                                                                moe_ffn_backward_ep)
        out, aux, sv = fwd(h, r, moe, grp.compute_view)
        dh = bwd(dout, torch.ones((), device="cuda"), moe, grp.compute_view, sv)
        torch.cuda.synchronize()
        w13g = moe.w13.grad if mode == "local" else torch.cat([moe.w13.grad, moe.w13_shared.grad])
        w2g = moe.w2.grad if mode == "local" else torch.cat([moe.w2.grad, moe.w2_shared.grad])
        res[mode] = dict(out=out, dh=dh, w13=w13g, w2=w2g, router=moe.router_weight.grad)
        if mode == "ep":
            ep.close()
    check_device_status()
    q.put((rank, _np(res)))
    dist.barrier()
    dist.destroy_process_group()


def test_expert_parallel_kernel_path_matches_local_one_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_one_rank_worker, args=(0, 1, _port(), q))
    p.start()
    _, res = _collect(q, [p], 1, 300)[0]
    p.join(timeout=60)
    assert p.exitcode == 0
    a, b = res["local"], res["ep"]
    for key in ("out", "dh", "w13", "w2", "router"):
        x, y = a[key], b[key]
        err = np.linalg.norm(x - y) / (np.linalg.norm(x) + 1e-12)
        assert err < 5e-3, (key, err)   # owner partial sums are rounded to bf16 once more


# ----------------------------------------------------------------------------- two GPUs
def _two_rank_worker(rank, world, port, q):
    _init(rank, world, port)
    from drivedit_b200.data import make_batch
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.ops._ext import check_device_status
    from drivedit_b200.training.trainer import WorldModelTrainer

    out = {}
    for name, parallel, fused in (("ep_fused", "fsdp_ep", True), ("ep_nccl", "fsdp_ep", False),
                                  ("fsdp", "fsdp", True)):
        cfg = _cfg(parallel, fused)
        torch.manual_seed(0)
        model = WorldDiT(cfg.model)
        tr = WorldModelTrainer(model, cfg.train, f"cuda:{rank}", process_group=dist.group.WORLD)
        batch = make_batch(cfg, generator=torch.Generator().manual_seed(100 + rank),
                           device=f"cuda:{rank}")
        sd0 = _np(model.state_dict())
        losses = [float(tr.train_step(batch))]
        sd1 = _np(model.state_dict())
        losses.append(float(tr.train_step(batch)))   # second step reuses every EP buffer
        torch.cuda.synchronize()
        out[name] = {"loss": losses, "lo": tr.ep.local_range()[0] if tr.ep is not None else 0,
                     "sd0": sd0, "sd1": sd1, "sd2": _np(model.state_dict())}
        tr.engine.close()
        if tr.ep is not None:
            tr.ep.close()
    check_device_status()
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fsdp_ep_two_gpus_matches_nccl_and_fsdp():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(_collect(q, procs, world, 600))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    E = 8
    for r in range(world):
        a, b, c = res[r]["ep_fused"], res[r]["ep_nccl"], res[r]["fsdp"]
        # peer-memory transport (per-owner partial sums) against the all-to-all transport
        assert abs(a["loss"][0] - b["loss"][0]) < 1e-3 * abs(b["loss"][0]), (a["loss"], b["loss"])
        assert abs(a["loss"][1] - b["loss"][1]) < 1e-3 * abs(b["loss"][1])
        # parameter updates (Adam moves every weight by about +-lr whatever its gradient's size,
        # so updates are compared by direction over each whole tensor)
        def cos(u, v):
            u, v = u.ravel().astype(np.float64), v.ravel().astype(np.float64)
            nu, nv = np.linalg.norm(u), np.linalg.norm(v)
            if nu < 1e-12 and nv < 1e-12:      # neither run moved this tensor
                return 1.0
            return float(u @ v / (nu * nv + 1e-30))

        for n in a["sd1"]:
            if "expert_bias" in n or "expert_load_ema" in n:
                continue
            assert cos(a["sd1"][n] - a["sd0"][n], b["sd1"][n] - b["sd0"][n]) > 0.97, n
        # against every expert on every rank (first step): equal up to bf16 rounding
        assert abs(a["loss"][0] - c["loss"][0]) < 2e-3 * abs(c["loss"][0])
        lo = a["lo"]

        def ref(sd, n):
            if n.endswith("moe.w13") or n.endswith("moe.w2"):
                return sd[n][lo:lo + E // world]
            if n.endswith("_shared"):
                return sd[n.replace("w13_shared", "w13").replace("w2_shared", "w2")][E:]
            return sd[n]

        for n in a["sd1"]:
            if "expert_bias" in n or "expert_load_ema" in n:
                continue
            assert cos(a["sd1"][n] - a["sd0"][n], ref(c["sd1"], n) - ref(c["sd0"], n)) > 0.95, n
