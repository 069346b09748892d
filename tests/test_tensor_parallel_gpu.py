"""Tensor-parallel streaming rollout.

* one rank: the tensor-parallel path (peer-shard A loads and peer-store reduce-scatter in
  the GEMM, row sums, bounded barriers) reproduces the single-GPU fused rollout;
* two ranks: the peer-memory transport and the NCCL transport both reproduce it, and every
  rank ends with the same frames;
* both layouts: row-sharded activations (all-gather / reduce-scatter) and, for small
  chunks, replicated rows with all-reduces by peer loads.
"""
import datetime
import os
import queue
import socket
import time

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


def _rollout(model, tp_transport=None, ag_tma_max_n=256, replicate_rows_max=0):
    from drivedit_b200.config import RolloutConfig
    from drivedit_b200.inference.rollout import StreamingRollout

    cfg = RolloutConfig(total_frames=8, chunk_frames=2, flow_steps=2, window_frames=4, context_frames=2)
    m = model.cfg
    g = torch.Generator(device="cuda").manual_seed(3)
    ctx = torch.randn(1, 2, m.latent_channels, m.latent_h, m.latent_w, device="cuda", generator=g)
    act = torch.rand(1, 8, m.action_dim, device="cuda", generator=g) * 2 - 1
    target = model
    tp = None
    if tp_transport is not None:
        from drivedit_b200.parallel.tensor import TensorParallelWorldDiT

        tp = TensorParallelWorldDiT(model, transport=tp_transport, ag_tma_max_n=ag_tma_max_n,
                                    replicate_rows_max=replicate_rows_max)
        target = tp
    res = StreamingRollout(target, cfg).run(ctx, act, 8, generator=g)
    torch.cuda.synchronize()
    if tp is not None:
        tp.close()
    return res.frames.float().cpu().numpy()


def _model():
    from drivedit_b200.config.presets import ModelConfig
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.parallel.flat import FlatParamGroup

    torch.manual_seed(0)
    cfg = ModelConfig(n_layers=2, d_model=256, n_heads=4, mlp_hidden=1024, latent_channels=16, latent_h=16,
                      latent_w=32, action_dim=3)
    model = WorldDiT(cfg).cuda().eval()
    with torch.no_grad():                       # a non-trivial output head
        model.out_proj.weight.normal_(0, 0.02)
    model.enable_fused(group=FlatParamGroup(model.named_parameters(), "cuda"))
    return model


def _worker(rank, world, port, q, transports):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from drivedit_b200.ops._ext import check_device_status

    model = _model()
    out = {"single": _rollout(model)}
    for t in transports:
        out[t] = _rollout(model, t)
        out[t + "_rep"] = _rollout(model, t, replicate_rows_max=1 << 30)
    if "fused" in transports:      # every all-gather inside the GEMM as peer TMA loads
        out["fused_tma"] = _rollout(model, "fused", ag_tma_max_n=1 << 20)
    check_device_status()
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


def _collect(q, procs, n, timeout):
    out, t0 = [], time.monotonic()
    while len(out) < n:
        try:
            out.append(q.get(timeout=5))
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            assert not dead, f"worker exited with {dead}"
            assert time.monotonic() - t0 < timeout, "workers timed out"
    return dict(out)


def _run(world, transports):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, transports)) for r in range(world)]
    for p in procs:
        p.start()
    res = _collect(q, procs, world, 600)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def _close(a, b, tol):
    err = np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-12)
    assert err < tol, err


def test_tensor_parallel_rollout_one_rank_matches_single_gpu():
    res = _run(1, ["fused"])[0]
    _close(res["fused"], res["single"], 2e-2)
    _close(res["fused_rep"], res["single"], 2e-2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_rollout_two_ranks():
    res = _run(2, ["fused", "nccl"])
    for r in range(2):
        _close(res[r]["fused"], res[r]["single"], 2e-2)
        _close(res[r]["nccl"], res[r]["single"], 2e-2)
        _close(res[r]["fused_tma"], res[r]["single"], 2e-2)
        _close(res[r]["fused_rep"], res[r]["single"], 2e-2)
        _close(res[r]["nccl_rep"], res[r]["single"], 2e-2)
    # replicated rows: both ranks hold bit-identical frames
    assert np.array_equal(res[0]["fused_rep"], res[1]["fused_rep"])
    np.testing.assert_array_equal(res[0]["fused"], res[1]["fused"])
