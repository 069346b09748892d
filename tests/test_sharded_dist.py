"""Sharded data parallelism (reduce-scatter -> clipped AdamW on the shard -> all-gather)
on 2 gloo ranks matches a single process that averages the ranks' gradients."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

pytestmark = pytest.mark.dist


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(16, 32)
        self.b = nn.Linear(32, 8)
        self.norm = nn.Parameter(torch.ones(8))

    def forward(self, x):
        return self.b(torch.tanh(self.a(x))) * self.norm

    def no_decay_names(self):
        return [n for n, p in self.named_parameters() if p.dim() < 2]


def _data(rank, step):
    g = torch.Generator().manual_seed(1000 * step + rank)
    return torch.randn(4, 16, generator=g), torch.randn(4, 8, generator=g)


def _worker(rank, world, port, steps, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from drivedit_b200.parallel.sharded import ShardedDataParallel

    torch.manual_seed(0)
    net = _Net()
    eng = ShardedDataParallel(net, transport="nccl", lr=1e-2, weight_decay=0.1, grad_clip=0.5)
    for s in range(steps):
        eng.zero_grad()
        x, y = _data(rank, s)
        ((net(x) - y) ** 2).mean().backward()
        eng.step()
    if rank == 0:
        q.put({k: v.detach().clone() for k, v in net.state_dict().items()})
    else:
        q.put(None)
    dist.destroy_process_group()


def test_sharded_matches_single_process():
    from drivedit_b200.parallel.flat import FlatParamGroup
    from drivedit_b200.training.optim import FlatAdamW

    world, steps = 2, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = [r for r in results if r is not None][0]
    # reference: one process, gradients averaged over the two ranks' batches
    torch.manual_seed(0)
    net = _Net()
    grp = FlatParamGroup(net.named_parameters(), "cpu", no_decay=net.no_decay_names())
    opt = FlatAdamW(grp, lr=1e-2, weight_decay=0.1, grad_clip=0.5)
    for s in range(steps):
        grp.zero_grad()
        for r in range(world):
            x, y = _data(r, s)
            ((net(x) - y) ** 2).mean().backward()
        opt.step(grad_scale=1.0 / world)
    for k, v in net.state_dict().items():
        assert torch.allclose(got[k], v, atol=1e-5, rtol=1e-4), k
