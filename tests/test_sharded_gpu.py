"""The peer-memory fused optimizer step (reduce-scatter by peer loads -> clipped AdamW on
the shard -> all-gather by peer stores) matches the NCCL collective path on 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(64, 256)
        self.b = nn.Linear(256, 64)
        self.norm = nn.Parameter(torch.ones(64))

    def forward(self, x):
        return self.b(torch.tanh(self.a(x))) * self.norm

    def no_decay_names(self):
        return [n for n, p in self.named_parameters() if p.dim() < 2]


def _worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from drivedit_b200.ops._ext import check_device_status
    from drivedit_b200.parallel.sharded import ShardedDataParallel

    out = {}
    for transport in ("fused", "nccl"):
        torch.manual_seed(0)
        net = _Net().cuda()
        eng = ShardedDataParallel(net, transport=transport, lr=1e-2, weight_decay=0.1, grad_clip=0.5)
        for s in range(3):
            eng.zero_grad()
            g = torch.Generator(device="cuda").manual_seed(100 * s + rank)
            x = torch.randn(32, 64, device="cuda", generator=g)
            y = torch.randn(32, 64, device="cuda", generator=g)
            ((net(x) - y) ** 2).mean().backward()
            eng.step()
        torch.cuda.synchronize()
        out[transport] = {k: v.detach().cpu().clone() for k, v in net.state_dict().items()}
        out[transport + "_compute"] = eng.flat.compute.float().cpu().clone()
        eng.close()
    check_device_status()
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_sharded_step_matches_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        for k, v in res[r]["nccl"].items():
            assert torch.allclose(res[r]["fused"][k], v, atol=1e-5, rtol=1e-4), (r, k)
    # both ranks hold identical weights, and the bf16 copy matches the fp32 master
    for k in res[0]["fused"]:
        assert torch.equal(res[0]["fused"][k], res[1]["fused"][k]), k
    assert torch.equal(res[0]["fused_compute"], res[1]["fused_compute"])
