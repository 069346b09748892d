"""Checkpointing (atomic, checksummed, sharded, fallback), heartbeat failure detection
on gloo ranks, reference-format export, metrics logging (CPU only)."""
import multiprocessing as mp
import os
import time

import pytest
import torch
import torch.nn as nn

from drivedit_b200.training.distributed import (CheckpointManager, Heartbeat, PeerFailure, check_finite,
                                                export_reference_checkpoint, get_available_port, reduce_dict)


def test_checkpoint_roundtrip_fallback_and_keep(tmp_path):
    torch.manual_seed(0)
    m = nn.Linear(4, 3)
    opt = torch.optim.AdamW(m.parameters(), lr=0.1)
    m(torch.randn(2, 4)).sum().backward()
    opt.step()
    cm = CheckpointManager(str(tmp_path), keep_checkpoints=2)
    for s in (10, 20, 30):
        cm.save_checkpoint(m, opt, None, epoch=0, step=s, loss=1.0 / s, metrics={"a": s})
    assert sorted(p.name for p in tmp_path.glob("checkpoint_step_*.pt")) == ["checkpoint_step_20.pt",
                                                                               "checkpoint_step_30.pt"]
    m2 = nn.Linear(4, 3)
    info = cm.load_checkpoint(m2, torch.optim.AdamW(m2.parameters()))
    assert info["step"] == 30 and torch.equal(m2.weight, m.weight)
    # corrupt the newest checkpoint: the loader verifies the checksum and falls back
    p = tmp_path / "checkpoint_step_30.pt"
    b = bytearray(p.read_bytes())
    b[len(b) // 2] ^= 0xFF
    p.write_bytes(bytes(b))
    info = cm.load_checkpoint(nn.Linear(4, 3))
    assert info["step"] == 20
    (tmp_path / "checkpoint_step_20.pt").write_bytes(b"truncated")
    assert cm.load_checkpoint(nn.Linear(4, 3)) == {}


def test_sharded_checkpoint_requires_all_shards(tmp_path):
    m = nn.Linear(2, 2)
    for r in range(2):
        cm = CheckpointManager(str(tmp_path), rank=r, world_size=2)
        cm.save_checkpoint(m, None, None, 0, 5, 0.5, optimizer_shard={"m": torch.full((3,), float(r))})
    got = CheckpointManager(str(tmp_path), rank=1, world_size=2).load_checkpoint(nn.Linear(2, 2))
    assert torch.equal(got["optimizer_shard"]["m"], torch.ones(3))
    (tmp_path / "checkpoint_step_5_rank1.pt").unlink()
    assert CheckpointManager(str(tmp_path), rank=1, world_size=2).load_checkpoint(nn.Linear(2, 2)) == {}
    assert CheckpointManager(str(tmp_path), rank=0, world_size=4).load_checkpoint(nn.Linear(2, 2)) == {}


def test_reference_export_and_sentinels(tmp_path):
    from drivedit_b200.layers.moe import MoEFFN
    m = nn.Module()
    m.moe = MoEFFN(32, num_experts=4, top_k=2, expert_dim=32, num_shared_experts=1)
    sd = export_reference_checkpoint(m, str(tmp_path / "ref.pt"))
    assert "moe.experts.3.w_out.weight" in sd and "moe.shared_gate.weight" in sd and "moe.w13" not in sd
    m2 = nn.Module()
    m2.moe = MoEFFN(32, num_experts=4, top_k=2, expert_dim=32, num_shared_experts=1)
    m2.load_state_dict(torch.load(tmp_path / "ref.pt")["model_state_dict"])
    assert torch.equal(m2.moe.w13, m.moe.w13)
    check_finite(torch.ones(3), torch.zeros(2))
    with pytest.raises(FloatingPointError):
        check_finite(torch.ones(3), torch.tensor([float("nan")]), names=["a", "b"])
    assert reduce_dict({"x": torch.tensor(2.0)}, 1) == {"x": 2.0}


def _hb_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, timeout_s=1.5)
    try:
        for step in range(40):
            if rank == 1 and step == 3:
                os._exit(0)  # this rank dies between steps, no collective in flight
            hb.beat(step)
            time.sleep(0.1)
            hb.check()
        q.put((rank, "no failure detected"))
    except PeerFailure as e:
        q.put((rank, f"peer failure: {e}"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}"))


def test_heartbeat_detects_dead_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = get_available_port()
    ps = [ctx.Process(target=_hb_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    rank, msg = q.get(timeout=60)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert rank == 0 and msg.startswith("peer failure: rank 1"), msg


def test_metrics_logger(tmp_path):
    from drivedit_b200.utils.observability import DeviceTimer, MetricsLogger, nvtx_range
    lg = MetricsLogger(str(tmp_path), config={"model": "tiny"})
    lg.log(1, {"loss": torch.tensor(0.5), "tok_s": 10.0})
    lg.close()
    import json
    rec = json.loads((tmp_path / "metrics.jsonl").read_text().splitlines()[0])
    assert rec["loss"] == 0.5 and rec["step"] == 1
    t = DeviceTimer()
    with nvtx_range("x"), t.time("x"):
        sum(range(1000))
    assert t.summary()["x"] >= 0
