"""Sharded checkpoints on 2 gloo ranks with expert parallelism: save after 2 steps, end
every process, resume in new processes and train 2 more steps -> bit-identical losses
and weights to 4 uninterrupted steps. Then consolidate the rank files into one
single-process state dict and export it in the reference's key layout."""
import os
import socket

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


def _cfg():
    from drivedit_b200.config.presets import Config, ModelConfig, MoEParams, TrainConfig

    m = ModelConfig(n_layers=2, d_model=32, n_heads=2, mlp_hidden=64, latent_channels=4,
                    latent_h=8, latent_w=8, moe=MoEParams(num_experts=4, top_k=2, expert_dim=32,
                                                          num_shared=1, aux_loss_weight=0.01))
    return Config(model=m, train=TrainConfig(batch_per_gpu=1, frames=2, lr=1e-2,
                                             parallel="fsdp_ep"))


def _worker(rank, world, port, q, ckdir, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from drivedit_b200.config import to_dict
    from drivedit_b200.data import make_batch
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.training.checkpoint import load_distributed, save_distributed
    from drivedit_b200.training.trainer import WorldModelTrainer

    cfg = _cfg()
    torch.manual_seed(0)
    tr = WorldModelTrainer(WorldDiT(cfg.model), cfg.train, "cpu", process_group=dist.group.WORLD)
    start, stop = {"full": (0, 4), "first": (0, 2), "resume": (2, 4)}[mode]
    if mode == "resume":
        assert load_distributed(tr, ckdir) == 2
    losses = []
    for step in range(start, stop):
        batch = make_batch(cfg, generator=torch.Generator().manual_seed(100 * step + rank))
        losses.append(float(tr.train_step(batch)))
    if mode == "first":
        save_distributed(tr, ckdir, 2, config=to_dict(cfg))
    sd = {k: v.detach().clone().numpy() for k, v in tr.model.state_dict().items()}
    q.put((rank, {"losses": losses, "sd": sd}))
    dist.destroy_process_group()


def _run(world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def test_resume_is_bit_identical_and_consolidates(tmp_path):
    ck = str(tmp_path / "ck")
    full = _run(2, ck, "full")
    _run(2, ck, "first")
    res = _run(2, ck, "resume")
    for r in range(2):
        assert res[r]["losses"] == full[r]["losses"][2:], (r, res[r]["losses"], full[r]["losses"])
        for k, v in full[r]["sd"].items():
            assert np.array_equal(res[r]["sd"][k], v), (r, k)
    # an interrupted save (no COMPLETE marker) is never picked up
    from drivedit_b200.training.checkpoint import consolidate, export_reference, latest_step

    (tmp_path / "ck" / "step_00000009").mkdir()
    assert latest_step(ck) == 2
    sd = consolidate(ck)
    w13 = [k for k in sd if k.endswith("moe.w13")]
    assert w13 and all(sd[k].shape[0] == 4 + 1 for k in w13)  # 4 routed + 1 shared
    assert not any(k.endswith("_shared") for k in sd)
    ref = export_reference(ck, str(tmp_path / "ref.pt"), _cfg().model)
    assert any(k.endswith("experts.3.w_gate.weight") for k in ref)
    assert any(k.endswith("shared_experts.0.w_out.weight") for k in ref)
