"""Gradient buckets of the overlapped reduce-scatter (``ShardedDataParallel._plan_pieces``):
for every world size the ranks' pieces partition the flat buffer exactly, every piece is
16-byte aligned, each block's weights form one bucket, and every rank plans the same
buckets (they take the same barriers)."""
import pytest
import torch


def _engine(world, rank, flat):
    from drivedit_b200.parallel.sharded import ShardedDataParallel
    eng = ShardedDataParallel.__new__(ShardedDataParallel)
    eng.world, eng.rank, eng.flat = world, rank, flat
    return eng


@pytest.mark.parametrize("world", [2, 3, 8])
def test_pieces_partition_the_flat_buffer(world):
    from drivedit_b200.config import get_config
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.parallel.flat import FlatParamGroup
    cfg = get_config("tiny", ["model.attention=sla"])
    m = WorldDiT(cfg.model)
    flat = FlatParamGroup(m.flat_layout(m.named_parameters()), "cpu", no_decay=m.no_decay_names(),
                          pad_to=world * 4)
    cover = torch.zeros(flat.numel, dtype=torch.int32)
    ids = None
    for r in range(world):
        eng = _engine(world, r, flat)
        pieces = eng._plan_pieces()
        assert pieces is not None
        ids = eng.bucket_ids if ids is None else ids
        assert eng.bucket_ids == ids == set(range(cfg.model.n_layers))
        off = 0
        for lo, hi, loc, b in pieces:
            assert lo % 4 == 0 and hi % 4 == 0 and hi > lo and loc == off
            off += hi - lo
            cover[lo:hi] += 1
    assert torch.equal(cover, torch.ones_like(cover))
    # a block's bucket holds its GEMM weights
    eng = _engine(world, 0, flat)
    eng._plan_pieces()
    o, k = flat.offsets["blocks.1.mlp.w13.weight"]
    runs = {}
    for r in range(world):
        for lo, hi, _, b in _engine(world, r, flat)._plan_pieces():
            if b is not None:
                runs.setdefault(b, [lo, hi])
                runs[b] = [min(runs[b][0], lo), max(runs[b][1], hi)]
    assert runs[1][0] <= o and o + k <= runs[1][1]
