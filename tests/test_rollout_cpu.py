"""Streaming rollout: the KV-cached chunked forward equals the full frame-causal forward,
the window truncation keeps positions absolute, and a rollout produces the right shapes."""
import torch

from drivedit_b200.config import get_config
from drivedit_b200.models.world_dit import KVCacheSet, WorldDiT, forward_cached
from drivedit_b200.inference.rollout import StreamingRollout


def _model(layers=2):
    torch.manual_seed(0)
    cfg = get_config("tiny", [f"model.n_layers={layers}"])
    m = WorldDiT(cfg.model)
    with torch.no_grad():
        for p in m.parameters():
            if p.abs().sum() == 0:
                p.normal_(0, 0.02)
    return cfg, m


def test_cached_chunks_equal_full_forward():
    cfg, m = _model()
    B, Fr = 2, 4
    x = torch.randn(B, Fr, 16, 16, 16)
    t = torch.rand(B)
    a = torch.rand(B, Fr, 2)
    full = m(x, t, a)
    cache = KVCacheSet(m, B, window_frames=8, chunk_frames=2, device="cpu", dtype=torch.float32)
    outs = []
    for f0 in (0, 2):
        outs.append(forward_cached(m, x[:, f0:f0 + 2], t, a[:, f0:f0 + 2], cache, commit=True))
    assert torch.allclose(torch.cat(outs, 1), full, atol=1e-4)


def test_window_truncation_matches_windowed_reference():
    # one layer: cached K/V of a frame depend only on that frame's own tokens
    cfg, m = _model(layers=1)
    B = 1
    x = torch.randn(B, 6, 16, 16, 16)
    t = torch.rand(B)
    a = torch.rand(B, 6, 2)
    cache = KVCacheSet(m, B, window_frames=2, chunk_frames=2, device="cpu", dtype=torch.float32)
    for f0 in (0, 2, 4):
        last = forward_cached(m, x[:, f0:f0 + 2], t, a[:, f0:f0 + 2], cache, commit=True)
    # reference: frames 2..5 through a fresh cache, but rotary positions must stay absolute,
    # so compare against a cache that starts at frame 2 with the same absolute offset
    ref_cache = KVCacheSet(m, B, window_frames=2, chunk_frames=2, device="cpu", dtype=torch.float32)
    ref_cache.frames = 2
    forward_cached(m, x[:, 2:4], t, a[:, 2:4], ref_cache, commit=True)
    ref = forward_cached(m, x[:, 4:6], t, a[:, 4:6], ref_cache, commit=True)
    assert torch.allclose(last, ref, atol=1e-4)


def test_rollout_shapes_and_latencies():
    cfg, m = _model()
    cfg.rollout.total_frames = 8
    cfg.rollout.chunk_frames = 2
    cfg.rollout.flow_steps = 2
    cfg.rollout.window_frames = 4
    r = StreamingRollout(m, cfg.rollout)
    ctx = torch.randn(2, 2, 16, 16, 16)
    act = torch.rand(2, 8, 2)
    res = r.run(ctx, act, generator=torch.Generator().manual_seed(0))
    assert res.frames.shape == (2, 8, 16, 16, 16)
    assert len(res.chunk_ms) == 3
    assert torch.isfinite(res.frames).all()
