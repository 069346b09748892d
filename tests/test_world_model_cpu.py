"""CPU slice: the tiny flow-matching world model trains (fwd + bwd + AdamW) in fp32."""
import math

import torch

from drivedit_b200.config import get_config
from drivedit_b200.data import make_batch
from drivedit_b200.models.world_dit import WorldDiT, patchify, unpatchify
from drivedit_b200.training.trainer import WorldModelTrainer


def test_patchify_roundtrip():
    x = torch.randn(2, 3, 16, 8, 12)
    t = patchify(x, 2)
    assert t.shape == (2, 3 * 4 * 6, 64)
    assert torch.equal(unpatchify(t, 3, 16, 8, 12, 2), x)


def test_tiny_config_shapes_and_params():
    cfg = get_config("tiny")
    m = WorldDiT(cfg.model)
    b = make_batch(cfg)
    v = m(b.latents, torch.rand(2), b.actions)
    assert v.shape == b.latents.shape
    n = sum(p.numel() for p in m.parameters())
    assert 5e6 < n < 6e6


def test_tiny_training_step_reduces_loss():
    torch.manual_seed(0)
    cfg = get_config("tiny", ["train.lr=1e-3"])
    m = WorldDiT(cfg.model)
    tr = WorldModelTrainer(m, cfg.train)
    b = make_batch(cfg, generator=torch.Generator().manual_seed(0))
    losses = []
    for _ in range(12):
        tr.gen.manual_seed(5)  # same noise and flow time every step: overfit one batch
        losses.append(float(tr.train_step(b)))
    assert all(math.isfinite(l) for l in losses)
    assert sum(losses[-3:]) / 3 < sum(losses[:3]) / 3


def test_frame_causality():
    """Changing frame f must not change the prediction for frames < f."""
    torch.manual_seed(0)
    cfg = get_config("tiny")
    m = WorldDiT(cfg.model)
    with torch.no_grad():
        for p in m.parameters():
            if p.abs().sum() == 0:
                p.normal_(0, 0.02)
    b = make_batch(cfg)
    t = torch.rand(2)
    v1 = m(b.latents, t, b.actions)
    lat = b.latents.clone()
    lat[:, 2:] += 1.0
    v2 = m(lat, t, b.actions)
    assert torch.allclose(v1[:, :2], v2[:, :2], atol=1e-5)
    assert not torch.allclose(v1[:, 2:], v2[:, 2:], atol=1e-3)
