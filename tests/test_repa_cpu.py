"""REPA alignment + HASTE schedule + frozen V-JEPA teacher (CPU)."""
import math

import torch
import torch.nn.functional as F

from drivedit_b200.models.vjepa import VJEPABackbone, VJEPAConfig, create_vjepa_backbone
from drivedit_b200.training.repa import (HASTEScheduler, REPAConfig, REPALoss, _pool_to,
                                         create_repa_loss)


def test_haste_schedule_phases():
    cfg = REPAConfig(total_training_steps=1000, haste_warmup_ratio=0.1, haste_termination_ratio=0.4)
    h = HASTEScheduler(cfg)
    assert h.get_weight(0) == 0.0
    assert abs(h.get_weight(50) - 0.5 * (1 - math.cos(math.pi * 0.5))) < 1e-12
    assert h.get_weight(200) == 1.0 and h.get_phase() == "active"
    assert h.get_weight(400) == 0.0 and h.get_phase() == "terminated"
    assert HASTEScheduler(REPAConfig(enable_haste=False)).get_weight(10 ** 6) == 1.0


def test_repa_loss_pooling_and_weights():
    torch.manual_seed(0)
    loss = create_repa_loss(64, 32, dit_layers=[1, 2], vjepa_layers=[3, 4], total_training_steps=10,
                            haste_termination_ratio=1.0, haste_warmup_ratio=0.0)
    dit = {"layer_1": torch.randn(2, 16, 64), "layer_2": torch.randn(2, 16, 64)}
    tea = {"layer_3": torch.randn(2, 8, 32), "layer_4": torch.randn(2, 8, 32)}
    out = loss(dit, tea, step=5)
    assert set(out["per_layer_losses"]) == {"layer_1", "layer_2"}
    assert torch.allclose(out["total_repa_loss"], out["raw_repa_loss"] * 0.1)
    x = torch.randn(2, 12, 5)
    assert torch.allclose(_pool_to(x, 4), F.adaptive_avg_pool1d(x.transpose(1, 2), 4).transpose(1, 2))
    assert loss.get_loss_stats()["repa_current"] == float(out["total_repa_loss"])
    # identical (normalised) features -> zero cosine loss
    from drivedit_b200.training.repa import alignment_loss
    f = torch.randn(2, 8, 32)
    assert alignment_loss(f, f * 3.0).abs() < 1e-6


def test_teacher_shapes_and_frozen():
    torch.manual_seed(1)
    cfg = VJEPAConfig(embed_dim=128, num_layers=3, num_heads=2, num_frames=4, image_size=(32, 64),
                      extract_layers=[1, 2])
    t = VJEPABackbone(cfg)
    assert not any(p.requires_grad for p in t.parameters())
    out = t(torch.rand(2, 4, 3, 32, 64))
    assert out["patch_features"].shape == (2, 2 * 2 * 4, 128)
    assert set(out["intermediate"]) == {"layer_1", "layer_2"}
    part = t(torch.rand(2, 4, 3, 32, 64), max_layer=1)
    assert set(part["intermediate"]) == {"layer_1"}
    assert create_vjepa_backbone("base", pretrained=False).config.embed_dim == 768


def test_world_model_repa_step_reduces_alignment_loss():
    from drivedit_b200.config import REPAParams, get_config
    from drivedit_b200.data.synthetic import make_batch
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.training.trainer import WorldModelTrainer

    cfg = get_config("tiny", ["train.lr=1e-3"])
    cfg.model.repa = REPAParams(layer=2, teacher_layers=2, teacher_dim=256, teacher_heads=4,
                                teacher_patch=16, image_h=32, image_w=64)
    torch.manual_seed(0)
    tr = WorldModelTrainer(WorldDiT(cfg.model), cfg.train, device="cpu")
    b = make_batch(cfg, rgb_frames=cfg.train.frames)
    first = None
    for _ in range(5):
        tr.train_step(b)
        first = first if first is not None else float(tr.last_losses["repa"])
    assert float(tr.last_losses["repa"]) < first
