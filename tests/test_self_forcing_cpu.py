"""Self-Forcing++ pieces and the trainer step (CPU)."""
import math

import torch
import torch.nn as nn

from drivedit_b200.training.self_forcing import (CurriculumScheduler, EMAModel, ExtendedControlEncoder,
                                                 FutureAnchorEncoder, PerLayerGradientClipper,
                                                 RollingKVCache, SelfForcingPlusConfig,
                                                 SelfForcingPlusTrainer, UncertaintyWeighting,
                                                 get_minimal_config)


def test_rolling_kv_cache_truncates_and_detaches():
    c = RollingKVCache(max_length=32, truncate_to=16, detach_interval=4)
    for i in range(10):
        k = torch.randn(2, 4, 8, 64, requires_grad=True)
        fk, fv = c.update(0, k, k * 2)
    assert fk.shape[1] <= 32 and c.get_length() == fk.shape[1]
    assert c.get_memory_usage() > 0
    c.reset()
    assert c.get_cache(0) is None


def test_curriculum_schedules():
    cfg = SelfForcingPlusConfig(initial_sequence_length=8, final_sequence_length=64,
                                sequence_curriculum_steps=100, self_forcing_warmup_steps=100,
                                curriculum_warmup_steps=100)
    s = CurriculumScheduler(cfg)
    assert s.get_sequence_length() == 8 and s.get_self_forcing_ratio() == 0.0
    s.update(50)
    assert s.get_sequence_length() == 8 + int(0.5 * 56)
    assert abs(s.get_self_forcing_ratio() - 0.5) < 1e-12
    assert s.get_curriculum_weights()["future_anchor"] == (0.5 - 0.3) / 0.7
    s.update(1000)
    assert s.get_sequence_length() == 64 and s.get_self_forcing_ratio() == 1.0


def test_control_and_anchor_encoders():
    cfg = SelfForcingPlusConfig(model_dim=32, control_hidden_dim=16)
    enc = ExtendedControlEncoder(cfg)
    raw = torch.tensor([[0.5, 10.0, 0.0, 25.0, 20.0, -2.0]])
    n = enc.normalize(raw)
    assert torch.allclose(n, torch.tensor([[0.5, 1.0, 0.0, 0.5, 0.0, -1.0]]), atol=1e-6)
    assert torch.allclose(enc.denormalize(n)[0, :2], torch.tensor([0.5, 5.0]))
    assert enc(torch.randn(2, 5, 6)).shape == (2, 5, 32)
    fa = FutureAnchorEncoder(cfg)
    assert fa.get_anchor_indices(0, 50) == [20, 40, 49]
    assert fa(torch.randn(2, 50, 5)).shape == (2, 32)


def test_ema_flat_matches_named():
    from drivedit_b200.parallel.flat import FlatParamGroup
    torch.manual_seed(0)
    a = nn.Linear(4, 3)
    b = nn.Linear(4, 3)
    b.load_state_dict(a.state_dict())
    g = FlatParamGroup(b.named_parameters(), "cpu")
    ea, eb = EMAModel(a, 0.9), EMAModel(b, 0.9, group=g)
    with torch.no_grad():
        for p, q in zip(a.parameters(), b.parameters()):
            p.add_(1.0)
            q.add_(1.0)
    ea.update(a)
    eb.update(b)
    for n in ea.shadow:
        assert torch.allclose(ea.shadow[n], eb.shadow[n])
    eb.apply_shadow(b)
    assert torch.allclose(b.weight, ea.shadow["weight"])
    eb.restore(b)
    assert torch.allclose(b.weight, a.weight)


def test_uncertainty_weighting_and_clipper():
    uw = UncertaintyWeighting(["a", "b"])
    total, w = uw({"a": torch.tensor(2.0)})
    assert torch.allclose(total, torch.tensor(1.0)) and float(w["a"]) == 1.0
    m = nn.Sequential(nn.Linear(4, 4), nn.Linear(4, 4))
    for p in m.parameters():
        p.grad = torch.ones_like(p) * 10
    clip = PerLayerGradientClipper(m, default_max_norm=1.0, layer_configs={"1.": 0.5})
    norms = clip.clip_gradients()
    assert float(norms["0.weight"]) == 40.0
    assert abs(float(m[0].weight.grad.norm()) - 1.0) < 1e-4
    assert abs(float(m[1].weight.grad.norm()) - 0.5) < 1e-4


def test_trainer_step_with_self_generated_context():
    from drivedit_b200.config import get_config
    from drivedit_b200.models.world_dit import WorldDiT
    torch.manual_seed(0)
    cfg = get_config("tiny", ["model.n_layers=2"])
    sc = get_minimal_config()
    sc.initial_sequence_length = sc.final_sequence_length = 12
    sc.self_forcing_warmup_steps = 1
    sc.flow_steps = 2
    tr = SelfForcingPlusTrainer(WorldDiT(cfg.model), sc, device="cpu")
    batch = {"frames": torch.randn(2, 12, 16, 16, 16), "controls": torch.randn(2, 12, 6),
             "ego_states": torch.randn(2, 12, 5)}
    w0 = tr.model.blocks[0].attn.qkv.weight.detach().clone()
    o1 = tr.train_step(batch)
    o2 = tr.train_step(batch)  # sf_ratio = 1: every non-context chunk before the loss chunk
    assert o2["sf_ratio"] == 1.0
    assert o2["self_generated_chunks"] == (o2["loss_chunk_start"] - sc.context_frames) // sc.chunk_frames
    assert torch.isfinite(o2["total_loss"]) and not torch.equal(w0, tr.model.blocks[0].attn.qkv.weight)
    sd = tr.state_dict()
    tr.load_state_dict(sd)
