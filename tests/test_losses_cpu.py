"""v1 and v2 training losses (CPU)."""
import torch

from drivedit_b200.training.losses import FlowMatchingLoss, ReconstructionLoss, TemporalConsistencyLoss, UnifiedLoss
from drivedit_b200.training.losses_v2 import (GradientSurgery, LossAggregator, LossConfig, LossType,
                                              ScaleInvariantDepthLoss, VICRegLoss, create_full_loss_config)


def test_unified_loss_v1():
    class C:
        enable_flow_matching = True
        enable_curriculum = True
        curriculum_warmup_steps = 100
    torch.manual_seed(0)
    f = torch.rand(2, 4, 3, 8, 8)
    p = (f + 0.1).requires_grad_(True)
    L = UnifiedLoss(C())
    out = L({"predictions": p, "flow_predictions": torch.zeros_like(f),
             "jepa_predictions": torch.randn(2, 2, 16), "hidden_states": torch.randn(2, 5, 16)},
            {"frames": f}, step=50)
    assert {"reconstruction", "l1", "perceptual", "temporal_consistency", "flow_matching", "jepa", "total"} <= set(out)
    assert abs(float(out["reconstruction"]) - 0.01) < 1e-5 and float(out["temporal_consistency"]) < 1e-10
    out["total"].backward()
    assert p.grad is not None and L.get_loss_stats()["total_current"] == float(out["total"])
    z0, z1 = torch.randn(3, 5), torch.randn(3, 5)
    assert FlowMatchingLoss.rectified_flow_loss(z1 - z0, z0, z1) == 0
    assert float(FlowMatchingLoss.velocity_matching_loss(z0, z1, torch.rand(3), "truncated_snr")) > 0
    assert ReconstructionLoss.gradient_loss(f, f) == 0 and float(ReconstructionLoss.multi_scale_loss(f, f)) == 0
    lin = torch.linspace(0, 1, 6).view(1, 6, 1)
    assert float(TemporalConsistencyLoss.smoothness_loss(lin)) < 1e-12


def test_loss_aggregator_all_types():
    torch.manual_seed(0)
    B, T = 2, 4
    frames = torch.rand(B, T, 3, 32, 32)
    preds = {"latents": torch.randn(B, T, 16, 4, 4, requires_grad=True),
             "predictions": frames.clone().requires_grad_(True), "flow_predictions": torch.randn(B, T, 16, 4, 4),
             "hidden_states": torch.randn(B, T, 32), "hidden_states_aug": torch.randn(B, T, 32),
             "control_features": torch.randn(B, 32), "depth_features": torch.randn(B, 32),
             "depth_predictions": torch.rand(B, T, 1, 32, 32) * 10 + 0.5, "predicted_actions": torch.rand(B, T, 6) * 2 - 1,
             "trajectory": torch.randn(5, B, 8), "kv_cache_history": [{"k": torch.randn(1, 4, 8), "v": torch.randn(1, 4, 8)},
                                                                      {"k": torch.randn(1, 5, 8), "v": torch.randn(1, 5, 8)}]}
    tg = {"latents": torch.randn(B, T, 16, 4, 4), "frames": frames, "noise": torch.randn(B, T, 16, 4, 4),
          "teacher_flow": torch.randn(B, T, 16, 4, 4), "teacher_trajectory": torch.randn(3, B, T, 16, 4, 4),
          "depth": torch.rand(B, T, 1, 32, 32) * 10 + 0.5, "controls": torch.rand(B, T, 6), "goals": torch.randn(B, 2)}
    cfg = create_full_loss_config()
    agg = LossAggregator(cfg)
    out = agg(preds, tg, step=cfg.curriculum_warmup_steps)
    assert len(out) == len(LossType) + 1 and torch.isfinite(out["total"])
    assert float(out["temporal_consistency"]) == 0.0  # prediction == target frames
    out["total"].backward()
    assert preds["latents"].grad is not None
    assert set(agg.get_loss_stats()) == {t.value for t in LossType}
    assert agg.get_curriculum_progress()["infonce"] == 1.0


def test_individual_losses():
    d = torch.rand(2, 1, 8, 8) + 0.5
    assert float(ScaleInvariantDepthLoss(lambda_scale=1.0)({"depth_predictions": d * 3}, {"depth": d})) < 1e-6  # lam=1: scale invariant
    a = torch.randn(64, 16)
    v = VICRegLoss()({"hidden_states": a, "hidden_states_aug": a}, {})
    assert torch.isfinite(v)
    g1, g2 = torch.tensor([1.0, 0.0]), torch.tensor([-1.0, 1.0])
    c = GradientSurgery.project_conflicting_gradients([g1, g2])
    assert float(c @ g1) >= -1e-6 and float(c @ g2) >= -1e-6
    agg = LossAggregator(LossConfig(enabled_losses=[LossType.LATENT_MSE, LossType.CONDITIONAL_FLOW_MATCHING],
                                    use_gradient_surgery=True, enable_curriculum=False))
    w = torch.randn(4, requires_grad=True)
    pr = {"latents": w * 2, "flow_predictions": w}
    out = agg(pr, {"latents": torch.zeros(4), "noise": torch.zeros(4)})
    agg.apply_gradient_surgery(out, [w])
    assert w.grad is not None and w.grad.shape == (4,)


def test_reference_loss_parameters():
    """The reference's constructor parameters carry their meaning."""
    from drivedit_b200.training.losses_v2 import (BoundaryActionClippingLoss, InfoNCELoss,
                                                  MultiScaleDepthLoss, SceneStabilityLoss,
                                                  TemporalContrastiveLoss, VICRegLoss)
    torch.manual_seed(0)
    h = torch.randn(4, 6, 16)
    for hard in (False, True):
        assert float(InfoNCELoss(1.0, 0.1, 2, hard)({"hidden_states": h}, {})) > 0
    assert float(TemporalContrastiveLoss(1.0, 0.1, 1, 3)({"hidden_states": h}, {})) > 0
    a = torch.tensor([[[1.5, 0.0]]])
    assert float(BoundaryActionClippingLoss(1.0, 1.0, (0.0, 2.0))({"predicted_actions": a}, {})) == 0.0
    assert float(BoundaryActionClippingLoss(1.0, 1.0, (-1.0, 1.0))({"predicted_actions": a}, {})) > 0.0
    d = torch.rand(2, 1, 16, 16) + 0.5
    # a constant log offset c costs (1 - lambda) c^2 per scale, weighted 1/scale
    import math
    expect = 0.5 * math.log(2.0) ** 2 * (1 + 1 / 2)
    assert abs(float(MultiScaleDepthLoss(1.0, (1, 2), True)({"depth_predictions": d * 2}, {"depth": d})) - expect) < 1e-4
    v = torch.rand(1, 3, 3, 16, 16)
    still = v[:, :1].expand(-1, 3, -1, -1, -1)
    assert float(SceneStabilityLoss(1.0, 0.1)({"predictions": still}, {"frames": still})) == 0.0
    assert float(VICRegLoss(1.0, variance_target=0.0)({"hidden_states": h, "hidden_states_aug": h}, {})) >= 0
