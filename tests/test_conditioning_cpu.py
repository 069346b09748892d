"""Rich conditioning encoders and their integration (shapes, masks, CFG dropout)."""
import torch

from drivedit_b200.models.conditioning import (ConditioningConfig, ConditioningIntegration,
                                               create_conditioning_module, normalize_intrinsics,
                                               rotation_matrix_to_6d)


def _inputs(B=3, N=6, W=10, O=5):
    K = torch.tensor([[500.0, 0, 256], [0, 500, 128], [0, 0, 1]]).expand(B, N, 3, 3)
    ext = torch.cat([torch.eye(3).expand(B, N, 3, 3), torch.randn(B, N, 3, 1)], -1)
    cam = {"intrinsics": K, "extrinsics": ext}
    road = {"waypoints": torch.randn(B, W, 6), "road_type": torch.randint(0, 8, (B,)),
            "lane_info": torch.randn(B, 3), "turn_info": torch.randn(B, 5),
            "waypoint_mask": torch.arange(W)[None].expand(B, W) < 7}
    mask = torch.ones(B, O, dtype=torch.bool)
    mask[0] = False
    bbox = {"positions": torch.randn(B, O, 3) * 10, "dimensions": torch.rand(B, O, 3),
            "headings": torch.randn(B, O), "velocities": torch.randn(B, O, 3),
            "object_classes": torch.randint(0, 11, (B, O)), "confidences": torch.rand(B, O),
            "object_mask": mask}
    ego = {"position": torch.randn(B, 3), "velocity": torch.randn(B, 3),
           "acceleration": torch.randn(B, 3), "heading": torch.randn(B),
           "heading_rate": torch.randn(B), "gps": torch.randn(B, 3), "imu": torch.randn(B, 6)}
    temporal = {"time_of_day": torch.rand(B) * 24, "weather": torch.randint(0, 8, (B,)),
                "season": torch.randint(0, 4, (B,))}
    return cam, road, bbox, ego, temporal


def test_integration_shapes_and_grad():
    torch.manual_seed(0)
    m = create_conditioning_module(model_dim=64, cond_dim=32, dropout=0.0).eval()
    out = m(*_inputs())
    assert out["conditioning"].shape == (3, 32)
    assert len(out["adaln_params"]) == 6 and out["adaln_params"][0].shape == (3, 64)
    assert out["road_context"].shape == (3, 10, 64)
    assert out["object_tokens"].shape == (3, 5, 64)
    assert out["modality_mask"].all()
    assert torch.isfinite(out["object_tokens"]).all()
    out["conditioning"].sum().backward()
    assert m.camera_encoder.proj[0].weight.grad is not None


def test_missing_modalities_and_cfg_dropout():
    torch.manual_seed(1)
    cfg = ConditioningConfig(model_dim=64, cond_dim=32, cfg_dropout_prob=1.0, dropout=0.0)
    m = ConditioningIntegration(cfg)
    cam, road, bbox, ego, temporal = _inputs()
    m.train()
    dropped = m(cam, road, bbox, ego, temporal)["conditioning"]
    m.eval()
    null = m.get_null_conditioning(3, "cpu")["conditioning"]
    assert torch.allclose(dropped, null, atol=1e-6)
    only_ego = m(ego_data=ego)
    assert only_ego["modality_mask"].tolist() == [[False, False, False, True, False]] * 3
    assert only_ego["road_context"] is None
    c, u = torch.randn(4), torch.randn(4)
    assert torch.allclose(ConditioningIntegration.apply_cfg(c, u, 1.0), c)


def test_geometry_helpers():
    K = torch.tensor([[100.0, 0, 50], [0, 80, 40], [0, 0, 1]])
    Kn = normalize_intrinsics(K, (80, 100))
    assert torch.allclose(Kn[0, 0], torch.tensor(1.0)) and torch.allclose(Kn[1, 2], torch.tensor(0.5))
    R = torch.eye(3)
    assert rotation_matrix_to_6d(R).tolist() == [1, 0, 0, 0, 1, 0]
