"""Reference-compatible config objects and the component-toggled WorldModel (CPU)."""
import torch

from drivedit_b200.config.base import get_config_diff, merge_configs
from drivedit_b200.config.model_config import DiTConfig, ModelConfig, get_large_config, get_small_config
from drivedit_b200.config.unified import (ComponentType as C, DriveDiTConfig, get_config, list_configs)
from drivedit_b200.models.world_model import WorldModel


def _cfg(components, **kw):
    c = DriveDiTConfig(model_dim=64, num_layers=2, num_heads=4, image_size=32, patch_size=16,
                       sequence_length=4, final_sequence_length=8, memory_dim=64,
                       jepa_prediction_head_dim=32, enabled_components=list(components), **kw)
    c.repa_config.alignment_layers = [1]
    c.causal_jepa_config.slot_dim = 32
    c.causal_jepa_config.max_objects = 4
    c.moe_config.num_experts = 4
    c.moe_config.expert_dim = 64
    return c


def test_config_presets_json_round_trip_and_components():
    assert list_configs() == ["minimal", "research", "production", "video_only", "flow_matching"]
    r = get_config("research")
    assert r.is_component_enabled(C.SLA) and not r.is_component_enabled(C.MOE)
    r.enable_component(C.MOE)
    r.disable_component(C.DEPTH)
    back = DriveDiTConfig.from_json(r.to_json())
    assert back.enabled_components == r.enabled_components
    assert back.moe_config.num_experts == r.moe_config.num_experts
    assert get_config_diff(r, back) == {}
    assert r.moe_num_experts == 8 and r.repa_feature_layers == [6, 12, 18]
    wc = r.to_world_config()
    assert wc.model.attention == "sla" and wc.model.moe is not None and wc.model.d_model == 768
    m = get_small_config()
    assert m.student.latent_dim == m.vae.latent_dim == 4 and not m.teacher.causal
    assert get_large_config().student.gradient_checkpointing
    merged = merge_configs(DiTConfig(), DiTConfig(d_model=512, n_heads=8))
    assert merged.d_model == 512 and merged.d_ff == (int(8 * 512 / 3) + 7) // 8 * 8
    assert ModelConfig.from_json(get_small_config().to_json()).image_size == (128, 128)


def test_world_model_modes_and_heads():
    torch.manual_seed(0)
    cfg = _cfg([C.CONTROL, C.DEPTH, C.MEMORY, C.JEPA, C.FLOW_MATCHING, C.REPA, C.CAUSAL_JEPA])
    m = WorldModel(cfg)
    x = torch.rand(2, 4, 3, 32, 32)
    ctl, dep = torch.randn(2, 4, 6), torch.rand(2, 4, 1, 32, 32) * 50
    out = m(x, ctl, dep)
    assert out["predictions"].shape == (2, 4, 3, 32, 32)
    assert out["hidden_states"].shape == (2, 16, 64)
    assert set(out["repa_projections"]) == {1}
    (out["predictions"].mean() + out["jepa_predictions"].pow(2).mean()
     + out["flow_predictions"].pow(2).mean()).backward()
    assert m.control_encoder.encoder[0].weight.grad.abs().sum() > 0   # context reaches frames
    assert m(x, ctl, dep, mode="sla")["attention_mode"] == "sla"
    sf = m(x, ctl, dep, mode="self_forcing", self_forcing_ratio=1.0)
    assert sf["predictions"].shape == (2, 2, 3, 32, 32)
    assert m(x, mode="cjepa")["cjepa_slots"].shape[-1] == 32
    assert set(m.get_component_status()["active"]) >= {"control", "depth", "memory", "repa", "causal_jepa"}


def test_world_model_cached_inference_matches_full_forward():
    torch.manual_seed(0)
    m = WorldModel(_cfg([C.FLOW_MATCHING])).eval()
    x = torch.rand(1, 3, 3, 32, 32)
    gen = m(x, mode="inference", num_steps=3)["generated_frames"]
    full = m(torch.cat([x, gen[:, :2]], 1))["predictions"]
    torch.testing.assert_close(gen[:, 1:2], full[:, 3:4], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(gen[:, 2:3], full[:, 4:5], rtol=1e-4, atol=1e-5)


def test_world_model_moe_and_rich_conditioning():
    torch.manual_seed(0)
    m = WorldModel(_cfg([C.MOE, C.RICH_CONDITIONING]))
    ego = {"position": torch.randn(2, 3), "velocity": torch.randn(2, 3), "acceleration": torch.randn(2, 3),
           "heading": torch.randn(2), "heading_rate": torch.randn(2)}
    x = torch.rand(2, 4, 3, 32, 32)
    out = m(x, mode="rich_cond", ego_data=ego)
    assert out["conditioning"].shape == (2, 64)
    assert m.get_moe_aux_loss() is not None
    # the conditioning modulates the blocks: another ego state changes the prediction
    for blk in m.backbone:                     # AdaLN starts at identity; open it
        torch.nn.init.normal_(blk.norm_attn.cond_proj.weight, std=0.1)
    a = m(x, mode="rich_cond", ego_data=ego)["predictions"]
    ego2 = {k: v + 1.0 for k, v in ego.items()}
    b = m(x, mode="rich_cond", ego_data=ego2)["predictions"]
    assert (a - b).abs().max() > 1e-6
