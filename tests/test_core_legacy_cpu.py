"""Earlier-generation components and the end-to-end system facade (CPU)."""
import torch

from drivedit_b200.core.base import DriveDiTConfig, DriveDiTSystem, TensorCache
from drivedit_b200.core.components import (AdaptiveLayerNorm, CausalVideoTransformer, FlowMatchingPredictor,
                                           MultiHeadAttention, RoPE3D, SAM2InspiredTracker)


def test_causal_transformer_cache_matches_full_sequence():
    torch.manual_seed(0)
    m = CausalVideoTransformer(dim=32, num_layers=2, num_heads=4, dropout=0.0).eval()
    x = torch.randn(2, 7, 32)
    full, _ = m(x)
    a, cache = m(x[:, :4], use_cache=True)
    b, _ = m(x[:, 4:], past_kvs=cache, use_cache=True)
    torch.testing.assert_close(torch.cat([a, b], 1), full, rtol=1e-4, atol=1e-5)


def test_rope_tables_and_components():
    sin, cos = RoPE3D(12)(2, 3, 4)
    assert sin.shape == (2, 3, 4, 12)
    assert torch.allclose(sin[0, 0, 0], torch.zeros(12)) and torch.allclose(cos[0, 0, 0], torch.ones(12))
    attn = MultiHeadAttention(32, 4, dropout=0.0)
    out, _ = attn(torch.randn(1, 24, 32), grid=(2, 3, 4))
    assert out.shape == (1, 24, 32)
    tr = SAM2InspiredTracker(dim=32, max_objects=5)
    feats = tr.encode_objects(torch.rand(2, 3, 3, 32, 32))
    assert tr.update_memory(feats, 0).shape == (2, 5, 32)
    ln = AdaptiveLayerNorm(16, 8)
    x = torch.randn(2, 5, 16)
    torch.testing.assert_close(ln(x, torch.randn(2, 8)), torch.nn.functional.layer_norm(x, (16,)))
    fp = FlowMatchingPredictor(16)
    assert fp.sample(torch.randn(3, 16)).shape == (3, 16)
    c = TensorCache(3)
    for i in range(5):
        c.append(torch.full((2, 4), float(i)))
    assert c.get_recent(2)[0, :, 0].tolist() == [3.0, 4.0] and c.get_recent(4) is None


def test_system_trains_and_generates():
    torch.manual_seed(0)
    cfg = DriveDiTConfig(latent_channels=4, model_dim=64, n_heads=2, n_layers=2, context_length=2,
                         image_size=32, device="cpu", flow_matching_steps=2, control_dim=3)
    sysm = DriveDiTSystem(cfg)
    frames = torch.rand(1, 4, 3, 32, 32)
    controls = torch.rand(1, 4, 3)
    out = sysm(frames, controls)
    out["loss"].backward()
    assert torch.isfinite(out["loss"]) and out["latents"].shape[1] == 4
    gen = sysm(frames, controls, mode="inference", horizon=2)
    assert gen["frames"].shape == (1, 2, 3, 32, 32) and gen["latents"].shape[1] == 2
