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


def test_core_encoders_memory_and_causal_dit():
    """The working counterparts of the reference's core sketch: encoders into the token
    space, the memory bank, and the causal DiT whose cached generation equals the
    full-sequence forward."""
    from drivedit_b200.core.base import (BaseEncoder, CausalDiT, ControlEncoder, DepthEncoder,
                                         MemoryBank, VAEEncoder)
    from drivedit_b200.core.components import create_attention_mask
    torch.manual_seed(0)
    cfg = DriveDiTConfig(latent_channels=4, latent_spatial_size=2, model_dim=32, n_heads=4,
                         n_layers=2, max_memory_frames=2, max_memory_objects=3, device="cpu",
                         dtype=torch.float32)
    vae = VAEEncoder(cfg)
    frames = torch.rand(1, 2, 3, 32, 32)
    tok = vae.encode(frames)
    assert isinstance(vae, BaseEncoder) and tok.shape == (1, 2, 4, 32) and vae.get_token_dim() == 32
    assert vae.decode(tok, (32, 32)).shape == (1, 2, 3, 32, 32)
    assert DepthEncoder(cfg).encode(torch.rand(1, 2, 1, 16, 16)).shape == (1, 2, 4, 32)
    assert ControlEncoder(cfg).encode(torch.randn(3, 6)).shape == (3, 1, 32)

    mem = MemoryBank(cfg)
    sp, ob = mem.get_memory_tokens()
    assert sp.shape == (1, 1, 32) and not sp.any()          # not full yet: one zero token
    for i in range(2):
        mem.update(torch.rand(1, 3, 16, 16), i)
    mem.add_objects(torch.randn(1, 32))
    sp, ob = mem.get_memory_tokens()
    assert sp.shape == (1, 2, 32) and ob.shape == (1, 1, 32)

    dit = CausalDiT(cfg).eval()
    x = torch.randn(1, 6, 32)
    with torch.no_grad():
        full, _ = dit(x, (sp, ob))
        dit.reset_cache()
        dit(x[:, :4], (sp, ob), use_cache=True)
        step, cache = dit(x[:, 4:], (sp, ob), use_cache=True)
    assert full.shape == (1, 4, 2, 2) and cache["layer_1"]["k"].shape[1] == 6
    torch.testing.assert_close(step, full, rtol=1e-4, atol=1e-5)

    m = create_attention_mask(3)
    assert m[0, 1] == float("-inf") and m[1, 0] == 0 and not create_attention_mask(2, False).any()
