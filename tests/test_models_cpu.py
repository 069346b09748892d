"""Reference-API models on CPU: DiTStudent KV-cache consistency, DiTTeacher flow sampling,
DiTBlock variants, FlowPredictor."""
import torch

from drivedit_b200.models.blocks import (DiTBlock, DiTBlockWithCrossAttention, FlowPredictor,
                                         MemoryEfficientDiTBlock)
from drivedit_b200.models.dit_student import DiTStudent, DiTTeacher


def test_student_cache_matches_full_forward():
    torch.manual_seed(0)
    m = DiTStudent(latent_dim=8, d_model=64, n_layers=2, n_heads=4, use_memory=False).eval()
    x = torch.randn(2, 10, 8)
    full, _ = m(x)
    out1, cache = m(x[:, :6], use_cache=True)
    out2, cache = m(x[:, 6:], kv_cache=cache, use_cache=True)
    assert torch.allclose(torch.cat([out1, out2], 1), full, atol=1e-5)


def test_student_generate_and_loss():
    torch.manual_seed(0)
    m = DiTStudent(latent_dim=8, d_model=64, n_layers=2, n_heads=4, memory_size=16).eval()
    seq = m.generate(torch.randn(1, 4, 8), max_new_tokens=5, temperature=0.1)
    assert seq.shape == (1, 9, 8)
    loss = m.compute_loss(torch.randn(2, 5, 8), torch.randn(2, 5, 8))
    assert loss.item() > 0


def test_teacher_sample_and_distill():
    torch.manual_seed(0)
    t = DiTTeacher(latent_dim=8, d_model=64, n_layers=2, n_heads=4, num_steps=4)
    x1 = torch.randn(2, 6, 8)
    assert t.compute_loss(x1).item() > 0
    s = t.sample((2, 6, 8))
    assert s.shape == (2, 6, 8) and torch.isfinite(s).all()


def test_block_variants():
    torch.manual_seed(0)
    x = torch.randn(2, 8, 32)
    b = DiTBlock(32, 4, cond_dim=16)
    y, _ = b(x, cond=torch.randn(2, 16))
    assert y.shape == x.shape
    c = DiTBlockWithCrossAttention(32, 4, context_dim=24)
    ctx = torch.randn(2, 5, 24)
    y, _, cross = c(x, context=ctx)
    assert y.shape == x.shape and cross["k"].shape == (2, 5, 4, 8)
    y2, _, _ = c(x, cross_kv_cache=cross)          # projected context reused
    torch.testing.assert_close(y2, y)
    from drivedit_b200.models.blocks import create_dit_block
    assert isinstance(create_dit_block(32, 4, "cross_attn", context_dim=24), DiTBlockWithCrossAttention)
    m = MemoryEfficientDiTBlock(32, 4).train()
    xr = x.clone().requires_grad_(True)
    m(xr)[0].sum().backward()
    assert xr.grad is not None


def test_flow_predictor_zero_init():
    from drivedit_b200.models.blocks import FlowMatchingConfig

    cfg = FlowMatchingConfig(dim=32, num_layers=2, num_heads=4, latent_dim=8, context_dim=12)
    fp = FlowPredictor(cfg)
    v = fp(torch.randn(2, 6, 8), torch.rand(2), None, torch.randn(2, 3, 12))
    assert v.shape == (2, 6, 8) and torch.count_nonzero(v) == 0
