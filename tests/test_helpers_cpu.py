"""Building blocks from the reference's ``layers/nn_helpers.py`` (CPU oracles)."""
import math

import torch

from drivedit_b200.layers.helpers import (FusedMLP, PositionalEncoding, ScaledDotProductAttention,
                                          apply_rotary_pos_emb, fused_add_norm, gelu_tanh, silu)
from drivedit_b200.layers.norms import RMSNorm


def test_activations():
    x = torch.linspace(-4, 4, 101)
    assert torch.allclose(silu(x), x * torch.sigmoid(x))
    ref = 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
    assert torch.allclose(gelu_tanh(x), ref, atol=1e-6)


def test_fused_mlp_matches_unfused():
    torch.manual_seed(0)
    m = FusedMLP(32, 48)
    x = torch.randn(2, 5, 32)
    g, u = (x @ m.gate_up_proj.weight.t()).chunk(2, -1)
    ref = (torch.nn.functional.silu(g) * u) @ m.down_proj.weight.t()
    assert torch.allclose(m(x), ref, atol=1e-6)
    assert set(m.state_dict()) == {"gate_up_proj.weight", "down_proj.weight"}


def test_sdpa_module_masks():
    torch.manual_seed(1)
    q, k, v = (torch.randn(2, 3, 6, 8) for _ in range(3))
    att = ScaledDotProductAttention(use_flash=True)
    out = att(q, k, v)  # causal
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert torch.allclose(out, ref, atol=1e-5)
    mask = torch.ones(6, 6)
    mask[:, -1] = 0
    out = ScaledDotProductAttention()(q, k, v, mask)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask.bool())
    assert torch.allclose(out, ref, atol=1e-5)


def test_fused_add_norm_and_rotary_and_positions():
    torch.manual_seed(2)
    x, r = torch.randn(2, 4, 16), torch.randn(2, 4, 16)
    n, s = fused_add_norm(x, r, RMSNorm(16))
    assert torch.allclose(s, x + r) and torch.allclose(n, RMSNorm(16)(x + r))
    q, k = torch.randn(1, 2, 5, 8), torch.randn(1, 2, 5, 8)
    ang = torch.arange(5.0)[:, None] * torch.tensor([1.0, 0.1, 0.01, 0.001])[None]
    qr, kr = apply_rotary_pos_emb(q, k, ang.cos(), ang.sin())
    # rotate-half pairs channel i with i + 4: the pair's norm is preserved
    pair = lambda t: t[..., :4] ** 2 + t[..., 4:] ** 2
    assert torch.allclose(pair(qr), pair(q), atol=1e-5) and torch.allclose(pair(kr), pair(k), atol=1e-5)
    pe = PositionalEncoding(6, max_len=10)
    y = pe(torch.zeros(1, 3, 6))
    assert torch.allclose(y[0, 1, 0], torch.tensor(math.sin(1.0)))
    assert torch.allclose(y[0, 2, 1], torch.tensor(math.cos(2.0)))


def test_ddim_sample_equals_euler_at_eta_zero_and_is_exact_on_straight_paths():
    from drivedit_b200.training.flow_matching import RectifiedFlowSampler, ddim_sample, euler_sample

    torch.manual_seed(3)
    x0, x1 = torch.randn(4, 8), torch.randn(4, 8)
    # the exact velocity field of the straight path through (x0, x1)
    vel = lambda x, t: x1 - x0
    fwd = ddim_sample(vel, x0, 5, t_start=0.0, t_end=1.0)
    assert torch.allclose(fwd, x1, atol=1e-5)
    assert torch.allclose(fwd, euler_sample(vel, x0, 5), atol=1e-5)
    back = ddim_sample(vel, x1, 5)  # reference schedule: t from 1 to 0
    assert torch.allclose(back, x0, atol=1e-5)
    g = torch.Generator().manual_seed(0)
    noisy = ddim_sample(vel, x1, 5, eta=0.5, generator=g)
    assert noisy.shape == x0.shape and not torch.allclose(noisy, x0)
    # the predictor form: v(z, t, mask, context), trajectory and final sample
    s = RectifiedFlowSampler(lambda z, t, mask, ctx: x1 - x0)
    out = s.sample(x0, 5)
    assert out["trajectory"].shape == (6, 4, 8) and torch.allclose(out["final_sample"], x1, atol=1e-5)
    assert torch.allclose(s.ddim_sample(x1, 5), x0, atol=1e-5)


def test_attention_backend_api_and_sla_stats():
    import warnings

    from drivedit_b200.layers.attention import (AttentionBackend, attention_reference,
                                                get_attention_backend, mha, set_attention_backend)
    from drivedit_b200.layers.sla import SLAConfig, SLAStats, classify_blocks

    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 12, 2, 8) for _ in range(3))
    assert get_attention_backend() is AttentionBackend.SM100
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        assert set_attention_backend(AttentionBackend.FLASH_ATTN_3) is False and w
    try:
        assert set_attention_backend(AttentionBackend.EINSUM)
        torch.testing.assert_close(mha(q, k, v, causal=True),
                                   attention_reference(q, k, v, torch.ones(12, 12).tril().bool()))
    finally:
        set_attention_backend(AttentionBackend.SM100)
    torch.testing.assert_close(mha(q, k, v), attention_reference(q, k, v), rtol=1e-4, atol=1e-5)
    c, m, n = classify_blocks(torch.randn(1, 256, 2, 32), torch.randn(1, 256, 2, 32),
                              SLAConfig(block_size=64, causal=True))
    st = SLAStats.from_masks(c, m, n, 64)
    assert st.total_blocks == 2 * 16 and st.critical_blocks + st.marginal_blocks + st.negligible_blocks == 32
    assert 0.0 <= st.compute_savings <= 1.0
