"""RoPE v2 class surface (reference ``layers/rope_v2.py``): 1-D layer equals the free
functions, 3-D factorised rotation equals the full-grid tables, packed sequences equal
per-sequence application, chunked equals unchunked, cache slicing, interpolation and
resolution-aware tables."""
import torch

from drivedit_b200.layers.rope import compute_rope_freqs, rope_apply
from drivedit_b200.layers.rope_v2 import (RoPEConfig, RoPEFrequencyCache, RoPELayerV2,
                                          apply_rope_3d_efficient, compute_rope_3d_freqs,
                                          compute_resolution_aware_rope_freqs,
                                          interpolate_rope_freqs, precompute_rope_3d_freqs)


def _layer(**kw):
    return RoPELayerV2(RoPEConfig(use_half_precision=False, **kw))


def test_forward_matches_free_functions_and_start_pos():
    torch.manual_seed(0)
    rope = _layer(dim=64, max_seq_len=128)
    x = torch.randn(2, 40, 3, 64)
    s, c = compute_rope_freqs(64, 128)
    ref = rope_apply(x, s[5:45, None, :], c[5:45, None, :])
    assert torch.allclose(rope(x, start_pos=5), ref, atol=1e-6)
    q, k = rope.forward_qk(x, x * 2, start_pos=5)
    assert torch.allclose(q, ref, atol=1e-6) and torch.allclose(k, 2 * ref, atol=1e-5)
    # beyond the table: computed on demand
    assert rope(torch.randn(1, 200, 1, 64)).shape == (1, 200, 1, 64)


def test_chunked_equals_unchunked():
    rope = _layer(dim=32, max_seq_len=512)
    x = torch.randn(1, 300, 2, 32)
    assert torch.allclose(rope.forward_chunked(x, chunk_size=64, start_pos=3), rope(x, 3),
                          atol=1e-6)


def test_packed_flash_equals_per_sequence():
    rope = _layer(dim=32, max_seq_len=256)
    lens = [5, 17, 9]
    cu = torch.tensor([0, 5, 22, 31])
    q = torch.randn(31, 4, 32)
    k = torch.randn(31, 4, 32)
    qr, kr = rope.forward_flash(q, k, start_pos=2, cu_seqlens=cu)
    for i, n in enumerate(lens):
        sl = slice(int(cu[i]), int(cu[i + 1]))
        eq, ek = rope.forward_qk(q[None, sl], k[None, sl], start_pos=2)
        assert torch.allclose(qr[sl], eq[0], atol=1e-6) and torch.allclose(kr[sl], ek[0], atol=1e-6)


def test_3d_factorised_equals_full_grid():
    for dim in (96, 64):   # equal thirds (dim % 6 == 0) and the 64-channel default split
        rope = _layer(dim=dim, max_seq_len=1024, temporal_base_factor=0.5)
        T, H, W = 3, 4, 5
        x = torch.randn(2, T * H * W, 2, dim)
        out = rope.forward_3d(x, T, H, W, t_offset=1)
        sin, cos = compute_rope_3d_freqs(dim, T + 1, H, W, temporal_base_factor=0.5,
                                         efficient_mode=False)
        sin = sin[1:].reshape(T * H * W, dim // 2)
        cos = cos[1:].reshape(T * H * W, dim // 2)
        # the full grid rotates each axis group with the reference output layout
        ft, fh, fw = compute_rope_3d_freqs(dim, T + 1, H, W, temporal_base_factor=0.5)
        g = [ft[0].shape[1], fh[0].shape[1], fw[0].shape[1]]
        parts, c0, p0 = [], 0, 0
        for n in g:
            parts.append(rope_apply(x[..., c0:c0 + 2 * n], sin[None, :, None, p0:p0 + n],
                                    cos[None, :, None, p0:p0 + n]))
            c0, p0 = c0 + 2 * n, p0 + n
        assert torch.allclose(out, torch.cat(parts, -1), atol=1e-5)
    assert precompute_rope_3d_freqs(96, 2, 3, 4)[0].shape == (2, 3, 4, 48)


def test_cache_slices_and_lazily_computes():
    cache = RoPEFrequencyCache(RoPEConfig(dim=16, max_seq_len=512, use_half_precision=False,
                                          cache_common_lengths=(64, 256)))
    s, c = cache.get(100)          # sliced from the 256 table
    ref_s, ref_c = compute_rope_freqs(16, 100)
    assert torch.allclose(s, ref_s) and torch.allclose(c, ref_c)
    s2, _ = cache.get(700)         # computed on demand
    assert s2.shape == (700, 8)
    (st, _), (sh, _), (sw, _) = cache.get_3d(4, 5, 6)
    assert st.shape[0] == 4 and sh.shape[0] == 5 and sw.shape[0] == 6
    cache.clear()
    assert cache.get(10)[0].shape == (10, 8)


def test_interpolation_and_resolution_aware():
    s, c = compute_rope_freqs(16, 10)
    s2, c2 = interpolate_rope_freqs(s, c, 19)
    assert torch.allclose(s2[::2], s, atol=1e-6)       # linear keeps the original points
    assert torch.allclose(s2[1], 0.5 * (s[0] + s[1]), atol=1e-6)
    sn, _ = interpolate_rope_freqs(s, c, 5, mode="nearest")
    assert sn.shape == (5, 8)
    sa, _ = interpolate_rope_freqs(s, c, 5, mode="area")
    assert torch.allclose(sa[0], s[:2].mean(0), atol=1e-6)
    # at the training resolution the tables are the plain 2-D factorisation
    rs, rc = compute_resolution_aware_rope_freqs(16, 3, 4, 3, 4)
    hs, _ = compute_rope_freqs(8, 3)
    assert torch.allclose(rs.view(3, 4, 8)[:, 0, :4], hs, atol=1e-6)
    # at twice the resolution the last row sits at the training grid's last row angle
    rs2, _ = compute_resolution_aware_rope_freqs(16, 6, 8, 3, 4)
    assert torch.allclose(rs2.view(6, 8, 8)[2, 0, :4], hs[1], atol=1e-6)


def test_yarn_scale_and_dynamic_ntk():
    y = _layer(dim=32, max_seq_len=4096, original_max_seq_len=1024, yarn_enabled=True)
    assert y.get_attention_scale() > 1.0
    d = _layer(dim=32, max_seq_len=512, original_max_seq_len=128, dynamic_ntk=True,
               ntk_factor=2.0)
    x = torch.randn(1, 400, 1, 32)
    out = d(x)
    assert out.shape == x.shape and not torch.allclose(out, _layer(dim=32, max_seq_len=512)(x))
