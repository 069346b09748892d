"""Causal video VAE on CPU: reference shape contracts, streaming, VQ / KL tools, and the
host-side rewrites the CUDA convolution path relies on (space-to-depth for strided
convolutions, flipped-weight input gradient)."""
import torch
import torch.nn.functional as F

from drivedit_b200.models.vae3d import (CausalConv3d, KLAnnealer, VAE3D, VAE3DConfig,
                                        VectorQuantizer, get_minimal_config)
from drivedit_b200.ops.conv3d import conv_stride1_reference, s2d_weight, space_to_depth


def test_vae_shapes_and_loss():
    torch.manual_seed(0)
    cfg = VAE3DConfig(hidden_dims=[32, 64, 64, 64], use_gradient_checkpointing=False)
    v = VAE3D(cfg)
    x = torch.rand(1, 3, 8, 32, 32)
    out = v(x)
    # stride-2 kernel-4 padding-2 downsampling maps 32 -> 17 -> 9 -> 5 (reference extents)
    assert out["mean"].shape == (1, 8, 2, 5, 5)
    assert out["recon"].shape == x.shape
    for k in ("recon_loss", "l1_loss", "kl_loss", "perceptual_loss", "total_loss"):
        assert torch.isfinite(out[k]), k
    out["total_loss"].backward()
    assert v.encoder.conv_in.conv.weight.grad is not None
    assert VAE3D(in_channels=3, hidden_dims=[32, 64], use_attention=False).config.hidden_dims == [32, 64]


def test_strided_conv_as_space_to_depth():
    torch.manual_seed(1)
    for kt, k, st, s, T, H, W in [(4, 4, 2, 2, 8, 10, 12), (3, 4, 1, 2, 5, 9, 7), (4, 4, 2, 2, 7, 9, 11)]:
        w = torch.randn(6, 5, kt, k, k, dtype=torch.float64)
        x = torch.randn(2, 5, T, H, W, dtype=torch.float64)
        ref = F.conv3d(F.pad(x, (0, 0, 0, 0, kt - 1, 0)), w, stride=(st, s, s), padding=(0, k // 2, k // 2))
        w2, ks, p2 = s2d_weight(w, (st, s, s), (kt - 1, k // 2, k // 2))
        xs = space_to_depth(x.permute(0, 2, 3, 4, 1), (st, s, s))
        y = conv_stride1_reference(xs, w2, p2, ref.shape[2:]).permute(0, 4, 1, 2, 3)
        assert torch.allclose(y.double(), ref, atol=1e-4)


def test_input_gradient_is_flipped_conv():
    torch.manual_seed(2)
    kt, kh, kw = 3, 3, 3
    pads = (2, 1, 1)
    x = torch.randn(1, 4, 5, 6, 7, requires_grad=True)  # [B, T, H, W, C]
    w = torch.randn(3, 7, kt, kh, kw)
    y = conv_stride1_reference(x, w, pads, (4, 5, 6))
    dy = torch.randn_like(y)
    (y * dy).sum().backward()
    wf = w.flip(2, 3, 4).transpose(0, 1)  # [Cin, Cout, ...]
    dx = conv_stride1_reference(dy, wf, (kt - 1 - pads[0], kh - 1 - pads[1], kw - 1 - pads[2]),
                                (4, 5, 6))
    assert torch.allclose(dx, x.grad, atol=1e-4)


def test_streaming_causal_conv_matches_full_sequence():
    torch.manual_seed(3)
    conv = CausalConv3d(4, 5, (3, 3, 3))
    x = torch.randn(1, 4, 9, 6, 6)
    full = conv.conv(x)  # no temporal padding: the streaming contract
    conv.reset_cache()
    parts = [conv(x[:, :, i:i + 3], streaming=True) for i in range(0, 9, 3)]
    assert torch.allclose(torch.cat(parts, 2), full, atol=1e-5)


def test_vq_and_kl_annealing():
    torch.manual_seed(4)
    vq = VectorQuantizer(16, 4).train()
    z = torch.randn(1, 4, 2, 3, 3, requires_grad=True)
    zq, loss, idx = vq(z)
    assert zq.shape == z.shape and idx.shape == (1, 2, 3, 3) and torch.isfinite(loss)
    zq.sum().backward()
    assert torch.allclose(z.grad, torch.ones_like(z))  # straight-through
    a = KLAnnealer("cyclical", cycle_period=10, start_beta=0.0, end_beta=1.0)
    betas = []
    for _ in range(10):
        betas.append(a.get_beta())
        a.update()
    assert betas[0] == 0.0 and abs(betas[5] - 0.5) < 1e-9 and max(betas) < 1.0
    lin = KLAnnealer("linear", warmup_steps=4)
    lin.step = 2
    assert lin.get_beta() == 0.5


def test_minimal_config_roundtrip_and_partial_load():
    torch.manual_seed(5)
    v = VAE3D(get_minimal_config()).eval()
    x = torch.rand(1, 3, 4, 16, 16)
    out = v(x, return_loss=False)
    assert out["recon"].shape == x.shape
    v2 = VAE3D.from_pretrained_v1(v.state_dict(), get_minimal_config())
    assert len(v2.loaded_keys) == len(v.state_dict())
