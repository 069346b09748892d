"""Video-VAE kernels (implicit-GEMM causal conv3d, GroupNorm+SiLU) vs fp32 PyTorch."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _ref_conv(x, w, b, stride):
    kt, kh, kw = w.shape[2:]
    xp = F.pad(x.bfloat16().float(), (0, 0, 0, 0, kt - 1, 0))
    return F.conv3d(xp, w.bfloat16().float(), b, stride=stride, padding=(0, kh // 2, kw // 2))


CASES = [
    # B, Cin, Cout, T, H, W, kernel, stride
    (1, 128, 128, 4, 16, 32, (3, 3, 3), (1, 1, 1)),
    (2, 64, 96, 3, 9, 33, (3, 3, 3), (1, 1, 1)),
    (1, 3, 128, 4, 16, 16, (3, 3, 3), (1, 1, 1)),
    (1, 128, 3, 2, 16, 16, (3, 3, 3), (1, 1, 1)),
    (1, 128, 128, 4, 16, 16, (4, 4, 4), (2, 2, 2)),
    (1, 128, 128, 3, 15, 17, (3, 4, 4), (1, 2, 2)),
    (1, 256, 512, 2, 4, 4, (1, 1, 1), (1, 1, 1)),
]


@pytest.mark.parametrize("case", CASES)
def test_conv3d_forward(case):
    from drivedit_b200.ops.conv3d import causal_conv3d
    B, Cin, Cout, T, H, W, k, st = case
    torch.manual_seed(0)
    x = torch.randn(B, Cin, T, H, W, device="cuda")
    w = torch.randn(Cout, Cin, *k, device="cuda") * 0.05
    b = torch.randn(Cout, device="cuda")
    y = causal_conv3d(x, w, b, st)
    ref = _ref_conv(x, w, b, st)
    assert y.shape == ref.shape
    assert _rel(y, ref) < 1e-2


@pytest.mark.parametrize("case", [CASES[0], CASES[3], CASES[4], CASES[1]])
def test_conv3d_backward(case):
    from drivedit_b200.ops.conv3d import causal_conv3d
    B, Cin, Cout, T, H, W, k, st = case
    torch.manual_seed(1)
    x = torch.randn(B, Cin, T, H, W, device="cuda").bfloat16().float().requires_grad_(True)
    w = (torch.randn(Cout, Cin, *k, device="cuda") * 0.05).bfloat16().float().requires_grad_(True)
    b = torch.randn(Cout, device="cuda", requires_grad=True)
    y = causal_conv3d(x, w, b, st)
    dy = torch.randn(y.shape, device="cuda").bfloat16().float()
    (y.float() * dy).sum().backward()
    gx, gw, gb = x.grad.clone(), w.grad.clone(), b.grad.clone()
    x.grad = w.grad = b.grad = None
    ref = _ref_conv(x, w, b, st)
    (ref * dy).sum().backward()
    assert _rel(gx, x.grad) < 2e-2
    assert _rel(gw, w.grad) < 2e-2
    assert _rel(gb, b.grad) < 1e-3


def test_groupnorm_silu_forward_backward():
    from drivedit_b200.ops.conv3d import group_norm_silu
    torch.manual_seed(2)
    x = (torch.randn(2, 256, 4, 8, 16, device="cuda") * 3 + 1).bfloat16().float().requires_grad_(True)
    w = torch.randn(256, device="cuda", requires_grad=True)
    b = torch.randn(256, device="cuda", requires_grad=True)
    for silu in (True, False):
        y = group_norm_silu(x, 32, w, b, 1e-5, silu)
        ref = F.group_norm(x, 32, w, b, 1e-5)
        ref = F.silu(ref) if silu else ref
        assert _rel(y, ref) < 1e-2
        dy = torch.randn_like(ref)
        g = torch.autograd.grad((y.float() * dy).sum(), (x, w, b))
        gr = torch.autograd.grad((ref * dy).sum(), (x, w, b))
        for a, r in zip(g, gr):
            assert _rel(a, r) < 2e-2


def test_vae_cuda_matches_cpu_fp32():
    from drivedit_b200.models.vae3d import VAE3D, VAE3DConfig
    torch.manual_seed(3)
    cfg = VAE3DConfig(hidden_dims=[128, 256, 512], use_gradient_checkpointing=False,
                      use_perceptual_loss=False, attention_resolution=[8])
    cpu = VAE3D(cfg).eval()
    gpu = VAE3D(cfg).eval()
    gpu.load_state_dict(cpu.state_dict())
    gpu.cuda()
    x = torch.rand(1, 3, 4, 32, 32)
    with torch.no_grad():
        ref = cpu(x, return_loss=False)
        out = gpu(x.cuda(), return_loss=False)
    assert _rel(out["mean"].cpu(), ref["mean"]) < 5e-2
    assert _rel(out["recon"].cpu(), ref["recon"]) < 5e-2
