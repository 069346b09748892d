"""tcgen05 GEMM vs a PyTorch fp32 reference of the same op (every epilogue/major mode)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, a_t=False, b_t=False):
    A = (a.t() if a_t else a).float()
    B = (b.t() if b_t else b).float()
    return A @ B.t()


def _close(x, y, tol=2e-2):
    err = (x.float() - y.float()).abs().max().item()
    scale = y.float().abs().max().item() + 1e-6
    assert err / scale < tol, f"rel err {err / scale:.3e}"


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 512, 256), (300, 384, 192), (1024, 2304, 768), (4096, 768, 3072)])
@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_bf16_kmajor(M, N, K, bn):
    from drivedit_b200.ops.gemm import gemm
    if bn == 256 and N % 256:
        pytest.skip("tile")
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    out = gemm(a, b, bn=bn)
    torch.cuda.synchronize()
    _close(out, _ref(a, b))


@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (1024, 768, 2304), (384, 256, 128)])
def test_gemm_b_transposed(M, N, K):
    from drivedit_b200.ops.gemm import gemm
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    bt = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)  # B stored [K, N]
    out = gemm(a, bt, b_t=True)
    _close(out, _ref(a, bt, b_t=True))


@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (768, 2304, 4096), (512, 256, 640)])
def test_gemm_both_transposed_f32(M, N, K):
    from drivedit_b200.ops.gemm import gemm
    at = torch.randn(K, M, device="cuda", dtype=torch.bfloat16)
    bt = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
    out = gemm(at, bt, epi="f32", a_t=True, b_t=True)
    _close(out, _ref(at, bt, a_t=True, b_t=True), tol=1e-2)
    acc = torch.ones(M, N, device="cuda", dtype=torch.float32)
    gemm(at, bt, acc, epi="f32_acc", a_t=True, b_t=True, splits=4)
    _close(acc, _ref(at, bt, a_t=True, b_t=True) + 1.0, tol=1e-2)


def test_gemm_bias_residual():
    from drivedit_b200.ops.gemm import gemm
    M, N, K = 512, 768, 256
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    bias = torch.randn(N, device="cuda", dtype=torch.float32)
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    out = gemm(a, b, bias=bias, residual=res)
    _close(out, _ref(a, b) + bias + res.float())
    # residual aliasing the output (in-place residual stream update)
    x = res.clone()
    gemm(a, b, x, residual=x)
    _close(x, _ref(a, b) + res.float())


def test_gemm_swiglu_and_back():
    from drivedit_b200.ops.gemm import gemm
    M, F, K = 512, 512, 256  # F = hidden width; gu has 2F columns
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * F, K, device="cuda", dtype=torch.bfloat16) * 0.1
    gu, act = torch.empty(M, 2 * F, device="cuda", dtype=torch.bfloat16), None
    act = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    gemm(a, w, gu, epi="swiglu", out2=act)
    ref = _ref(a, w)
    _close(gu, ref)
    r = ref.view(M, F // 32, 2, 32)
    g, u = r[:, :, 0].reshape(M, F), r[:, :, 1].reshape(M, F)
    _close(act, torch.nn.functional.silu(g) * u, tol=3e-2)
    # backward: d(act) = dy @ w2 ; here just use a random dA via a GEMM with dswiglu
    dy = torch.randn(M, 256, device="cuda", dtype=torch.bfloat16)
    w2 = torch.randn(256, F, device="cuda", dtype=torch.bfloat16) * 0.1  # [D, F]
    dgu = gemm(dy, w2, epi="dswiglu", b_t=True, residual=gu)
    da = dy.float() @ w2.float()
    gg = gu.float().view(M, F // 32, 2, 32)
    g, u = gg[:, :, 0].reshape(M, F), gg[:, :, 1].reshape(M, F)
    s = torch.sigmoid(g)
    dg = da * u * s * (1 + g * (1 - s))
    du = da * g * s
    ref_dgu = torch.stack([dg.view(M, F // 32, 32), du.view(M, F // 32, 32)], 2).view(M, 2 * F)
    _close(dgu, ref_dgu, tol=3e-2)


def test_gemm_rope():
    from drivedit_b200.ops.gemm import gemm
    M, H, Dh, K = 512, 4, 64, 256
    N = 3 * H * Dh
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    T = 256
    ang = torch.rand(T, Dh // 2, device="cuda") * 6.0
    tab = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    out = gemm(a, b, epi="rope", rope_tab=tab, rope_cols=2 * H * Dh, rope_rows_per_seq=T)
    ref = _ref(a, b)
    qk = ref[:, : 2 * H * Dh].view(M, 2 * H, Dh // 2, 2)
    pos = torch.arange(M, device="cuda") % T
    c, s_ = tab[pos, :, 0][:, None], tab[pos, :, 1][:, None]
    x0, x1 = qk[..., 0], qk[..., 1]
    rot = torch.stack([x0 * c - x1 * s_, x0 * s_ + x1 * c], -1).view(M, 2 * H * Dh)
    ref = torch.cat([rot, ref[:, 2 * H * Dh:]], 1)
    _close(out, ref)


def test_status_clean():
    from drivedit_b200.ops._ext import device_status
    torch.cuda.synchronize()
    assert device_status() == 0
