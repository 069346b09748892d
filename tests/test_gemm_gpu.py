"""tcgen05 GEMM vs a PyTorch fp32 reference of the same op (every epilogue/major mode)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["single", "pairs"])
def pair_mode(request):
    """Every test runs with single-CTA tiles only and with CTA-pair (cta_group::2, 256-row)
    tiles wherever a GEMM is eligible for them."""
    from drivedit_b200.ops._ext import ext
    prev = ext().gemm_set_pair_mode(0 if request.param == "single" else 1)
    yield request.param
    ext().gemm_set_pair_mode(prev)


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


class _Gather:
    """Launch arguments of the fused weight gather for a B emulated as sharded over
    ``world`` ranks whose buffers all live on this GPU."""

    def __init__(self, bufs, rank, elem0, shard, rows):
        self.bufs, self.rank, self.elem0, self.shard = bufs, rank, elem0, shard
        self.counters = torch.zeros((rows + 127) // 128, dtype=torch.int32, device="cuda")
        self.epoch = 0

    def launch_args(self, b):
        self.epoch += 1
        peers = [buf.data_ptr() + 2 * self.elem0 for buf in self.bufs]
        assert peers[self.rank] == b.data_ptr()
        return self.counters, peers, self.rank, self.elem0, self.shard, self.epoch


@pytest.mark.parametrize("world,rank,N,K,epi", [(2, 0, 768, 256, "bf16"), (4, 2, 2304, 768, "rope"),
                                                 (8, 5, 1536, 512, "swiglu"), (3, 1, 640, 3072, "bf16")])
def test_gemm_fused_weight_gather(world, rank, N, K, epi):
    """B lives at flat offset elem0 of a buffer sharded over `world` ranks; the local
    copy holds garbage outside this rank's shard, the other ranks' copies hold the
    truth for their shards. The GEMM must gather B (restoring the local copy exactly)
    and match a GEMM on the true weight, on two launches in a row."""
    from drivedit_b200.ops._ext import check_device_status
    from drivedit_b200.ops.gemm import gemm

    torch.manual_seed(world * 10 + rank)
    M = 1024
    elem0 = 512
    total = elem0 + N * K + 1024
    shard = -(-total // (world * 256)) * 256
    truth = (torch.randn(world * shard, device="cuda") * 0.05).bfloat16()
    bufs = []
    for r in range(world):
        b = torch.full_like(truth, float("nan"))
        b[r * shard:(r + 1) * shard] = truth[r * shard:(r + 1) * shard]
        bufs.append(b)
    W_true = truth[elem0:elem0 + N * K].view(N, K)
    W_local = bufs[rank][elem0:elem0 + N * K].view(N, K)
    g = _Gather(bufs, rank, elem0, shard, N)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    kw = {}
    if epi == "rope":
        from drivedit_b200.layers.rope import rope_angles_3d, rope_table

        kw = dict(rope_tab=rope_table(rope_angles_3d(64, 4, 8, 32)).cuda(), rope_cols=1024,
                  rope_rows_per_seq=M, rope_head_dim=64)
    for call in range(2):
        if call == 1:  # the peers' shards changed (an optimizer step) and are gathered again
            truth.mul_(1.5)
            for r in range(world):
                if r != rank:
                    bufs[r][r * shard:(r + 1) * shard] = truth[r * shard:(r + 1) * shard]
            bufs[rank][rank * shard:(rank + 1) * shard] = truth[rank * shard:(rank + 1) * shard]
        if epi == "swiglu":
            out = gemm(x, W_local, epi="swiglu", gather=g)
            ref = gemm(x, W_true.contiguous(), epi="swiglu")
        else:
            out = gemm(x, W_local, epi=epi, gather=g, **kw)
            ref = gemm(x, W_true.contiguous(), epi=epi, **kw)
        torch.cuda.synchronize()
        check_device_status()
        assert torch.equal(W_local, W_true), f"call {call}: local copy not restored"
        assert torch.equal(out, ref), f"call {call}: differs from the GEMM on the gathered weight"
