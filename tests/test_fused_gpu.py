"""Fused memory-bound kernels and the fused world-model block path vs PyTorch fp32."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.mark.parametrize("D", [256, 768, 1024, 1536, 2048])
def test_adaln_fwd_bwd(D):
    from drivedit_b200.ops.fused import adaln_rmsnorm, adaln_rmsnorm_bwd
    M, tpf = 1024, 128
    G = M // tpf
    x = torch.randn(M, D, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(D, device="cuda"))
    mod = 0.2 * torch.randn(G, 4 * D, device="cuda")
    h, r = adaln_rmsnorm(x, w, mod, 2 * D, 3 * D, tpf)
    xf = x.float().requires_grad_(True)
    wf = w.clone().requires_grad_(True)
    mf = mod.clone().requires_grad_(True)
    sc = mf[:, 2 * D:3 * D].repeat_interleave(tpf, 0)
    sh = mf[:, 3 * D:4 * D].repeat_interleave(tpf, 0)
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf * (1 + sc) + sh
    assert _rel(h, ref) < 1e-2
    dh = torch.randn(M, D, device="cuda").bfloat16()
    dres = torch.randn(M, D, device="cuda").bfloat16()
    ref.backward(dh.float())
    dmod = torch.zeros_like(mod)
    dw = torch.zeros_like(w)
    dx = adaln_rmsnorm_bwd(dh, x, r, w, mod, 2 * D, 3 * D, tpf, dmod, dw, dres)
    assert _rel(dx, xf.grad + dres.float()) < 2e-2
    assert _rel(dw, wf.grad) < 1e-2
    assert _rel(dmod, mf.grad) < 1e-2


def test_adaln_bwd_odd_groups_no_dw_no_residual():
    """Groups of 100 rows (not a multiple of 8: CTAs of 50 rows), no norm-weight gradient,
    no residual."""
    from drivedit_b200.ops.fused import adaln_rmsnorm, adaln_rmsnorm_bwd
    M, D, tpf = 1000, 768, 100
    G = M // tpf
    x = torch.randn(M, D, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(D, device="cuda"))
    mod = 0.2 * torch.randn(G, 2 * D, device="cuda")
    h, r = adaln_rmsnorm(x, w, mod, 0, D, tpf)
    xf = x.float().requires_grad_(True)
    mf = mod.clone().requires_grad_(True)
    sc = mf[:, :D].repeat_interleave(tpf, 0)
    sh = mf[:, D:].repeat_interleave(tpf, 0)
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w * (1 + sc) + sh
    dh = torch.randn(M, D, device="cuda").bfloat16()
    ref.backward(dh.float())
    dmod = torch.zeros_like(mod)
    dx = adaln_rmsnorm_bwd(dh, x, r, w, mod, 0, D, tpf, dmod)
    assert _rel(dx, xf.grad) < 2e-2
    assert _rel(dmod, mf.grad) < 1e-2


def test_adamw_matches_reference():
    from drivedit_b200.ops.fused import adamw_flat
    n = 4096
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    comp = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    ref = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(1, 4):
        ref.grad = g.clone()
        opt.step()
        adamw_flat(p, g, m, v, comp, torch.ones((), device="cuda"), lr=1e-2, b1=0.9, b2=0.95,
                   eps=1e-8, wd=0.1, bc1=1 - 0.9 ** step, bc2=1 - 0.95 ** step)
    assert _rel(p, ref.detach()) < 1e-5
    assert _rel(comp, ref.detach()) < 1e-2


def test_rope_rotate_roundtrip():
    from drivedit_b200.ops.fused import rope_rotate_
    M, C = 512, 256
    x = torch.randn(M, 3 * C, device="cuda").bfloat16()
    ang = torch.rand(M, 32, device="cuda") * 3
    tab = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
    y = x.clone()
    rope_rotate_(y, 2 * C, tab, 64, M, 0, inverse=False)
    rope_rotate_(y, 2 * C, tab, 64, M, 0, inverse=True)
    assert _rel(y, x) < 2e-2


def _small_cfg(attention="dense"):
    from drivedit_b200.config import get_config
    cfg = get_config("tiny", ["model.n_layers=2", "model.latent_h=32", "model.latent_w=32",
                              f"model.attention={attention}", "train.frames=2",
                              "train.batch_per_gpu=2", "train.dtype=bf16"])
    return cfg


@pytest.mark.parametrize("batched_mods", [False, True])
def test_fused_model_matches_torch_path(batched_mods):
    """Fused CUDA path vs the PyTorch path, forward and every parameter gradient; with
    ``batched_mods`` the flat layout groups the AdaLN modulation projections so all of
    them run as one GEMM (forward) and one GEMM pair (backward)."""
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.parallel.flat import FlatParamGroup
    torch.manual_seed(0)
    cfg = _small_cfg()
    m_ref = WorldDiT(cfg.model).cuda()
    # non-trivial modulation / head so every path carries signal
    with torch.no_grad():
        for p in m_ref.parameters():
            if p.abs().sum() == 0:
                p.normal_(0, 0.02)
    m = WorldDiT(cfg.model).cuda()
    m.load_state_dict(m_ref.state_dict())
    named = m.flat_layout(m.named_parameters()) if batched_mods else m.named_parameters()
    group = FlatParamGroup(named, "cuda")
    m.enable_fused(group=group)
    B, Fr = 2, 2
    x = torch.randn(B, Fr, 16, 32, 32, device="cuda")
    t = torch.rand(B, device="cuda")
    a = torch.rand(B, Fr, 2, device="cuda") * 2 - 1
    v_ref = m_ref(x, t, a)
    v = m(x.bfloat16(), t, a)
    assert _rel(v, v_ref) < 3e-2
    dv = torch.randn_like(v_ref)
    v_ref.backward(dv)
    group.zero_grad()
    v.float().backward(dv)
    torch.cuda.synchronize()
    ref_params = dict(m_ref.named_parameters())
    worst = {}
    for n, p in m.named_parameters():
        g_ref = ref_params[n].grad
        if g_ref is None or g_ref.abs().max() == 0:
            continue
        worst[n] = _rel(p.grad, g_ref)
    bad = {k: v for k, v in worst.items() if v > 6e-2}
    assert not bad, bad
    assert (m.fused._runs is not None) == batched_mods


def test_video_augment_kernel():
    from drivedit_b200.data.transforms import AugmentationPipeline, clip_augment_reference
    torch.manual_seed(0)
    x = torch.rand(3, 4, 3, 17, 33, device="cuda")
    flip = torch.tensor([1, 0, 1], device="cuda")
    br = torch.tensor([0.1, -0.2, 0.0], device="cuda")
    ct = torch.tensor([1.2, 0.8, 1.0], device="cuda")
    mean, std = [0.5, 0.4, 0.3], [0.2, 0.25, 0.3]
    y = AugmentationPipeline.fused_clip_augment(x, flip, br, ct, mean, std)
    ref = clip_augment_reference(x, flip, br, ct, mean, std)
    assert (y - ref).abs().max() < 1e-5
    u8 = (x.permute(0, 1, 3, 4, 2) * 255).round().to(torch.uint8).contiguous()
    y2 = AugmentationPipeline.fused_clip_augment(u8, flip, br, ct, mean, std, out_bf16=True, input_u8_hwc=True)
    ref2 = clip_augment_reference(u8.permute(0, 1, 4, 2, 3).float() / 255, flip, br, ct, mean, std)
    assert (y2.float() - ref2).abs().max() < 3e-2


@pytest.mark.parametrize("moe", [False, True])
def test_block_recompute_matches_saved_activations(moe):
    """Activation checkpointing in the fused engine (each block keeps only its input and
    reruns its forward in the backward): the same output, the same parameter gradients
    and the same MoE routing-bias state as keeping the activations."""
    from drivedit_b200.config import MoEParams
    from drivedit_b200.models.world_dit import WorldDiT
    from drivedit_b200.ops.debug import deterministic
    from drivedit_b200.parallel.flat import FlatParamGroup
    torch.manual_seed(0)
    cfg = _small_cfg()
    if moe:
        cfg.model.mlp_hidden = 0
        cfg.model.moe = MoEParams(num_experts=8, top_k=2, expert_dim=128, num_shared=2,
                                  aux_loss_weight=0.01)
    m = WorldDiT(cfg.model).cuda().train()
    with torch.no_grad():
        for p in m.parameters():
            if p.abs().sum() == 0:
                p.normal_(0, 0.02)
    group = FlatParamGroup(m.flat_layout(m.named_parameters()), "cuda")
    m.enable_fused(group=group)
    x = torch.randn(2, 2, 16, 32, 32, device="cuda").bfloat16()
    t = torch.rand(2, device="cuda")
    a = torch.rand(2, 2, 2, device="cuda")
    dv = torch.randn(2, 2, 16, 32, 32, device="cuda")
    moes = [b.moe for b in m.blocks if b.moe is not None]
    state0 = [(mo.expert_bias.clone(), mo.expert_load_ema.clone()) for mo in moes]
    out = {}
    with deterministic():
        for rec in (False, True):
            for mo, (b0, e0) in zip(moes, state0):  # both runs start from the same balancing state
                mo.expert_bias.copy_(b0)
                mo.expert_load_ema.copy_(e0)
            m.fused.recompute = rec
            group.zero_grad()
            v, aux = m(x, t, a, return_aux=True)
            (v.float() * dv).sum().add(aux).backward()
            torch.cuda.synchronize()
            out[rec] = (v.float().clone(), group.grad.clone(),
                        [b.moe.expert_bias.clone() for b in m.blocks if b.moe is not None])
    assert _rel(out[True][0], out[False][0]) < 1e-6
    assert _rel(out[True][1], out[False][1]) < 1e-3
    for b1, b2 in zip(out[True][2], out[False][2]):
        assert torch.equal(b1, b2)
