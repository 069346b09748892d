"""Fused sm_100a forward/backward of the world-model DiT blocks.

Per block, with ``M = B*T`` token rows, ``d`` model width, ``F`` SwiGLU width:

forward                                           kernels
  h1, r1 = adaln_rmsnorm(x, w1, mod[s1, b1])        fused/norm.cu
  qkv    = h1 Wqkv^T  (+ 3-D RoPE on q, k)          gemm.cu, rope epilogue
  o, lse = attention(qkv)  (dense or SLA)           attn/*.cu
  x1     = x + o Wo^T (+ o_lin Wlin^T)              gemm.cu, residual epilogue
  h2, r2 = adaln_rmsnorm(x1, w2, mod[s2, b2])
  gu, a  = h2 W13^T, silu(g) * u                    gemm.cu, SwiGLU epilogue
  x2     = x1 + a W3^T                              gemm.cu, residual epilogue

backward: the transposed products read operands in place (MN-major TMA tiles), weight
gradients accumulate in fp32 straight into the flat gradient buffer, the SwiGLU
derivative is the epilogue of the ``dA`` GEMM, and the norm backward adds the
residual-stream gradient and reduces the norm-weight and modulation gradients.

Non-block pieces (patch embedding, output head) use the same GEMM through
:func:`drivedit_b200.ops.linear.linear`; the conditioning MLPs (``[B*F, d]``, a few
hundred rows) stay in PyTorch.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from ..parallel.flat import FlatParamGroup
from .attention import attention_bwd, attention_fwd
from .fused import adaln_rmsnorm, adaln_rmsnorm_bwd, rope_rotate_
from .gemm import gemm
from .linear import linear


class BlockCtx:
    """Static per-call data shared by all blocks of one forward."""

    def __init__(self, B, T, frames, tpf, d, H, Dh, rope_tab, attn_mode, sla_cfg, causal,
                 rope_pos_offset=0):
        self.B, self.T, self.frames, self.tpf = B, T, frames, tpf
        self.d, self.H, self.Dh = d, H, Dh
        self.rope_tab = rope_tab
        self.attn_mode = attn_mode
        self.sla_cfg = sla_cfg
        self.causal = causal
        self.rope_pos_offset = rope_pos_offset
        self.recompute = False  # activation checkpointing: blocks rerun their forward in backward
        self.grad_ready = None  # callback(block index) once a block's backward is enqueued


def _gather_of(W):
    """The fused weight all-gather handle lookup of a weight-sharded group (or none)."""
    fn = getattr(getattr(W, "__self__", None), "gather_for", None)
    return fn if fn is not None else (lambda p: None)


def _attn_forward(x, mod, blk, W, bc):
    d = bc.d
    G = _gather_of(W)
    h1, r1 = adaln_rmsnorm(x, blk.norm1.weight, mod, 0, d, bc.tpf)
    qkv = gemm(h1, W(blk.attn.qkv.weight), epi="rope", rope_tab=bc.rope_tab, rope_cols=2 * d,
               rope_rows_per_seq=bc.T, rope_pos_offset=bc.rope_pos_offset, rope_head_dim=bc.Dh,
               gather=G(blk.attn.qkv.weight))
    o, o_lin, lse, aux = attention_fwd(qkv, bc)
    x1 = gemm(o, W(blk.attn.proj.weight), residual=x, gather=G(blk.attn.proj.weight))
    if o_lin is not None:
        gemm(o_lin, W(blk.attn.proj_lin.weight), x1, residual=x1,
             gather=G(blk.attn.proj_lin.weight))
    return x1, dict(x=x, h1=h1, r1=r1, qkv=qkv, o=o, o_lin=o_lin, lse=lse, aux=aux)


def _attn_backward(dx1, sa, blk, W, bc, mod, dmod):
    """Gradient of the block input given the gradient of the attention-residual output."""
    d = bc.d
    do = gemm(dx1, W(blk.attn.proj.weight), b_t=True)
    gemm(dx1, sa["o"], blk.attn.proj.weight.grad, epi="f32_acc", a_t=True, b_t=True)
    do_lin = None
    if sa["o_lin"] is not None:
        do_lin = gemm(dx1, W(blk.attn.proj_lin.weight), b_t=True)
        gemm(dx1, sa["o_lin"], blk.attn.proj_lin.weight.grad, epi="f32_acc", a_t=True, b_t=True)
    dqkv = attention_bwd(sa["qkv"], sa["o"], sa["lse"], do, do_lin, sa["aux"], bc)
    # q, k gradients back through the rotation
    rope_rotate_(dqkv, 2 * d, bc.rope_tab, bc.Dh, bc.T, bc.rope_pos_offset, inverse=True)
    dh1 = gemm(dqkv, W(blk.attn.qkv.weight), b_t=True)
    gemm(dqkv, sa["h1"], blk.attn.qkv.weight.grad, epi="f32_acc", a_t=True, b_t=True)
    return adaln_rmsnorm_bwd(dh1, sa["x"], sa["r1"], blk.norm1.weight, mod, 0, d, bc.tpf, dmod,
                             blk.norm1.weight.grad, dx1)


def _mlp_forward(x1, mod, blk, W, bc):
    d = bc.d
    G = _gather_of(W)
    h2, r2 = adaln_rmsnorm(x1, blk.norm2.weight, mod, 2 * d, 3 * d, bc.tpf)
    w13 = W(blk.mlp.w13.weight)
    gu = torch.empty(x1.shape[0], w13.shape[0], device=x1.device, dtype=torch.bfloat16)
    a = torch.empty(x1.shape[0], w13.shape[0] // 2, device=x1.device, dtype=torch.bfloat16)
    gemm(h2, w13, gu, epi="swiglu", out2=a, gather=G(blk.mlp.w13.weight))
    x2 = gemm(a, W(blk.mlp.w3.weight), residual=x1, gather=G(blk.mlp.w3.weight))
    return x2, dict(x1=x1, h2=h2, r2=r2, gu=gu, a=a)


def _mlp_backward(dx2, sm, blk, W, bc, mod, dmod):
    d = bc.d
    dgu = gemm(dx2, W(blk.mlp.w3.weight), epi="dswiglu", b_t=True, residual=sm["gu"])
    gemm(dx2, sm["a"], blk.mlp.w3.weight.grad, epi="f32_acc", a_t=True, b_t=True)
    dh2 = gemm(dgu, W(blk.mlp.w13.weight), b_t=True)
    gemm(dgu, sm["h2"], blk.mlp.w13.weight.grad, epi="f32_acc", a_t=True, b_t=True)
    del dgu
    return adaln_rmsnorm_bwd(dh2, sm["x1"], sm["r2"], blk.norm2.weight, mod, 2 * d, 3 * d, bc.tpf,
                             dmod, blk.norm2.weight.grad, dx2)


def _moe_forward(x1, mod, blk, W, bc):
    from .moe import moe_ffn_forward, moe_ffn_forward_ep

    d = bc.d
    h2, r2 = adaln_rmsnorm(x1, blk.norm2.weight, mod, 2 * d, 3 * d, bc.tpf)
    fwd = moe_ffn_forward if blk.moe.ep is None else moe_ffn_forward_ep
    x2, aux, sv = fwd(h2, x1, blk.moe, W)
    sv.update(x1=x1, r2=r2)
    return x2, aux, sv


def _moe_backward(dx2, d_aux, sv, blk, W, bc, mod, dmod):
    from .moe import moe_ffn_backward, moe_ffn_backward_ep

    d = bc.d
    bwd = moe_ffn_backward if blk.moe.ep is None else moe_ffn_backward_ep
    dh2 = bwd(dx2, d_aux, blk.moe, W, sv)
    return adaln_rmsnorm_bwd(dh2, sv["x1"], sv["r2"], blk.norm2.weight, mod, 2 * d, 3 * d, bc.tpf,
                             dmod, blk.norm2.weight.grad, dx2)


class _BlockFn(torch.autograd.Function):
    """One dense (attention + SwiGLU) or MoE (attention + experts) block; returns
    ``(x_out, aux_loss)`` where ``aux_loss`` is the unweighted MoE load-balance term.

    With ``dmod_out`` (batched modulations, :class:`_AllMods`) ``mod`` is a detached view
    of the shared modulation matrix; the backward accumulates the modulation gradient
    into ``dmod_out`` (this block's columns of the shared gradient buffer) and returns a
    zero gradient for ``token``, the scalar that ties every block to the one GEMM
    backward of all modulations."""

    @staticmethod
    def _run(x, mod, blk, W, bc):
        x1, sa = _attn_forward(x, mod, blk, W, bc)
        if blk.moe is None:
            x2, sm = _mlp_forward(x1, mod, blk, W, bc)
            aux = torch.zeros((), device=x.device)
        else:
            x2, aux, sm = _moe_forward(x1, mod, blk, W, bc)
        return x2, aux, sa, sm

    @staticmethod
    def forward(ctx, x, mod, blk, group: FlatParamGroup, bc: BlockCtx, token=None, dmod_out=None):
        W = group.compute_view
        # with recomputation the routing bias this forward used is kept, so the backward's
        # rerun routes every token exactly as this forward did
        bias = blk.moe.expert_bias.clone() if (bc.recompute and blk.moe is not None) else None
        x2, aux, sa, sm = _BlockFn._run(x, mod, blk, W, bc)
        if bc.recompute:  # keep only the block input; the activations are rebuilt in backward
            sa = sm = None
            ctx.x_in, ctx.bias = x, bias
        ctx.sa, ctx.sm, ctx.mod = sa, sm, mod
        ctx.blk, ctx.group, ctx.bc = blk, group, bc
        ctx.dmod_out = dmod_out
        return x2, aux

    @staticmethod
    def backward(ctx, dx2, d_aux):
        blk, bc, mod = ctx.blk, ctx.bc, ctx.mod
        W = ctx.group.compute_view
        if ctx.sa is None:  # recompute the forward (no MoE bias update, the forward's bias)
            moe = blk.moe
            cur = None
            if moe is not None:
                cur = moe.expert_bias.clone()
                moe.expert_bias.copy_(ctx.bias)
                moe.frozen_bias = True
            try:
                _, _, ctx.sa, ctx.sm = _BlockFn._run(ctx.x_in, mod, blk, W, bc)
            finally:
                if moe is not None:
                    moe.expert_bias.copy_(cur)
                    moe.frozen_bias = False
            ctx.x_in = ctx.bias = None
        dx2 = dx2.contiguous()
        batched = ctx.dmod_out is not None
        dmod = ctx.dmod_out if batched else torch.zeros(mod.shape, device=mod.device,
                                                        dtype=torch.float32)
        if blk.moe is None:
            dx1 = _mlp_backward(dx2, ctx.sm, blk, W, bc, mod, dmod)
        else:
            # d_aux already carries the aux-loss weight (the caller scales the output)
            dx1 = _moe_backward(dx2, d_aux, ctx.sm, blk, W, bc, mod, dmod)
        dx = _attn_backward(dx1, ctx.sa, blk, W, bc, mod, dmod)
        ctx.sa = ctx.sm = ctx.dmod_out = None
        if bc.grad_ready is not None:  # the block's weight gradients are final
            bc.grad_ready(getattr(blk, "block_index", -1))
        if batched:
            return dx, None, None, None, None, torch.zeros((), device=dx.device), None
        return dx, dmod, None, None, None, None, None


def _mod_runs(model, group: FlatParamGroup):
    """(weight offset, bias offset) of the contiguous runs that hold every block's
    modulation projection followed by the final one, or ``None`` when the group's
    layout keeps them apart."""
    mods = [blk.ada for blk in model.blocks] + [model.final_ada]
    if not all(group.owns(m.weight) and group.owns(m.bias) for m in mods):
        return None
    w_off = [group.offsets[group.names[group.index(m.weight)]][0] for m in mods]
    b_off = [group.offsets[group.names[group.index(m.bias)]][0] for m in mods]
    w_len = [m.weight.numel() for m in mods]
    b_len = [m.bias.numel() for m in mods]
    for i in range(len(mods) - 1):
        if w_off[i] + w_len[i] != w_off[i + 1] or b_off[i] + b_len[i] != b_off[i + 1]:
            return None
    return w_off[0], b_off[0], sum(w_len), sum(b_len)


class _AllMods(torch.autograd.Function):
    """Every block's AdaLN modulation (and the final layer's) from the per-frame
    conditioning in one tcgen05 GEMM: ``mods [B*F, sum n_mod d] = c W_all^T + b_all``,
    where ``W_all`` is the contiguous run of all modulation weights in the flat buffer.
    Backward (after every block has written its columns of the shared gradient):
    one split-K GEMM for ``dc = dmods W_all``, one weight-gradient GEMM
    ``dW_all += dmods^T c`` into the flat gradient run, and one column sum for the
    biases. Outputs: the modulation matrix (no autograd edge), its gradient buffer and
    ``token``, the scalar each block returns a zero gradient for."""

    @staticmethod
    def forward(ctx, c2, group: FlatParamGroup, runs):
        w0, b0, wn, bn = runs
        d = c2.shape[1]
        W_all = group.compute[w0:w0 + wn].view(-1, d)
        b_all = group.master[b0:b0 + bn]
        cb = c2.detach().to(torch.bfloat16).contiguous()
        mods = gemm(cb, W_all, epi="f32", bias=b_all)
        dmods = torch.zeros_like(mods)
        ctx.save_for_backward(cb)
        ctx.group, ctx.runs, ctx.dmods = group, runs, dmods
        ctx.mark_non_differentiable(mods, dmods)
        return mods, dmods, torch.zeros((), device=c2.device)

    @staticmethod
    def backward(ctx, _dm, _dd, _dtoken):
        (cb,) = ctx.saved_tensors
        g = ctx.group
        w0, b0, wn, bn = ctx.runs
        d = cb.shape[1]
        dm = ctx.dmods.to(torch.bfloat16)
        W_all = g.compute[w0:w0 + wn].view(-1, d)
        dW = g.grad[w0:w0 + wn].view(-1, d)
        gemm(dm, cb, dW, epi="f32_acc", a_t=True, b_t=True)          # dW_all += dm^T c
        g.grad[b0:b0 + bn].add_(ctx.dmods.sum(0))
        # dc = dm W_all, read as dm^T [K, M] and W_all [K, N] (both MN-major, split-K);
        # dm^T rows are padded to a multiple of 8 elements (16 bytes, the TMA row rule)
        M = dm.shape[0]
        Mp = (M + 7) // 8 * 8
        if Mp == M:
            dmT = dm.t().contiguous()
        else:
            dmT = torch.zeros(dm.shape[1], Mp, device=dm.device, dtype=dm.dtype)
            dmT[:, :M] = dm.t()
            dmT = dmT[:, :M]
        dc = gemm(dmT, W_all, epi="f32_acc", a_t=True, b_t=True)
        ctx.dmods = None
        return dc, None, None


class FusedWorldDiT:
    """CUDA execution engine of :class:`~drivedit_b200.models.world_dit.WorldDiT`."""

    def __init__(self, model, group: Optional[FlatParamGroup] = None):
        self.model = model
        if group is None:
            named = model.named_parameters()
            if hasattr(model, "flat_layout"):
                named = model.flat_layout(named)
            group = FlatParamGroup(named)
        self.group = group
        self._runs = False  # modulation weight runs of the group, looked up on first use
        self.recompute = False  # activation checkpointing (TrainConfig.checkpoint_blocks)
        # set by a sharded engine: called with a block's index after its backward, so that
        # block's gradient bucket can be reduced while the rest of the backward runs
        self.grad_ready = None

    def forward(self, model, x_t, t, actions, frame_offset=0, return_aux=False,
                return_features=None, extra_cond=None):
        from ..models.world_dit import patchify, unpatchify

        cfg = model.cfg
        g = self.group
        B, Fr, C, H, W_ = x_t.shape
        d = cfg.d_model
        tok = patchify(x_t, cfg.patch).reshape(-1, cfg.patch_dim).to(torch.bfloat16).contiguous()
        T = tok.shape[0] // B
        x = linear(tok, g.compute_view(model.patch_embed.weight), model.patch_embed.bias,
                   model.patch_embed.weight, model.patch_embed.bias)
        c = model.condition(t, actions, extra_cond)                # [B, F, d] fp32
        c2 = c.reshape(B * Fr, d)
        tab = model.rope.table(Fr, frame_offset).to(x.device)
        bc = BlockCtx(B, T, Fr, T // Fr, d, cfg.n_heads, cfg.d_head, tab, cfg.attention,
                      cfg.sla, cfg.causal)
        bc.recompute = self.recompute and torch.is_grad_enabled()
        bc.grad_ready = self.grad_ready
        feats = None
        aux = torch.zeros((), device=x.device)
        if self._runs is False:
            self._runs = _mod_runs(model, g)
        if self._runs is not None:  # all modulations in one GEMM (+ one backward pair)
            mods, dmods, token = _AllMods.apply(c2, g, self._runs)
            widths = [blk.ada.weight.shape[0] for blk in model.blocks]
        col = 0
        for i, blk in enumerate(model.blocks):
            blk.block_index = i
            if self._runs is not None:
                n = widths[i]
                x, a = _BlockFn.apply(x, mods[:, col:col + n], blk, g, bc, token,
                                      dmods[:, col:col + n])
                col += n
            else:
                mod = blk.ada(c2)                                  # [B*F, 4d] fp32
                x, a = _BlockFn.apply(x, mod, blk, g, bc)
            if blk.moe is not None:
                aux = aux + a * blk.moe.aux_loss_weight
            if return_features is not None and i + 1 == return_features:
                feats = x
        if self._runs is not None:
            fm = _FinalMod.apply(mods[:, col:], dmods[:, col:], token)
        else:
            fm = model.final_ada(c2)
        h, _ = _FinalNorm.apply(x, fm, model.final_norm.weight, bc.tpf, cfg.norm_eps)
        out = linear(h, g.compute_view(model.out_proj.weight), model.out_proj.bias,
                     model.out_proj.weight, model.out_proj.bias)
        v = unpatchify(out.view(B, T, cfg.patch_dim), Fr, C, H, W_, cfg.patch)
        if return_features is not None:
            return v, aux, feats
        return (v, aux) if return_aux else v


class _FinalMod(torch.autograd.Function):
    """The final layer's columns of the batched modulations as a differentiable input of
    the final norm: its gradient lands in the shared buffer, and ``token`` orders the
    batched backward after it."""

    @staticmethod
    def forward(ctx, fm, dfm, token):
        ctx.dfm = dfm
        return fm.clone()

    @staticmethod
    def backward(ctx, g):
        ctx.dfm.add_(g)
        ctx.dfm = None
        return None, None, torch.zeros((), device=g.device)


class _FinalNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mod, w, tpf, eps):
        d = x.shape[1]
        h, r = adaln_rmsnorm(x, w, mod, 0, d, tpf, eps)
        ctx.save_for_backward(x, mod, r)
        ctx.w, ctx.tpf = w, tpf
        return h, r

    @staticmethod
    def backward(ctx, dh, _dr):
        x, mod, r = ctx.saved_tensors
        d = x.shape[1]
        dmod = torch.zeros(mod.shape, device=mod.device, dtype=torch.float32)
        dx = adaln_rmsnorm_bwd(dh.contiguous(), x, r, ctx.w, mod, 0, d, ctx.tpf, dmod,
                               ctx.w.grad, None)
        return dx, dmod, None, None, None


# ----------------------------------------------------------------------------- KV-cached
def _forward_cached_fused(self, model, x_t, t, actions, cache, commit, extra_cond=None):
    """Inference-only forward of a chunk over the cached K/V window (no autograd):
    every block is AdaLN-RMSNorm -> QKV GEMM (rotary by absolute frame) -> K/V into the
    cache window -> flash attention with absolute query/key offsets -> output GEMM with
    residual -> AdaLN-RMSNorm -> SwiGLU GEMM -> down GEMM with residual."""
    from ..models.world_dit import patchify, unpatchify
    from ._ext import ext

    cfg = model.cfg
    g = self.group
    W = g.compute_view
    B, Fc, C, H, W_ = x_t.shape
    d, Hh = cfg.d_model, cfg.n_heads
    tok = patchify(x_t, cfg.patch).reshape(-1, cfg.patch_dim).to(torch.bfloat16).contiguous()
    T = tok.shape[0] // B
    tpf = T // Fc
    x = gemm(tok, W(model.patch_embed.weight), bias=model.patch_embed.bias)
    c2 = model.condition(t, actions, extra_cond).reshape(B * Fc, d)
    tab = model.rope.table(Fc, cache.frames).to(x.device)
    row = cache.reserve(T)
    if self._runs is False:
        self._runs = _mod_runs(model, g)
    mods = None
    if self._runs is not None:  # every modulation of this forward in one GEMM
        w0, b0, wn, bn = self._runs
        mods = gemm(c2.to(torch.bfloat16).contiguous(), g.compute[w0:w0 + wn].view(-1, d),
                    epi="f32", bias=g.master[b0:b0 + bn])
    col = 0
    for blk, lc in zip(model.blocks, cache.layers):
        if mods is not None:
            n = blk.ada.weight.shape[0]
            mod = mods[:, col:col + n]
            col += n
        else:
            mod = blk.ada(c2)
        h1, _ = adaln_rmsnorm(x, blk.norm1.weight, mod, 0, d, tpf)
        qkv = gemm(h1, W(blk.attn.qkv.weight), epi="rope", rope_tab=tab, rope_cols=2 * d,
                   rope_rows_per_seq=T, rope_head_dim=cfg.d_head)
        q3 = qkv.view(B, T, 3 * d)
        lc.k[:, row:row + T].copy_(q3[:, :, d:2 * d])
        lc.v[:, row:row + T].copy_(q3[:, :, 2 * d:])
        cap = lc.k.shape[1]
        k2 = lc.k.view(B * cap, d)[lc.start:]
        v2 = lc.v.view(B * cap, d)[lc.start:]
        S = row + T - lc.start
        o = torch.empty(B * T, d, device=x.device, dtype=torch.bfloat16)
        ext().attn_fwd(qkv, k2, v2, o, None, 0, 0, 0, 0, B, Hh, T, S, T, cap, 1, tpf,
                       lc.pos0 + row, lc.pos0 + lc.start, 1.0 / math.sqrt(cfg.d_head),
                       None, None, None)
        x1 = gemm(o, W(blk.attn.proj.weight), residual=x)
        h2, _ = adaln_rmsnorm(x1, blk.norm2.weight, mod, 2 * d, 3 * d, tpf)
        w13 = W(blk.mlp.w13.weight)
        gu = torch.empty(x.shape[0], w13.shape[0], device=x.device, dtype=torch.bfloat16)
        a = torch.empty(x.shape[0], w13.shape[0] // 2, device=x.device, dtype=torch.bfloat16)
        gemm(h2, w13, gu, epi="swiglu", out2=a)
        x = gemm(a, W(blk.mlp.w3.weight), residual=x1)
    if commit:
        cache.commit(Fc)
    fm = mods[:, col:] if mods is not None else model.final_ada(c2)
    h, _ = adaln_rmsnorm(x, model.final_norm.weight, fm, 0, d, tpf, cfg.norm_eps)
    out = gemm(h, W(model.out_proj.weight), bias=model.out_proj.bias)
    return unpatchify(out.view(B, T, cfg.patch_dim), Fc, C, H, W_, cfg.patch)


FusedWorldDiT.forward_cached = _forward_cached_fused
