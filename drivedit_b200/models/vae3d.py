"""Causal 3-D video VAE with asymmetric (temporal x4, spatial x8) compression.

Same public surface, module tree and checkpoint keys as the reference
``models/vae3d.py``: ``VAE3DConfig`` (:48-112), ``CausalConv3d`` (:119-173),
``CausalConvTranspose3d`` (:176-232), ``ResidualBlock3D`` (:239-285),
``AttentionBlock3D`` (:288-341), ``Downsample3D``/``Upsample3D`` (:344-400),
``VectorQuantizer`` (:407-470), ``LearnablePrior`` (:477-505), ``PerceptualLoss``
(:512-564), ``KLAnnealer`` (:571-624), ``Encoder3D`` (:631-744), ``Decoder3D``
(:751-906), ``VAE3Dv2`` (:913-1212), presets (:1219-1269) and the ``VAE3D`` /
``causal_conv3d`` compatibility names (:1281-1301). Output extents follow the reference
exactly (a stride-2 downsample with kernel 4 and padding 2 maps H to H//2 + 1).

On CUDA every CausalConv3d (including the strided downsamples and the 1x1 skips and
attention projections), every GroupNorm(+SiLU) and the residual adds run on the
hand-written kernels of ``ops/conv3d.py`` in bf16 with channels-last storage; on the CPU
the same modules run the PyTorch operators in the input dtype (the oracle).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint


class QuantizationMode(Enum):
    NONE = "none"
    VQ = "vq"
    FSQ = "fsq"


@dataclass
class VAE3DConfig:
    in_channels: int = 3
    out_channels: int = 3
    latent_dim: int = 8
    temporal_compression: int = 4
    spatial_compression: int = 8
    hidden_dims: List[int] = field(default_factory=lambda: [128, 256, 512, 512])
    num_res_blocks: int = 2
    use_attention: bool = True
    attention_resolution: List[int] = field(default_factory=lambda: [16, 8])
    use_skip_connections: bool = True
    skip_connection_scale: float = 0.5
    quantization_mode: QuantizationMode = QuantizationMode.NONE
    num_codebook_vectors: int = 8192
    codebook_dim: int = 8
    commitment_cost: float = 0.25
    use_kl_annealing: bool = True
    kl_anneal_mode: str = "cyclical"
    kl_cycle_period: int = 10000
    kl_start_beta: float = 0.0
    kl_end_beta: float = 1.0
    kl_free_bits: float = 0.0
    kl_warmup_steps: int = 1000
    use_learnable_prior: bool = False
    prior_hidden_dim: int = 256
    use_hierarchical_latents: bool = False
    num_latent_levels: int = 2
    use_perceptual_loss: bool = True
    perceptual_weight: float = 0.1
    perceptual_layers: List[int] = field(default_factory=lambda: [0, 1, 2, 3])
    use_spectral_norm: bool = False
    latent_dropout: float = 0.0
    gradient_penalty_weight: float = 0.0
    enable_streaming: bool = True
    max_cache_frames: int = 8
    use_gradient_checkpointing: bool = True
    mixed_precision: bool = True


def _use_kernels(x: torch.Tensor) -> bool:
    if not x.is_cuda:
        return False
    from ..ops._ext import available

    return available()


def _maybe_sn(conv: nn.Module, on: bool) -> nn.Module:
    return nn.utils.spectral_norm(conv) if on else conv


# ----------------------------------------------------------------------------- convs
class CausalConv3d(nn.Module):
    """Time-causal conv: ``kt - 1`` zero frames in front (or, when streaming, the last
    ``kt - 1`` input frames of the previous call), symmetric spatial padding."""

    def __init__(self, in_channels, out_channels, kernel_size=(3, 3, 3), stride=(1, 1, 1),
                 bias=True, enable_streaming=True, use_spectral_norm=False):
        super().__init__()
        kt, kh, kw = kernel_size
        st, sh, sw = stride if isinstance(stride, tuple) else (stride,) * 3
        self.kernel_size = tuple(kernel_size)
        self.stride = (st, sh, sw)
        self.enable_streaming = enable_streaming
        self.temporal_padding = kt - 1
        self.pad_h, self.pad_w = kh // 2, kw // 2
        self.conv = _maybe_sn(nn.Conv3d(in_channels, out_channels, kernel_size, stride=(st, sh, sw),
                                        padding=(0, self.pad_h, self.pad_w), bias=bias),
                              use_spectral_norm)
        self._cache: Optional[torch.Tensor] = None

    def reset_cache(self):
        self._cache = None

    def forward(self, x: torch.Tensor, streaming: bool = False,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        tpad = self.temporal_padding
        if streaming and self.enable_streaming:
            if self._cache is not None:
                x = torch.cat([self._cache.to(x.dtype), x], dim=2)
            if self.temporal_padding > 0:
                self._cache = x[:, :, -self.temporal_padding:].detach()
            tpad = 0
        if _use_kernels(x) and not hasattr(self.conv, "weight_orig"):
            from ..ops.conv3d import causal_conv3d

            return causal_conv3d(x, self.conv.weight, self.conv.bias, self.stride,
                                 temporal_pad=tpad, residual=residual)
        if tpad > 0:
            x = F.pad(x, (0, 0, 0, 0, tpad, 0))
        y = self.conv(x)
        return y if residual is None else y + residual


class CausalConvTranspose3d(nn.Module):
    """Trilinear upsampling followed by a causal (kt, 3, 3) convolution."""

    def __init__(self, in_channels, out_channels, kernel_size=(4, 4, 4), stride=(2, 2, 2),
                 bias=True, use_spectral_norm=False):
        super().__init__()
        kt, kh, kw = kernel_size
        st, sh, sw = stride if isinstance(stride, tuple) else (stride,) * 3
        self.kernel_size = (kt, kh, kw)
        self.stride = (st, sh, sw)
        self.upsample_t, self.upsample_s = st, sh
        self.conv = _maybe_sn(nn.Conv3d(in_channels, out_channels, kernel_size=(kt, 3, 3),
                                        padding=(0, 1, 1), bias=bias), use_spectral_norm)

    def forward(self, x, target_size=None):
        B, C, T, H, W = x.shape
        if target_size is None:
            target_size = (T * self.upsample_t, H * self.upsample_s, W * self.upsample_s)
        out = F.interpolate(x, size=tuple(target_size), mode="trilinear", align_corners=False)
        if _use_kernels(out) and not hasattr(self.conv, "weight_orig"):
            from ..ops.conv3d import causal_conv3d

            return causal_conv3d(out, self.conv.weight, self.conv.bias)
        if self.kernel_size[0] > 1:
            out = F.pad(out, (0, 0, 0, 0, self.kernel_size[0] - 1, 0))
        return self.conv(out)


def _group_norm(norm: nn.GroupNorm, x: torch.Tensor, silu: bool) -> torch.Tensor:
    if _use_kernels(x):
        from ..ops.conv3d import group_norm_silu

        return group_norm_silu(x, norm.num_groups, norm.weight, norm.bias, norm.eps, silu)
    h = norm(x)
    return F.silu(h) if silu else h


class ResidualBlock3D(nn.Module):
    def __init__(self, in_channels, out_channels=None, kernel_size=(3, 3, 3), dropout=0.0,
                 use_spectral_norm=False, enable_streaming=True):
        super().__init__()
        out_channels = out_channels or in_channels
        self.norm1 = nn.GroupNorm(min(32, in_channels), in_channels)
        self.conv1 = CausalConv3d(in_channels, out_channels, kernel_size,
                                  use_spectral_norm=use_spectral_norm,
                                  enable_streaming=enable_streaming)
        self.norm2 = nn.GroupNorm(min(32, out_channels), out_channels)
        self.conv2 = CausalConv3d(out_channels, out_channels, kernel_size,
                                  use_spectral_norm=use_spectral_norm,
                                  enable_streaming=enable_streaming)
        self.dropout = nn.Dropout3d(dropout) if dropout > 0 else nn.Identity()
        self.skip = (nn.Conv3d(in_channels, out_channels, 1) if in_channels != out_channels
                     else nn.Identity())

    def _skip(self, x):
        if isinstance(self.skip, nn.Conv3d) and _use_kernels(x):
            from ..ops.conv3d import causal_conv3d

            return causal_conv3d(x, self.skip.weight, self.skip.bias)
        return self.skip(x)

    def forward(self, x, streaming: bool = False):
        residual = self._skip(x)
        h = self.conv1(_group_norm(self.norm1, x, True), streaming=streaming)
        h = self.dropout(_group_norm(self.norm2, h, True))
        # the residual add is fused into the second convolution's epilogue on CUDA
        return self.conv2(h, streaming=streaming, residual=residual)


class AttentionBlock3D(nn.Module):
    """Multi-head self-attention over all T*H*W positions (no mask)."""

    def __init__(self, channels, num_heads=8, use_spectral_norm=False):
        super().__init__()
        assert channels % num_heads == 0
        self.channels, self.num_heads = channels, num_heads
        self.head_dim = channels // num_heads
        self.norm = nn.GroupNorm(min(32, channels), channels)
        self.qkv = _maybe_sn(nn.Conv3d(channels, 3 * channels, 1), use_spectral_norm)
        self.proj = _maybe_sn(nn.Conv3d(channels, channels, 1), use_spectral_norm)
        self.scale = self.head_dim ** -0.5

    def forward(self, x):
        B, C, T, H, W = x.shape
        P, nh, hd = T * H * W, self.num_heads, self.head_dim
        h = _group_norm(self.norm, x, False)
        kern = _use_kernels(x) and not hasattr(self.qkv, "weight_orig")
        if kern:
            from ..ops.conv3d import causal_conv3d, from_cl, to_cl

            qkv = to_cl(causal_conv3d(h, self.qkv.weight, self.qkv.bias)).view(B, P, 3, nh, hd)
            if hd == 64 and not (torch.is_grad_enabled() and (x.requires_grad or self.qkv.weight.requires_grad)):
                from ..ops.attention_kernels import flash_attention

                o, _ = flash_attention(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], "none",
                                       scale=self.scale)
            else:
                q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
                o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2)
            o = o.reshape(B, T, H, W, C)
            return causal_conv3d(from_cl(o), self.proj.weight, self.proj.bias, residual=x)
        qkv = self.qkv(h).view(B, 3, nh, hd, P).permute(1, 0, 2, 4, 3)
        o = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2])
        o = o.permute(0, 1, 3, 2).reshape(B, C, T, H, W)
        return self.proj(o) + x


class Downsample3D(nn.Module):
    def __init__(self, in_channels, out_channels, temporal_stride=1, spatial_stride=2,
                 use_spectral_norm=False, enable_streaming=True):
        super().__init__()
        kt = temporal_stride * 2 if temporal_stride > 1 else 3
        ks = spatial_stride * 2 if spatial_stride > 1 else 3
        self.conv = CausalConv3d(in_channels, out_channels, kernel_size=(kt, ks, ks),
                                 stride=(temporal_stride, spatial_stride, spatial_stride),
                                 use_spectral_norm=use_spectral_norm,
                                 enable_streaming=enable_streaming)

    def forward(self, x, streaming: bool = False):
        return self.conv(x, streaming=streaming)


class Upsample3D(nn.Module):
    def __init__(self, in_channels, out_channels, temporal_stride=1, spatial_stride=2,
                 use_spectral_norm=False):
        super().__init__()
        self.temporal_stride, self.spatial_stride = temporal_stride, spatial_stride
        kt = temporal_stride * 2 if temporal_stride > 1 else 3
        ks = spatial_stride * 2 if spatial_stride > 1 else 3
        self.conv = CausalConvTranspose3d(in_channels, out_channels, kernel_size=(kt, ks, ks),
                                          stride=(temporal_stride, spatial_stride, spatial_stride),
                                          use_spectral_norm=use_spectral_norm)

    def forward(self, x, target_size=None):
        return self.conv(x, target_size=target_size)


# ----------------------------------------------------------------------------- latent tools
class VectorQuantizer(nn.Module):
    """Codebook quantiser (VQ-VAE, van den Oord et al. 2017) whose codebook follows the
    exponential moving average of the vectors assigned to each code (Razavi et al. 2019).

    Forward: each latent vector (channel dim 1) snaps to its nearest code; the output
    passes gradients straight through to the encoder; the loss is the codebook term
    plus ``commitment_cost`` times the commitment term. The EMA update runs in one pass
    over the assignments: ``bincount`` gives the per-code counts and ``index_add_`` the
    per-code sums (no one-hot matrix), then the counts are Laplace-smoothed so that an
    unused code keeps a finite centroid.
    """

    def __init__(self, num_embeddings, embedding_dim, commitment_cost=0.25, decay=0.99,
                 epsilon=1e-5):
        super().__init__()
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        self.commitment_cost, self.decay, self.epsilon = commitment_cost, decay, epsilon
        self.embeddings = nn.Embedding(num_embeddings, embedding_dim)
        bound = 1.0 / num_embeddings
        with torch.no_grad():
            self.embeddings.weight.uniform_(-bound, bound)
        self.register_buffer("ema_cluster_size", torch.zeros(num_embeddings))
        self.register_buffer("ema_w", self.embeddings.weight.detach().clone())

    def assign(self, vectors: torch.Tensor) -> torch.Tensor:
        """Index of the nearest code for each row of ``vectors [N, C]``."""
        code = self.embeddings.weight
        # |v - e|^2 = |v|^2 - 2 v.e + |e|^2; |v|^2 is the same for every code of a row
        score = torch.addmm(code.pow(2).sum(1)[None, :], vectors, code.t(), alpha=-2.0)
        return score.argmin(dim=1)

    @torch.no_grad()
    def _ema_update(self, vectors: torch.Tensor, idx: torch.Tensor) -> None:
        K, keep = self.num_embeddings, self.decay
        counts = torch.bincount(idx, minlength=K).to(vectors.dtype)
        sums = torch.zeros_like(self.ema_w).index_add_(0, idx, vectors.to(self.ema_w.dtype))
        self.ema_cluster_size.lerp_(counts, 1.0 - keep)
        self.ema_w.lerp_(sums, 1.0 - keep)
        total = self.ema_cluster_size.sum()
        smoothed = (self.ema_cluster_size + self.epsilon) * (total / (total + K * self.epsilon))
        self.embeddings.weight.copy_(self.ema_w / smoothed[:, None])

    def forward(self, z):
        C = z.shape[1]
        channels_last = z.movedim(1, -1)
        vectors = channels_last.reshape(-1, C)
        idx = self.assign(vectors)
        quant = self.embeddings(idx).view_as(channels_last).movedim(-1, 1)
        codebook_term = (quant - z.detach()).pow(2).mean()
        commitment_term = (z - quant.detach()).pow(2).mean()
        loss = codebook_term + self.commitment_cost * commitment_term
        out = z + (quant - z).detach()
        if self.training:
            self._ema_update(vectors.detach(), idx)
        return out, loss, idx.view(channels_last.shape[:-1])


class LearnablePrior(nn.Module):
    """Learned Gaussian prior over the latent grid: a learned base tensor through a
    small conv net gives (mean, log-variance). The prior does not depend on the sample,
    so it is computed once and broadcast over the batch."""

    def __init__(self, latent_dim, hidden_dim=256, latent_shape=(2, 32, 32)):
        super().__init__()
        self.latent_dim, self.latent_shape = latent_dim, latent_shape
        self.base_embedding = nn.Parameter(0.02 * torch.randn(1, hidden_dim, *latent_shape))
        self.net = nn.Sequential(nn.Conv3d(hidden_dim, hidden_dim, 3, padding=1), nn.SiLU(),
                                 nn.Conv3d(hidden_dim, 2 * latent_dim, 3, padding=1))

    def forward(self, batch_size, device):
        params = self.net(self.base_embedding.to(device))
        mean, logvar = params.split(self.latent_dim, dim=1)
        return (mean.expand(batch_size, *mean.shape[1:]),
                logvar.expand(batch_size, *logvar.shape[1:]))


class PerceptualLoss(nn.Module):
    """Feature-matching loss over a frozen random conv pyramid, softplus layer weights."""

    def __init__(self, in_channels=3, feature_channels=None, normalize=True):
        super().__init__()
        feature_channels = feature_channels or [64, 128, 256, 256]
        self.normalize = normalize
        layers, ch = [], in_channels
        for oc in feature_channels:
            layers += [nn.Conv3d(ch, oc, 3, stride=2, padding=1), nn.SiLU(),
                       nn.Conv3d(oc, oc, 3, padding=1), nn.SiLU()]
            ch = oc
        self.features = nn.Sequential(*layers)
        self.layer_weights = nn.Parameter(torch.ones(len(feature_channels)))
        for p in self.features.parameters():
            p.requires_grad = False

    def forward(self, pred, target):
        if self.normalize:
            pred, target = pred * 2 - 1, target * 2 - 1
        dt = self.features[0].weight.dtype
        a, b = pred.to(dt), target.to(dt)
        losses = []
        for i, layer in enumerate(self.features):
            a, b = layer(a), layer(b)
            if (i + 1) % 4 == 0:
                losses.append(F.mse_loss(a, b) * F.softplus(self.layer_weights[len(losses)]))
        return sum(losses) / len(losses)


class KLAnnealer:
    """Weight of the KL term by training step, on the shared piecewise schedule:
    ``constant`` (``end_beta``), ``linear`` (warm-up from ``start_beta`` to ``end_beta``
    over ``warmup_steps``, then hold) or ``cyclical`` (a half-cosine ramp from
    ``start_beta`` towards ``end_beta`` repeated every ``cycle_period`` steps, the
    cyclical schedule of Fu et al. 2019). ``free_bits`` > 0 subtracts a per-dimension
    allowance from the KL before it is weighted (no gradient below the allowance)."""

    def __init__(self, mode="cyclical", cycle_period=10000, start_beta=0.0, end_beta=1.0,
                 warmup_steps=1000, free_bits=0.0):
        from ..utils.schedules import PiecewiseSchedule, Segment

        self.mode, self.cycle_period = mode, cycle_period
        self.start_beta, self.end_beta = start_beta, end_beta
        self.warmup_steps, self.free_bits = warmup_steps, free_bits
        self.step = 0
        if mode == "constant":
            segs, period = [Segment(None, end_beta, end_beta, "constant")], None
        elif mode == "linear":
            segs = [Segment(max(1, warmup_steps), start_beta, end_beta, "linear", "warmup"),
                    Segment(None, end_beta, end_beta, "constant", "hold")]
            period = None
        elif mode == "cyclical":
            segs, period = [Segment(cycle_period, start_beta, end_beta, "cosine")], cycle_period
        else:
            raise ValueError(f"Unknown annealing mode: {mode}")
        self.schedule = PiecewiseSchedule(segs, period)

    def get_beta(self) -> float:
        return self.schedule(self.step)

    def update(self):
        self.step += 1

    def warm_restart(self):
        self.schedule.restart(self.step)

    def apply_free_bits(self, kl_per_dim):
        if self.free_bits <= 0:
            return kl_per_dim
        return (kl_per_dim - self.free_bits).clamp_min(0.0)


# ----------------------------------------------------------------------------- encoder / decoder
def _strides(total: int, levels: int) -> List[int]:
    out, rem = [], total
    for _ in range(levels):
        if rem >= 2:
            out.append(2)
            rem //= 2
        else:
            out.append(1)
    return out


class Encoder3D(nn.Module):
    def __init__(self, config: VAE3DConfig):
        super().__init__()
        c = self.config = config
        hd = c.hidden_dims
        L = len(hd) - 1
        self.temporal_strides = _strides(c.temporal_compression, L)
        self.spatial_strides = _strides(c.spatial_compression, L)
        sn, stm = c.use_spectral_norm, c.enable_streaming
        self.conv_in = CausalConv3d(c.in_channels, hd[0], (3, 3, 3), use_spectral_norm=sn,
                                    enable_streaming=stm)
        self.down_blocks = nn.ModuleList()
        res = c.spatial_compression * (2 ** L)
        for i in range(L):
            ind, outd = hd[i], hd[i + 1]
            blocks = nn.ModuleList([ResidualBlock3D(ind if j == 0 else outd, outd, use_spectral_norm=sn,
                                                    enable_streaming=stm)
                                    for j in range(c.num_res_blocks)])
            down = Downsample3D(outd, outd, self.temporal_strides[i], self.spatial_strides[i],
                                use_spectral_norm=sn, enable_streaming=stm)
            res //= self.spatial_strides[i]
            attn = (AttentionBlock3D(outd, use_spectral_norm=sn)
                    if c.use_attention and res in c.attention_resolution else nn.Identity())
            self.down_blocks.append(nn.ModuleDict({"res_blocks": blocks, "downsample": down,
                                                   "attn": attn}))
        fd = hd[-1]
        self.mid_block1 = ResidualBlock3D(fd, use_spectral_norm=sn)
        self.mid_attn = AttentionBlock3D(fd, use_spectral_norm=sn) if c.use_attention else nn.Identity()
        self.mid_block2 = ResidualBlock3D(fd, use_spectral_norm=sn)
        self.norm_out = nn.GroupNorm(min(32, fd), fd)
        self.conv_out = CausalConv3d(fd, 2 * c.latent_dim, (3, 3, 3), use_spectral_norm=sn)

    def _compute_strides(self, total_compression, num_levels):
        return _strides(total_compression, num_levels)

    def forward(self, x, return_skips: bool = False, streaming: bool = False):
        skips = []
        h = self.conv_in(x, streaming=streaming)
        for blk in self.down_blocks:
            for rb in blk["res_blocks"]:
                h = rb(h, streaming=streaming)
            if return_skips:
                skips.append(h)
            h = blk["downsample"](h, streaming=streaming)
            h = blk["attn"](h)
        h = self.mid_block1(h, streaming=streaming)
        h = self.mid_attn(h)
        h = self.mid_block2(h, streaming=streaming)
        h = self.conv_out(_group_norm(self.norm_out, h, True), streaming=streaming)
        mean, logvar = h.chunk(2, dim=1)
        return (mean, logvar, skips) if return_skips else (mean, logvar)


class Decoder3D(nn.Module):
    def __init__(self, config: VAE3DConfig):
        super().__init__()
        c = self.config = config
        hd = list(reversed(c.hidden_dims))
        L = self.num_levels = len(hd) - 1
        self.temporal_strides = list(reversed(_strides(c.temporal_compression, L)))
        self.spatial_strides = list(reversed(_strides(c.spatial_compression, L)))
        sn = c.use_spectral_norm
        self.conv_in = CausalConv3d(c.latent_dim, hd[0], (3, 3, 3), use_spectral_norm=sn)
        self.mid_block1 = ResidualBlock3D(hd[0], use_spectral_norm=sn)
        self.mid_attn = AttentionBlock3D(hd[0], use_spectral_norm=sn) if c.use_attention else nn.Identity()
        self.mid_block2 = ResidualBlock3D(hd[0], use_spectral_norm=sn)
        self.up_blocks = nn.ModuleList()
        self.skip_weights = nn.ParameterList() if c.use_skip_connections else None
        res = c.spatial_compression // (2 ** L) * 2
        for i in range(L):
            ind, outd = hd[i], hd[i + 1]
            up = Upsample3D(ind, ind, self.temporal_strides[i], self.spatial_strides[i],
                            use_spectral_norm=sn)
            res *= self.spatial_strides[i]
            fuse = ind + (ind if c.use_skip_connections else 0)
            blocks = nn.ModuleList([ResidualBlock3D(fuse if j == 0 else outd, outd, use_spectral_norm=sn)
                                    for j in range(c.num_res_blocks)])
            attn = (AttentionBlock3D(outd, use_spectral_norm=sn)
                    if c.use_attention and res in c.attention_resolution else nn.Identity())
            if c.use_skip_connections:
                self.skip_weights.append(nn.Parameter(torch.tensor(c.skip_connection_scale)))
            self.up_blocks.append(nn.ModuleDict({"upsample": up, "res_blocks": blocks, "attn": attn}))
        fd = hd[-1]
        self.norm_out = nn.GroupNorm(min(32, fd), fd)
        self.conv_out = CausalConv3d(fd, c.out_channels, (3, 3, 3), use_spectral_norm=sn)

    def _compute_strides(self, total_compression, num_levels):
        return _strides(total_compression, num_levels)

    def _compute_target_sizes(self, latent_shape, output_shape=None):
        Tl, Hl, Wl = latent_shape
        if output_shape is not None:
            T, H, W = output_shape
        else:
            T = Tl * self.config.temporal_compression
            H = Hl * self.config.spatial_compression
            W = Wl * self.config.spatial_compression
        sizes = [(T, H, W)]
        for i in range(self.num_levels - 1, -1, -1):
            T, H, W = T // self.temporal_strides[i], H // self.spatial_strides[i], W // self.spatial_strides[i]
            sizes.insert(0, (T, H, W))
        return sizes[1:]

    def forward(self, z, skips=None, output_shape=None):
        targets = self._compute_target_sizes(tuple(z.shape[2:]), output_shape)
        h = self.conv_in(z)
        h = self.mid_block2(self.mid_attn(self.mid_block1(h)))
        if skips is not None:
            skips = list(reversed(skips))
        for i, blk in enumerate(self.up_blocks):
            h = blk["upsample"](h, target_size=targets[i])
            if self.skip_weights is not None:
                if skips is not None:
                    s = skips[i]
                    if s.shape[2:] != h.shape[2:]:
                        s = F.interpolate(s, size=h.shape[2:], mode="trilinear", align_corners=False)
                    h = torch.cat([h, (s * self.skip_weights[i]).to(h.dtype)], dim=1)
                else:
                    # decoding latents alone (sampling, streaming): the skip half of the
                    # fused input is zero, so the same weights apply (the reference
                    # concatenates nothing here and its res-blocks then see too few channels)
                    h = torch.cat([h, torch.zeros_like(h)], dim=1)
            for rb in blk["res_blocks"]:
                h = rb(h)
            h = blk["attn"](h)
        return self.conv_out(_group_norm(self.norm_out, h, True))


# ----------------------------------------------------------------------------- VAE
class VAE3Dv2(nn.Module):
    def __init__(self, config: Optional[VAE3DConfig] = None, **kwargs):
        super().__init__()
        if config is None:
            config = VAE3DConfig(**kwargs)
        self.config = config
        c = config
        self.encoder = Encoder3D(c)
        self.decoder = Decoder3D(c)
        if c.quantization_mode == QuantizationMode.VQ:
            self.quantizer = VectorQuantizer(c.num_codebook_vectors, c.codebook_dim, c.commitment_cost)
            if c.latent_dim != c.codebook_dim:
                self.pre_quant = nn.Conv3d(c.latent_dim, c.codebook_dim, 1)
                self.post_quant = nn.Conv3d(c.codebook_dim, c.latent_dim, 1)
            else:
                self.pre_quant = self.post_quant = nn.Identity()
        else:
            self.quantizer = None
        self.prior = LearnablePrior(c.latent_dim, c.prior_hidden_dim) if c.use_learnable_prior else None
        self.perceptual = PerceptualLoss(c.in_channels, normalize=True) if c.use_perceptual_loss else None
        self.kl_annealer = KLAnnealer(c.kl_anneal_mode, c.kl_cycle_period, c.kl_start_beta,
                                      c.kl_end_beta, c.kl_warmup_steps, c.kl_free_bits)
        self.latent_dropout = nn.Dropout(c.latent_dropout) if c.latent_dropout > 0 else nn.Identity()
        self._streaming_mode = False

    # streaming
    def enable_streaming(self):
        self._streaming_mode = True
        self._reset_caches()

    def disable_streaming(self):
        self._streaming_mode = False
        self._reset_caches()

    def _reset_caches(self):
        for m in self.modules():
            if isinstance(m, CausalConv3d):
                m.reset_cache()

    def encode(self, x, return_skips: bool = False):
        if self.config.use_gradient_checkpointing and self.training and torch.is_grad_enabled():
            return checkpoint(self.encoder, x, return_skips, self._streaming_mode, use_reentrant=False)
        return self.encoder(x, return_skips=return_skips, streaming=self._streaming_mode)

    def decode(self, z, skips=None, output_shape=None):
        if self.config.use_gradient_checkpointing and self.training and torch.is_grad_enabled():
            return checkpoint(self.decoder, z, skips, output_shape, use_reentrant=False)
        return self.decoder(z, skips=skips, output_shape=output_shape)

    def reparameterize(self, mean, logvar, deterministic: bool = False):
        if deterministic or not self.training:
            return mean
        z = mean + torch.randn_like(mean) * torch.exp(0.5 * logvar)
        return self.latent_dropout(z)

    def quantize(self, z):
        if self.quantizer is None:
            return z, None, None
        zq, loss, idx = self.quantizer(self.pre_quant(z))
        return self.post_quant(zq), loss, idx

    def forward(self, x, return_loss: bool = True, deterministic: bool = False) -> Dict[str, Any]:
        shape = tuple(x.shape[2:])
        if self.config.use_skip_connections:
            mean, logvar, skips = self.encode(x, return_skips=True)
        else:
            (mean, logvar), skips = self.encode(x), None
        z = self.reparameterize(mean, logvar, deterministic)
        z, vq_loss, idx = self.quantize(z)
        recon = self.decode(z, skips=skips, output_shape=shape)
        out = {"recon": recon, "mean": mean, "logvar": logvar, "z": z}
        if idx is not None:
            out["indices"] = idx
        if return_loss:
            out.update(self.compute_loss(x, recon, mean, logvar, vq_loss))
        return out

    def compute_loss(self, x, recon, mean, logvar, vq_loss=None) -> Dict[str, torch.Tensor]:
        recon, mean, logvar = recon.float(), mean.float(), logvar.float()
        x = x.float()
        losses = {"recon_loss": F.mse_loss(recon, x), "l1_loss": F.l1_loss(recon, x)}
        if self.prior is not None:
            pm, plv = self.prior(x.size(0), x.device)
            kl = 0.5 * (plv - logvar + (logvar.exp() + (mean - pm).pow(2)) / plv.exp() - 1)
        else:
            kl = -0.5 * (1 + logvar - mean.pow(2) - logvar.exp())
        kl = self.kl_annealer.apply_free_bits(kl).mean()
        beta = self.kl_annealer.get_beta()
        losses["kl_loss"] = kl
        losses["kl_loss_weighted"] = beta * kl
        losses["beta"] = torch.tensor(beta, device=x.device)
        total = losses["recon_loss"] + losses["kl_loss_weighted"]
        if vq_loss is not None:
            losses["vq_loss"] = vq_loss
            total = total + vq_loss
        if self.perceptual is not None:
            losses["perceptual_loss"] = self.perceptual(recon, x)
            total = total + self.config.perceptual_weight * losses["perceptual_loss"]
        losses["total_loss"] = total
        return losses

    @torch.no_grad()
    def sample(self, num_samples, device, latent_shape=None):
        if latent_shape is None:
            latent_shape = (8 // self.config.temporal_compression, 256 // self.config.spatial_compression,
                            256 // self.config.spatial_compression)
        if self.prior is not None:
            mean, logvar = self.prior(num_samples, device)
        else:
            mean = torch.zeros(num_samples, self.config.latent_dim, *latent_shape, device=device)
            logvar = torch.zeros_like(mean)
        z, _, _ = self.quantize(self.reparameterize(mean, logvar))
        return self.decode(z)

    def encode_frame(self, frame):
        if not self._streaming_mode:
            self.enable_streaming()
        return self.encode(frame, return_skips=False)

    def decode_frame(self, z):
        return self.decode(z)

    def training_step(self):
        self.kl_annealer.update()

    def get_latent_shape(self, input_shape):
        T, H, W = input_shape
        return (T // self.config.temporal_compression, H // self.config.spatial_compression,
                W // self.config.spatial_compression)

    @classmethod
    def from_config(cls, config_dict: Dict[str, Any]) -> "VAE3Dv2":
        d = dict(config_dict)
        if isinstance(d.get("quantization_mode"), str):
            d["quantization_mode"] = QuantizationMode(d["quantization_mode"])
        return cls(VAE3DConfig(**d))

    @classmethod
    def from_pretrained_v1(cls, v1_state_dict, config=None) -> "VAE3Dv2":
        """Shape-matched partial load (keys whose name and shape agree)."""
        model = cls(config)
        own = model.state_dict()
        loaded = {k: v for k, v in v1_state_dict.items() if k in own and own[k].shape == v.shape}
        own.update(loaded)
        model.load_state_dict(own, strict=False)
        model.loaded_keys = sorted(loaded)
        return model


def get_default_config() -> VAE3DConfig:
    return VAE3DConfig()


def get_minimal_config() -> VAE3DConfig:
    return VAE3DConfig(hidden_dims=[64, 128, 256], num_res_blocks=1, temporal_compression=2,
                       spatial_compression=4, use_attention=False, use_skip_connections=False,
                       use_perceptual_loss=False, use_gradient_checkpointing=False)


def get_high_quality_config() -> VAE3DConfig:
    return VAE3DConfig(hidden_dims=[128, 256, 512, 512], num_res_blocks=3, temporal_compression=4,
                       spatial_compression=8, use_attention=True, attention_resolution=[32, 16, 8],
                       use_skip_connections=True, skip_connection_scale=0.5, use_kl_annealing=True,
                       kl_anneal_mode="cyclical", use_learnable_prior=True, use_perceptual_loss=True,
                       perceptual_weight=0.1, use_gradient_checkpointing=True)


def get_vqvae_config() -> VAE3DConfig:
    return VAE3DConfig(hidden_dims=[128, 256, 512, 512], num_res_blocks=2,
                       quantization_mode=QuantizationMode.VQ, num_codebook_vectors=8192,
                       codebook_dim=8, commitment_cost=0.25, use_skip_connections=True,
                       use_perceptual_loss=True)


VAE3D = VAE3Dv2
Encoder3D_v2 = Encoder3D
Decoder3D_v2 = Decoder3D


def causal_conv3d(in_channels, out_channels, kernel_size=(3, 3, 3), stride=1, bias=True) -> CausalConv3d:
    st = (stride,) * 3 if isinstance(stride, int) else tuple(stride)
    return CausalConv3d(in_channels, out_channels, kernel_size, stride=st, bias=bias)
