"""Frozen V-JEPA / ViT video teacher for representation alignment (REPA).

Same module tree, keys and call contract as the reference ``core/vjepa_backbone.py``:
``VJEPAConfig`` (:22-52), ``PatchEmbed3D`` (tubelet conv, :55-89), ``VJEPAAttentionBlock``
(pre-norm MHSA + GELU MLP, :92-131), ``VJEPAEncoder`` (pos-embed, CLS token, intermediate
features of ``extract_layers``, :134-226), ``VJEPABackbone`` (frozen, ImageNet
normalisation, preprocess, ``from_pretrained``, :229-400) and ``create_vjepa_backbone``
(:403-446). ``image_size`` may also be an ``(H, W)`` pair (e.g. 256 x 512 driving frames).

On CUDA the no-grad forward runs on the hand-written kernels: the tubelet embedding as
one GEMM over patchified video, LayerNorm kernel, QKV GEMM (+bias), flash attention
(no mask, any sequence length), output GEMM with bias and the residual fused, fc1 GEMM
with the bias+GELU epilogue, fc2 GEMM with bias+residual. Weights are cast to bf16 once.
"""
from __future__ import annotations

import math
import warnings
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple, Union

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class VJEPAConfig:
    embed_dim: int = 1024
    num_layers: int = 24
    num_heads: int = 16
    mlp_ratio: float = 4.0
    patch_size: int = 16
    tubelet_size: int = 2
    num_frames: int = 16
    image_size: Union[int, Tuple[int, int]] = 224
    extract_layers: List[int] = field(default_factory=lambda: [18, 19, 20, 21, 22, 23])
    pool_type: str = "mean"
    use_fp16: bool = True
    gradient_checkpointing: bool = False

    def __post_init__(self):
        self.d_head = self.embed_dim // self.num_heads
        self.mlp_dim = int(self.embed_dim * self.mlp_ratio)
        h, w = self.image_hw
        self.num_spatial_patches = (h // self.patch_size) * (w // self.patch_size)
        self.num_temporal_patches = self.num_frames // self.tubelet_size
        self.num_patches = self.num_spatial_patches * self.num_temporal_patches

    @property
    def image_hw(self) -> Tuple[int, int]:
        s = self.image_size
        return (s, s) if isinstance(s, int) else tuple(s)


class PatchEmbed3D(nn.Module):
    def __init__(self, image_size=224, patch_size=16, tubelet_size=2, in_channels=3, embed_dim=768):
        super().__init__()
        self.image_size, self.patch_size, self.tubelet_size = image_size, patch_size, tubelet_size
        hw = (image_size, image_size) if isinstance(image_size, int) else tuple(image_size)
        self.num_spatial_patches = (hw[0] // patch_size) * (hw[1] // patch_size)
        self.proj = nn.Conv3d(in_channels, embed_dim, kernel_size=(tubelet_size, patch_size, patch_size),
                              stride=(tubelet_size, patch_size, patch_size))

    def forward(self, x):
        return self.proj(x).flatten(2).transpose(1, 2)


class VJEPAAttentionBlock(nn.Module):
    def __init__(self, dim, num_heads, mlp_ratio=4.0, dropout=0.0):
        super().__init__()
        self.dim, self.num_heads = dim, num_heads
        self.d_head = dim // num_heads
        self.norm1 = nn.LayerNorm(dim)
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)
        self.norm2 = nn.LayerNorm(dim)
        m = int(dim * mlp_ratio)
        self.mlp = nn.Sequential(nn.Linear(dim, m), nn.GELU(), nn.Dropout(dropout), nn.Linear(m, dim),
                                 nn.Dropout(dropout))

    def forward(self, x):
        B, N, D = x.shape
        q, k, v = self.qkv(self.norm1(x)).reshape(B, N, 3, self.num_heads, self.d_head).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, N, D)
        x = x + self.proj(o)
        return x + self.mlp(self.norm2(x))


class VJEPAEncoder(nn.Module):
    def __init__(self, config: VJEPAConfig):
        super().__init__()
        self.config = config
        self.patch_embed = PatchEmbed3D(config.image_size, config.patch_size, config.tubelet_size,
                                        embed_dim=config.embed_dim)
        self.pos_embed = nn.Parameter(torch.zeros(1, config.num_patches, config.embed_dim))
        self.cls_token = nn.Parameter(torch.zeros(1, 1, config.embed_dim))
        self.blocks = nn.ModuleList([VJEPAAttentionBlock(config.embed_dim, config.num_heads, config.mlp_ratio)
                                     for _ in range(config.num_layers)])
        self.norm = nn.LayerNorm(config.embed_dim)
        nn.init.trunc_normal_(self.pos_embed, std=0.02)
        nn.init.trunc_normal_(self.cls_token, std=0.02)
        self._bf16: Optional[Dict[str, torch.Tensor]] = None

    def _interpolate_pos_embed(self, n: int) -> torch.Tensor:
        if n == self.pos_embed.shape[1]:
            return self.pos_embed
        return F.interpolate(self.pos_embed.transpose(1, 2), size=n, mode="linear",
                             align_corners=False).transpose(1, 2)

    def forward(self, x, return_intermediate: bool = True, max_layer: Optional[int] = None):
        """``max_layer``: stop after that block (intermediate features only; 'final' /
        'pooled' / 'patch_features' are then taken from that block's output)."""
        if x.is_cuda and not torch.is_grad_enabled():
            from ..ops._ext import available

            if available() and self.config.embed_dim % 256 == 0 and self.config.d_head == 64:
                return self._forward_fused(x, return_intermediate, max_layer)
        B = x.shape[0]
        x = self.patch_embed(x)
        x = x + self._interpolate_pos_embed(x.shape[1]).to(x.dtype)
        x = torch.cat([self.cls_token.expand(B, -1, -1).to(x.dtype), x], 1)
        inter = {}
        last = len(self.blocks) - 1 if max_layer is None else max_layer
        for i, blk in enumerate(self.blocks[:last + 1]):
            x = blk(x)
            if return_intermediate and i in self.config.extract_layers:
                inter[f"layer_{i}"] = x[:, 1:]
        x = self.norm(x)
        return {"final": x[:, 0], "pooled": x[:, 1:].mean(1), "patch_features": x[:, 1:],
                "intermediate": inter}

    # ------------------------------------------------------------------ fused path
    def _weights(self):
        if self._bf16 is None or next(iter(self._bf16.values())).device != self.pos_embed.device:
            self._bf16 = {n: p.detach().to(torch.bfloat16).contiguous()
                          for n, p in self.named_parameters() if p.dim() >= 2}
        return self._bf16

    @torch.no_grad()
    def _forward_fused(self, video, return_intermediate, max_layer):
        from ..ops.attention_kernels import packed_self_attention
        from ..ops.fused import layer_norm
        from ..ops.gemm import gemm

        c = self.config
        W = self._weights()
        B, C, T, H, Wd = video.shape
        tb, p = c.tubelet_size, c.patch_size
        Tn, Hn, Wn = T // tb, H // p, Wd // p
        # tubelet patchify in the conv weight's (c, t, h, w) order -> one GEMM
        v = video[:, :, :Tn * tb, :Hn * p, :Wn * p].to(torch.bfloat16)
        v = v.view(B, C, Tn, tb, Hn, p, Wn, p).permute(0, 2, 4, 6, 1, 3, 5, 7)
        tok = v.reshape(B * Tn * Hn * Wn, C * tb * p * p).contiguous()
        wpe = W["patch_embed.proj.weight"].reshape(c.embed_dim, -1)
        kpad = (-tok.shape[1]) % 64
        if kpad:
            tok = F.pad(tok, (0, kpad))
            wpe = F.pad(wpe, (0, kpad))
        x = gemm(tok, wpe.contiguous(), bias=self.patch_embed.proj.bias.float())
        N = Tn * Hn * Wn
        pos = self._interpolate_pos_embed(N).to(torch.bfloat16)
        x = (x.view(B, N, -1) + pos)
        x = torch.cat([self.cls_token.to(torch.bfloat16).expand(B, -1, -1), x], 1)
        S = N + 1
        D = c.embed_dim
        x = x.reshape(B * S, D).contiguous()
        inter = {}
        last = len(self.blocks) - 1 if max_layer is None else max_layer
        for i, blk in enumerate(self.blocks[:last + 1]):
            pre = f"blocks.{i}."
            h = layer_norm(x, blk.norm1.weight, blk.norm1.bias, blk.norm1.eps)
            qkv = gemm(h, W[pre + "qkv.weight"], bias=blk.qkv.bias.float())
            o = packed_self_attention(qkv, B, S, c.num_heads, scale=c.d_head ** -0.5)
            x = gemm(o, W[pre + "proj.weight"], bias=blk.proj.bias.float(), residual=x)
            h = layer_norm(x, blk.norm2.weight, blk.norm2.bias, blk.norm2.eps)
            f = gemm(h, W[pre + "mlp.0.weight"], bias=blk.mlp[0].bias.float(), epi="gelu")
            x = gemm(f, W[pre + "mlp.3.weight"], bias=blk.mlp[3].bias.float(), residual=x)
            if return_intermediate and i in c.extract_layers:
                inter[f"layer_{i}"] = x.view(B, S, D)[:, 1:]
        y = layer_norm(x, self.norm.weight, self.norm.bias, self.norm.eps).view(B, S, D)
        return {"final": y[:, 0], "pooled": y[:, 1:].float().mean(1), "patch_features": y[:, 1:],
                "intermediate": inter}


class VJEPABackbone(nn.Module):
    """Frozen teacher: every parameter has ``requires_grad=False`` and ``train()`` keeps
    the encoder in eval mode."""

    def __init__(self, config: Optional[VJEPAConfig] = None):
        super().__init__()
        self.config = config or VJEPAConfig()
        self.encoder = VJEPAEncoder(self.config)
        for p in self.parameters():
            p.requires_grad = False
        self.register_buffer("pixel_mean", torch.tensor([0.485, 0.456, 0.406]).view(1, 3, 1, 1, 1))
        self.register_buffer("pixel_std", torch.tensor([0.229, 0.224, 0.225]).view(1, 3, 1, 1, 1))

    @classmethod
    def from_pretrained(cls, model_name_or_path: str, config: Optional[VJEPAConfig] = None,
                        device=None) -> "VJEPABackbone":
        """Loads a local checkpoint (``model`` / ``state_dict`` nesting accepted); with no
        network a hub name falls back to random initialisation with a warning."""
        backbone = cls(config or VJEPAConfig())
        try:
            sd = torch.load(model_name_or_path, map_location="cpu")
            sd = sd.get("model", sd)
            sd = sd.get("state_dict", sd)
            backbone.encoder.load_state_dict(sd, strict=False)
        except Exception as e:  # noqa: BLE001 - any load failure means random init
            warnings.warn(f"Could not load pretrained weights: {e}. Using random initialization.")
        return backbone.to(device) if device is not None else backbone

    def preprocess(self, video: torch.Tensor) -> torch.Tensor:
        """``[B, T, C, H, W]`` or ``[B, C, T, H, W]`` in [0, 1] (or [0, 255]) ->
        normalised ``[B, C, T', H', W']`` at the configured frames / size."""
        if video.dim() == 5 and video.shape[1] != 3:
            video = video.transpose(1, 2)
        B, C, T, H, W = video.shape
        tf = self.config.num_frames
        th, tw = self.config.image_hw
        if T != tf:
            video = video[:, :, torch.linspace(0, T - 1, tf).long().to(video.device)]
        if (H, W) != (th, tw):
            v = video.transpose(1, 2).reshape(B * tf, C, H, W)
            v = F.interpolate(v.float(), size=(th, tw), mode="bilinear", align_corners=False)
            video = v.view(B, tf, C, th, tw).transpose(1, 2)
        if video.max() > 1.0:
            video = video / 255.0
        return (video - self.pixel_mean.to(video.dtype)) / self.pixel_std.to(video.dtype)

    @torch.no_grad()
    def forward(self, video, preprocess: bool = True, return_all_layers: bool = True,
                max_layer: Optional[int] = None):
        self.encoder.eval()
        if preprocess:
            video = self.preprocess(video)
        if self.config.use_fp16 and video.is_cuda:
            video = video.to(torch.bfloat16)
        elif not video.is_cuda:
            video = video.float()
        return self.encoder(video, return_intermediate=return_all_layers, max_layer=max_layer)

    def get_feature_dim(self) -> int:
        return self.config.embed_dim

    def train(self, mode: bool = True):
        self.encoder.eval()
        return self


def create_vjepa_backbone(model_size: str = "large", pretrained: bool = True, device=None,
                          **kwargs) -> VJEPABackbone:
    configs = {
        "base": dict(embed_dim=768, num_layers=12, num_heads=12, extract_layers=[6, 7, 8, 9, 10, 11]),
        "large": dict(embed_dim=1024, num_layers=24, num_heads=16, extract_layers=list(range(18, 24))),
        "huge": dict(embed_dim=1280, num_layers=32, num_heads=16, extract_layers=list(range(26, 32))),
    }
    if model_size not in configs:
        raise ValueError(f"Unknown model size: {model_size}")
    cfg = VJEPAConfig(**{**configs[model_size], **{k: v for k, v in kwargs.items()
                                                    if k in VJEPAConfig.__dataclass_fields__}})
    if pretrained:
        warnings.warn("no pretrained V-JEPA weights are available offline; using random initialization")
    bb = VJEPABackbone(cfg)
    return bb.to(device) if device is not None else bb
