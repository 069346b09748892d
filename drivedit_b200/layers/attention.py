"""Attention: reference-semantics ``mha()``, masks, multi-head attention with KV cache.

Mirrors the reference's ``layers/mha.py``: ``mha()`` on ``[B, T, H, D]`` tensors
(:190-231, einsum path with ``mask == 0 -> -1e4`` and fp32 softmax :88-116), masks
(:234-281), ``MultiHeadAttention`` with a fused ``qkv`` projection, init std 0.02 and
output-projection std 0.02/sqrt(24) (:284-378), causal / bidirectional variants
(:381-428).

Differences, chosen on purpose:
  * the reference has several global "backends" (flash_attn / SDPA / einsum) selected at
    import time (:24-81) and crashes when flash_attn is importable but tensors are on
    the CPU. Here there is one path per device (PyTorch SDPA in modules, the sm_100a
    kernels in ``drivedit_b200.ops.attention`` in the fused engine); the backend API is
    kept, and its one real choice is the fp32 einsum oracle (``AttentionBackend.EINSUM``).
  * the reference drops the causal mask whenever a KV cache is passed (:406-408), so a
    multi-token step attends to its own future; here the mask always covers the new
    tokens (offset by the cache length).
  * RoPE positions continue from the cache length instead of restarting at 0
    (reference bug ``models/dit_student.py:362-366``).
  * ``frame_causal_mask`` adds the video masking the world models use: every token of
    frame f sees all tokens of frames <= f.
"""
from __future__ import annotations

import math
import warnings
from enum import Enum
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


def create_causal_mask(T: int, device=None, S: Optional[int] = None) -> torch.Tensor:
    """``[1, 1, T, S]`` bool, True = attend. With ``S > T`` the queries are the last T."""
    S = S or T
    q = torch.arange(S - T, S, device=device)[:, None]
    k = torch.arange(S, device=device)[None, :]
    return (k <= q)[None, None]


def create_block_causal_mask(block_size: int, num_blocks: int, device=None) -> torch.Tensor:
    """``[1, 1, L, L]`` float mask (1 = attend) over ``L = block_size * num_blocks``
    tokens, the reference's block-causal mask (layers/mha.py:249-281): every earlier
    block in full and the current block causally, which is token-causal attention. The
    block-bidirectional mask (a whole block sees itself) is :func:`frame_causal_mask`."""
    L = block_size * num_blocks
    return create_causal_mask(L, device).float()


def frame_causal_mask(T: int, tokens_per_frame: int, S: Optional[int] = None,
                      device=None) -> torch.Tensor:
    """Frame-causal over a KV sequence of ``S`` tokens whose last ``T`` are the queries."""
    S = S or T
    qf = torch.arange(S - T, S, device=device)[:, None] // tokens_per_frame
    kf = torch.arange(S, device=device)[None, :] // tokens_per_frame
    return (kf <= qf)[None, None]


def attention_reference(q, k, v, mask: Optional[torch.Tensor] = None,
                        scale: Optional[float] = None, return_lse: bool = False):
    """fp32 softmax attention on ``[B, T, H, D]``; ``mask`` is bool (True = attend),
    broadcastable to ``[B, H, T, S]``. Rows with no visible key return zeros."""
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    s = torch.einsum("bthd,bshd->bhts", q.float(), k.float()) * scale
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None]).nan_to_num(0.0)
    o = torch.einsum("bhts,bshd->bthd", p, v.float())
    return (o, lse) if return_lse else o


class AttentionBackend(Enum):
    """The reference's backend names (layers/mha.py:24-28) plus this framework's own.
    There is no dispatch between libraries: ``SM100`` (the default) is PyTorch SDPA for
    module-level attention and this framework's tcgen05 kernels in the fused engine;
    ``EINSUM`` makes :func:`mha` compute the fp32 einsum oracle instead (for numerical
    comparisons). The flash-attention names are never available."""
    SM100 = "sm100"
    FLASH_ATTN_3 = "flash_attn_3"
    FLASH_ATTN_2 = "flash_attn_2"
    EINSUM = "einsum"


_BACKEND = AttentionBackend.SM100


def get_available_backends() -> list:
    return [AttentionBackend.SM100, AttentionBackend.EINSUM]


def get_attention_backend() -> AttentionBackend:
    return _BACKEND


def set_attention_backend(backend: AttentionBackend) -> bool:
    """Select the backend; an unavailable one warns and returns False (the reference's
    behaviour, layers/mha.py:73-81)."""
    global _BACKEND
    if backend not in get_available_backends():
        warnings.warn(f"Backend {backend} not available. Available: {get_available_backends()}")
        return False
    _BACKEND = backend
    return True


def mha(q, k, v, mask: Optional[torch.Tensor] = None, dropout_p: float = 0.0,
        training: bool = False, is_causal: bool = False, backend: Optional[AttentionBackend] = None,
        causal: bool = False) -> torch.Tensor:
    """Reference-compatible scaled dot-product attention on ``[B, T, H, D]``.

    ``mask`` follows the reference: 0 = blocked (any dtype) or a bool tensor. ``backend``
    ``EINSUM`` selects the fp32 oracle for this call (see :class:`AttentionBackend`)."""
    causal = causal or is_causal
    if backend is AttentionBackend.EINSUM and _BACKEND is not AttentionBackend.EINSUM:
        if mask is not None and mask.dtype != torch.bool:
            mask = mask != 0
        if causal and mask is None:
            mask = create_causal_mask(q.shape[1], q.device, k.shape[1])
        return attention_reference(q, k, v, mask).to(q.dtype)
    if mask is not None and mask.dtype != torch.bool:
        mask = mask != 0
    if _BACKEND is AttentionBackend.EINSUM:
        if causal and mask is None:
            mask = create_causal_mask(q.shape[1], q.device, k.shape[1])
        o = attention_reference(q, k, v, mask)
        if training and dropout_p > 0:
            o = F.dropout(o, dropout_p)
        return o.to(q.dtype)
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    o = F.scaled_dot_product_attention(
        qt, kt, vt, attn_mask=mask, dropout_p=dropout_p if training else 0.0,
        is_causal=causal and mask is None)
    return o.transpose(1, 2)


class KVCache:
    """Rolling key/value cache ``[B, S, H, D]`` bounded to ``max_tokens`` (oldest dropped).

    Mirrors the reference's ``RollingKVCache`` (training/self_forcing_plus.py:29-145)
    with the window expressed in tokens; callers pass ``frames * tokens_per_frame``.
    ``start`` is the absolute position of the first cached token, so RoPE positions
    of new tokens continue correctly after truncation."""

    def __init__(self, max_tokens: Optional[int] = None):
        self.max_tokens = max_tokens
        self.k: Optional[torch.Tensor] = None
        self.v: Optional[torch.Tensor] = None
        self.start = 0

    def __len__(self):
        return 0 if self.k is None else self.k.shape[1]

    @property
    def end(self) -> int:
        return self.start + len(self)

    def append(self, k: torch.Tensor, v: torch.Tensor):
        if self.k is None:
            self.k, self.v = k, v
        else:
            self.k = torch.cat([self.k, k], 1)
            self.v = torch.cat([self.v, v], 1)
        if self.max_tokens is not None and self.k.shape[1] > self.max_tokens:
            drop = self.k.shape[1] - self.max_tokens
            self.k, self.v = self.k[:, drop:], self.v[:, drop:]
            self.start += drop
        return self.k, self.v

    def reset(self):
        self.k = self.v = None
        self.start = 0

    def as_dict(self) -> Dict[str, torch.Tensor]:
        return {"k": self.k, "v": self.v}


class MultiHeadAttention(nn.Module):
    """Self-attention with fused ``qkv`` and ``proj`` (reference state-dict names)."""

    def __init__(self, d_model: int, n_heads: int, dropout: float = 0.0, bias: bool = False,
                 rope_layer: Optional[nn.Module] = None, causal: bool = False,
                 tokens_per_frame: Optional[int] = None):
        super().__init__()
        assert d_model % n_heads == 0
        self.d_model, self.n_heads = d_model, n_heads
        self.d_head = d_model // n_heads
        self.dropout = dropout
        self.rope_layer = rope_layer
        self.causal = causal
        self.tokens_per_frame = tokens_per_frame
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=bias)
        self.proj = nn.Linear(d_model, d_model, bias=bias)
        nn.init.normal_(self.qkv.weight, std=0.02)
        nn.init.normal_(self.proj.weight, std=0.02 / math.sqrt(2 * 12))
        if bias:
            nn.init.zeros_(self.qkv.bias)
            nn.init.zeros_(self.proj.bias)

    def _rope(self, x, start_pos):
        if self.rope_layer is None:
            return x
        return self.rope_layer(x, start_pos)

    def forward(self, x: torch.Tensor, kv_cache=None, mask: Optional[torch.Tensor] = None,
                start_pos: Optional[int] = None):
        B, T, D = x.shape
        q, k, v = self.qkv(x).view(B, T, 3, self.n_heads, self.d_head).unbind(2)
        cache_obj = kv_cache if isinstance(kv_cache, KVCache) else None
        past = 0
        if cache_obj is not None:
            past = cache_obj.end
        elif isinstance(kv_cache, dict) and kv_cache.get("k") is not None:
            past = kv_cache["k"].shape[1]
        pos = past if start_pos is None else start_pos
        q, k = self._rope(q, pos), self._rope(k, pos)
        new_cache = None
        if cache_obj is not None:
            k, v = cache_obj.append(k.detach(), v.detach())
            new_cache = cache_obj
        elif isinstance(kv_cache, dict):
            if kv_cache.get("k") is not None:
                k = torch.cat([kv_cache["k"], k], 1)
                v = torch.cat([kv_cache["v"], v], 1)
            new_cache = {"k": k.detach(), "v": v.detach()}
        S = k.shape[1]
        if mask is None and self.causal and (T > 1 or S > T):
            if self.tokens_per_frame:
                mask = frame_causal_mask(T, self.tokens_per_frame, S, x.device)
            else:
                mask = create_causal_mask(T, x.device, S)
        o = mha(q, k, v, mask=mask, dropout_p=self.dropout, training=self.training)
        return self.proj(o.reshape(B, T, D)), new_cache


class CausalMultiHeadAttention(MultiHeadAttention):
    def __init__(self, *a, **kw):
        kw["causal"] = True
        super().__init__(*a, **kw)

    def forward(self, x, kv_cache=None, start_pos: Optional[int] = None):
        return super().forward(x, kv_cache, None, start_pos)


class BidirectionalMultiHeadAttention(MultiHeadAttention):
    def __init__(self, *a, **kw):
        kw["causal"] = False
        super().__init__(*a, **kw)

    def forward(self, x, kv_cache=None, start_pos: Optional[int] = None):
        return super().forward(x, kv_cache, None, start_pos)


class CrossAttention(nn.Module):
    """Cross-attention from tokens to a conditioning context (the reference's
    ``DiTBlockWithCrossAttention`` never projects its context, blocks/dit_block.py:230-234;
    this one does)."""

    def __init__(self, d_model: int, n_heads: int, context_dim: Optional[int] = None,
                 bias: bool = False):
        super().__init__()
        context_dim = context_dim or d_model
        self.n_heads, self.d_head = n_heads, d_model // n_heads
        self.q = nn.Linear(d_model, d_model, bias=bias)
        self.kv = nn.Linear(context_dim, 2 * d_model, bias=bias)
        self.proj = nn.Linear(d_model, d_model, bias=bias)
        nn.init.zeros_(self.proj.weight)

    def project_context(self, context: torch.Tensor) -> Dict[str, torch.Tensor]:
        """The context's keys and values ``{"k", "v"}`` ``[B, S, H, d_head]``."""
        B, S = context.shape[:2]
        k, v = self.kv(context).view(B, S, 2, self.n_heads, self.d_head).unbind(2)
        return {"k": k, "v": v}

    def attend(self, x, kv: Dict[str, torch.Tensor], context_mask: Optional[torch.Tensor] = None):
        B, T, D = x.shape
        q = self.q(x).view(B, T, self.n_heads, self.d_head)
        m = None if context_mask is None else context_mask[:, None, None, :].bool()
        return self.proj(mha(q, kv["k"], kv["v"], mask=m).reshape(B, T, D))

    def forward(self, x, context, context_mask: Optional[torch.Tensor] = None):
        return self.attend(x, self.project_context(context), context_mask)
