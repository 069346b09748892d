"""Batch collation for video / latent / control samples.

API of the reference ``data/collate.py``: ``VideoCollator`` (pad or truncate sequences
to a common length with a validity mask, :11-170), ``LatentCollator`` (:173-286),
``custom_collate_fn`` (:289-305), ``MemoryEfficientCollator`` (drop samples beyond a
memory budget, :308-383), ``ChunkedBatchCollator`` (split long sequences into overlapping
chunks, :386-468).
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch


def _pad_time(x: torch.Tensor, T: int, value: float = 0.0) -> torch.Tensor:
    if x.shape[0] >= T:
        return x[:T]
    pad = x.new_full((T - x.shape[0],) + tuple(x.shape[1:]), value)
    return torch.cat([x, pad], 0)


class VideoCollator:
    """Sequence samples -> a batch (data/collate.py:11-170). Sequence tensors (time
    first) are truncated to ``max_sequence_length`` and, with ``pad_to_max``, padded with
    ``padding_value`` to the longest in the batch; ``drop_incomplete`` keeps only samples
    of at least ``max_sequence_length`` frames (all of them when none is that long).
    Adds ``sequence_mask`` ``[B, T]`` and ``sequence_lengths``; non-tensor fields stay
    lists."""

    def __init__(self, pad_to_max: bool = True, max_sequence_length: Optional[int] = None,
                 padding_value: float = 0.0, drop_incomplete: bool = False,
                 sequence_keys=("frames", "controls", "depth", "ego_transform", "anchor_mask")):
        self.pad_to_max, self.max_sequence_length = pad_to_max, max_sequence_length
        self.padding_value, self.drop_incomplete = padding_value, drop_incomplete
        self.sequence_keys = tuple(sequence_keys)

    def _filter_incomplete_sequences(self, batch):
        if self.max_sequence_length is None:
            return batch
        keep = [b for b in batch if b["frames"].shape[0] >= self.max_sequence_length]
        return keep or batch

    def __call__(self, batch: List[Dict[str, Any]]) -> Dict[str, Any]:
        if not batch:
            return {}
        if self.drop_incomplete:
            batch = self._filter_incomplete_sequences(batch)
        lens = [b["frames"].shape[0] for b in batch]
        T = max(lens) if self.max_sequence_length is None else min(max(lens), self.max_sequence_length)
        out: Dict[str, Any] = {}
        for k in batch[0]:
            vals = [b.get(k) for b in batch]
            if k in self.sequence_keys and all(torch.is_tensor(v) for v in vals):
                vals = [v[:T] for v in vals]
                if self.pad_to_max:
                    vals = [_pad_time(v, T, self.padding_value) for v in vals]
                out[k] = torch.stack(vals) if len({tuple(v.shape) for v in vals}) == 1 else vals
            elif all(torch.is_tensor(v) for v in vals) and len({tuple(v.shape) for v in vals}) == 1:
                out[k] = torch.stack(vals)
            else:
                out[k] = vals
        out["sequence_mask"] = torch.arange(T)[None] < torch.tensor(lens)[:, None]
        out["sequence_lengths"] = torch.tensor([min(l, T) for l in lens])
        return out


class LatentCollator:
    """Latents ``[T, C, h, w]`` (or ``[C, h, w]``: one step) -> with ``tokenize``, tokens
    ``latent_tokens [B, T, C*h*w]`` padded with ``pad_token_id`` to the longest (at most
    ``max_tokens`` steps), else ``latents`` zero-padded in time to the longest;
    ``latent_mask`` marks the real steps (data/collate.py:173-286)."""

    def __init__(self, tokenize: bool = True, max_tokens: Optional[int] = None, pad_token_id: int = 0):
        self.tokenize, self.max_tokens, self.pad_token_id = tokenize, max_tokens, pad_token_id

    def __call__(self, batch: List[Dict[str, Any]]) -> Dict[str, Any]:
        if not batch:
            return {}
        lat = [b["latents"] if b["latents"].dim() != 3 else b["latents"][None] for b in batch]
        if self.tokenize:
            lat = [x.flatten(1) if x.dim() > 2 else x for x in lat]
        L = max(x.shape[0] for x in lat)
        if self.max_tokens is not None and self.tokenize:
            L = min(L, self.max_tokens)
        key = "latent_tokens" if self.tokenize else "latents"
        pad = float(self.pad_token_id) if self.tokenize else 0.0
        out = {key: torch.stack([_pad_time(x[:L], L, pad) for x in lat]),
               "latent_mask": torch.arange(L)[None] < torch.tensor([x.shape[0] for x in lat])[:, None]}
        for k in batch[0]:
            if k == "latents":
                continue
            vals = [b[k] for b in batch]
            if all(torch.is_tensor(v) for v in vals) and len({tuple(v.shape) for v in vals}) == 1:
                out[k] = torch.stack(vals)
            else:
                out[k] = vals
        return out


def custom_collate_fn(batch: List[Dict[str, Any]]) -> Dict[str, Any]:
    out: Dict[str, Any] = {}
    for k in batch[0]:
        vals = [b[k] for b in batch]
        if all(torch.is_tensor(v) for v in vals) and len({tuple(v.shape) for v in vals}) == 1:
            out[k] = torch.stack(vals)
        else:
            out[k] = vals
    return out


class MemoryEfficientCollator:
    """Keeps the leading samples of a batch while their frames total at most
    ``max_batch_frames`` and ``frame_memory_limit_mb`` megabytes (at least one sample),
    when ``adaptive_batching``; then collates (data/collate.py:308-383)."""

    def __init__(self, max_batch_frames: int = 128, adaptive_batching: bool = True,
                 frame_memory_limit_mb: float = 1000.0, base_collator=None):
        self.max_batch_frames, self.adaptive_batching = max_batch_frames, adaptive_batching
        self.frame_memory_limit_mb = frame_memory_limit_mb
        self.base_collator = self.base = base_collator or VideoCollator()

    @staticmethod
    def _estimate_frame_memory(frames: torch.Tensor) -> float:
        return frames.numel() * frames.element_size() / 2 ** 20

    def _filter_by_memory_limit(self, batch):
        out, frames, used = [], 0, 0.0
        for b in batch:
            f = b["frames"]
            n, m = f.shape[0], self._estimate_frame_memory(f)
            if frames + n > self.max_batch_frames or used + m > self.frame_memory_limit_mb:
                break
            out.append(b)
            frames, used = frames + n, used + m
        return out or batch[:1]

    def __call__(self, batch):
        if not batch:
            return {}
        return self.base_collator(self._filter_by_memory_limit(batch) if self.adaptive_batching else batch)


class ChunkedBatchCollator:
    """Each sample's sequences are cut into chunks of ``chunk_size`` frames with
    ``overlap`` frames shared between neighbours; all chunks form the batch."""

    def __init__(self, chunk_size: int = 32, overlap: int = 4, shuffle_chunks: bool = True,
                 sequence_keys=("frames", "controls", "depth", "ego_transform", "anchor_mask")):
        assert 0 <= overlap < chunk_size
        self.chunk_size, self.overlap, self.sequence_keys = chunk_size, overlap, tuple(sequence_keys)
        self.shuffle_chunks = shuffle_chunks

    def _create_chunks(self, sample):
        T = sample["frames"].shape[0]
        step = self.chunk_size - self.overlap
        starts = list(range(0, max(T - self.chunk_size, 0) + 1, step)) or [0]
        chunks = []
        for s in starts:
            c = {k: (v[s:s + self.chunk_size] if k in self.sequence_keys and torch.is_tensor(v) else v)
                 for k, v in sample.items()}
            c["chunk_start"] = torch.tensor(s)
            chunks.append(c)
        return chunks

    def __call__(self, batch):
        chunks = [c for b in batch for c in self._create_chunks(b)]
        if self.shuffle_chunks:
            chunks = [chunks[i] for i in torch.randperm(len(chunks)).tolist()]
        return VideoCollator(max_sequence_length=self.chunk_size)(chunks)
