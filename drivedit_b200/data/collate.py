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
    def __init__(self, max_sequence_length: Optional[int] = None, pad_value: float = 0.0,
                 drop_incomplete: bool = False, min_sequence_length: int = 1,
                 sequence_keys=("frames", "controls", "depth", "ego_transform", "anchor_mask")):
        self.max_sequence_length, self.pad_value = max_sequence_length, pad_value
        self.drop_incomplete, self.min_sequence_length = drop_incomplete, min_sequence_length
        self.sequence_keys = tuple(sequence_keys)

    def _filter_incomplete_sequences(self, batch):
        return [b for b in batch if b["frames"].shape[0] >= self.min_sequence_length]

    def __call__(self, batch: List[Dict[str, Any]]) -> Dict[str, Any]:
        if self.drop_incomplete:
            batch = self._filter_incomplete_sequences(batch)
        if not batch:
            return {}
        lens = [b["frames"].shape[0] for b in batch]
        T = max(lens) if self.max_sequence_length is None else min(max(lens), self.max_sequence_length)
        out: Dict[str, Any] = {}
        for k in batch[0]:
            vals = [b.get(k) for b in batch]
            if k in self.sequence_keys and all(torch.is_tensor(v) for v in vals):
                out[k] = torch.stack([_pad_time(v, T, self.pad_value) for v in vals])
            elif all(torch.is_tensor(v) for v in vals) and len({tuple(v.shape) for v in vals}) == 1:
                out[k] = torch.stack(vals)
            else:
                out[k] = vals
        out["sequence_mask"] = torch.arange(T)[None] < torch.tensor(lens)[:, None]
        out["sequence_lengths"] = torch.tensor([min(l, T) for l in lens])
        return out


class LatentCollator:
    """Latents ``[T, C, h, w]`` or tokenised ``[N, D]`` -> padded batch + mask."""

    def __init__(self, pad_value: float = 0.0, max_tokens: Optional[int] = None):
        self.pad_value, self.max_tokens = pad_value, max_tokens

    def __call__(self, batch: List[Dict[str, Any]]) -> Dict[str, Any]:
        lat = [b["latents"] for b in batch]
        L = max(x.shape[0] for x in lat)
        if self.max_tokens is not None:
            L = min(L, self.max_tokens)
        out = {"latents": torch.stack([_pad_time(x, L, self.pad_value) for x in lat]),
               "latent_mask": torch.arange(L)[None] < torch.tensor([x.shape[0] for x in lat])[:, None]}
        for k in batch[0]:
            if k == "latents":
                continue
            vals = [b[k] for b in batch]
            if all(torch.is_tensor(v) for v in vals):
                out[k] = torch.stack([_pad_time(v, L) if v.dim() and v.shape[0] == b["latents"].shape[0] else v
                                      for v, b in zip(vals, batch)])
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
    def __init__(self, max_memory_mb: float = 1024.0, base_collator=None):
        self.max_memory_mb = max_memory_mb
        self.base = base_collator or VideoCollator()

    @staticmethod
    def _estimate_frame_memory(frames: torch.Tensor) -> float:
        return frames.numel() * frames.element_size() / 2 ** 20

    def _filter_by_memory_limit(self, batch):
        out, used = [], 0.0
        for b in batch:
            m = self._estimate_frame_memory(b["frames"])
            if out and used + m > self.max_memory_mb:
                break
            out.append(b)
            used += m
        return out

    def __call__(self, batch):
        return self.base(self._filter_by_memory_limit(batch))


class ChunkedBatchCollator:
    """Each sample's sequences are cut into chunks of ``chunk_size`` frames with
    ``overlap`` frames shared between neighbours; all chunks form the batch."""

    def __init__(self, chunk_size: int = 8, overlap: int = 2,
                 sequence_keys=("frames", "controls", "depth", "ego_transform", "anchor_mask")):
        assert 0 <= overlap < chunk_size
        self.chunk_size, self.overlap, self.sequence_keys = chunk_size, overlap, tuple(sequence_keys)

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
        return VideoCollator(max_sequence_length=self.chunk_size)(chunks)
