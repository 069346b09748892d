"""Index samplers over sequence datasets.

API of the reference ``data/sampler.py``: ``TemporalSampler`` (windows per sequence
with a stride, :15-131), ``BalancedSampler`` (inverse-frequency class balancing,
:134-279), ``ChunkedSampler`` (shuffled contiguous chunks for cache locality, :282-379),
``SequentialChunkSampler`` (ordered chunks per sequence, :382-474) and
``AdaptiveSampler`` (difficulty-weighted, :477-570). All draw from a seeded
``torch.Generator`` and support ``set_epoch`` for distributed reshuffling.
"""
from __future__ import annotations

from typing import Any, Dict, Iterator, List, Optional, Sequence, Tuple

import torch
from torch.utils import data


class _Seeded(data.Sampler):
    def __init__(self, seed: int = 0):
        self.seed, self.epoch = seed, 0

    def set_epoch(self, epoch: int):
        self.epoch = epoch

    def _gen(self):
        return torch.Generator().manual_seed(self.seed + 1009 * self.epoch)


class TemporalSampler(_Seeded):
    """``sequence_lengths[i]`` frames per sequence -> flat indices of windows of
    ``window`` frames every ``stride`` frames (index = (sequence, start) flattened)."""

    def __init__(self, sequence_lengths: Sequence[int], window: int = 16, stride: int = 8,
                 shuffle: bool = True, seed: int = 0):
        super().__init__(seed)
        self.sequence_lengths, self.window, self.stride, self.shuffle = list(sequence_lengths), window, stride, shuffle
        self.temporal_indices = self._build_temporal_indices()

    def _build_temporal_indices(self) -> List[Tuple[int, int]]:
        out = []
        for si, n in enumerate(self.sequence_lengths):
            out.extend(self._sample_from_sequence(n, si))
        return out

    def _sample_from_sequence(self, num_frames: int, seq_idx: int):
        if num_frames < self.window:
            return []
        return [(seq_idx, s) for s in range(0, num_frames - self.window + 1, self.stride)]

    def __iter__(self) -> Iterator[int]:
        n = len(self.temporal_indices)
        order = torch.randperm(n, generator=self._gen()) if self.shuffle else torch.arange(n)
        return iter(order.tolist())

    def __len__(self) -> int:
        return len(self.temporal_indices)


class BalancedSampler(_Seeded):
    """Draws ``num_samples`` indices with probability inversely proportional to the
    frequency of each sample's label (``labels[i]``)."""

    def __init__(self, labels: Sequence[Any], num_samples: Optional[int] = None, replacement: bool = True,
                 seed: int = 0):
        super().__init__(seed)
        self.labels = list(labels)
        self.num_samples = num_samples or len(self.labels)
        self.replacement = replacement
        self.class_indices = self._build_class_indices()

    def _build_class_indices(self) -> Dict[Any, List[int]]:
        d: Dict[Any, List[int]] = {}
        for i, l in enumerate(self.labels):
            d.setdefault(l, []).append(i)
        return d

    def _create_balanced_indices(self) -> List[int]:
        w = torch.tensor([1.0 / len(self.class_indices[l]) for l in self.labels])
        return torch.multinomial(w, self.num_samples, self.replacement, generator=self._gen()).tolist()

    def __iter__(self):
        return iter(self._create_balanced_indices())

    def __len__(self):
        return self.num_samples

    def get_class_distribution(self) -> Dict[Any, int]:
        return {k: len(v) for k, v in self.class_indices.items()}


class ChunkedSampler(_Seeded):
    def __init__(self, dataset_size: int, chunk_size: int = 64, shuffle_chunks: bool = True,
                 shuffle_within: bool = False, seed: int = 0):
        super().__init__(seed)
        self.n, self.chunk_size = dataset_size, chunk_size
        self.shuffle_chunks, self.shuffle_within = shuffle_chunks, shuffle_within
        self.chunks = self._create_chunks()

    def _create_chunks(self) -> List[List[int]]:
        return [list(range(s, min(s + self.chunk_size, self.n))) for s in range(0, self.n, self.chunk_size)]

    def __iter__(self):
        g = self._gen()
        order = torch.randperm(len(self.chunks), generator=g).tolist() if self.shuffle_chunks else range(len(self.chunks))
        out = []
        for ci in order:
            c = self.chunks[ci]
            if self.shuffle_within:
                c = [c[j] for j in torch.randperm(len(c), generator=g).tolist()]
            out.extend(c)
        return iter(out)

    def __len__(self):
        return self.n

    def get_chunk_info(self) -> Dict[str, Any]:
        return {"num_chunks": len(self.chunks), "chunk_size": self.chunk_size, "dataset_size": self.n}


class SequentialChunkSampler(_Seeded):
    """Chunks never cross sequence boundaries; chunk order optionally shuffled, order
    inside a chunk kept (for streaming / stateful training)."""

    def __init__(self, sequence_lengths: Sequence[int], chunk_size: int = 8, shuffle: bool = True, seed: int = 0):
        super().__init__(seed)
        self.sequence_lengths, self.chunk_size, self.shuffle = list(sequence_lengths), chunk_size, shuffle
        self.chunks = self._create_sequence_chunks()

    def _create_sequence_chunks(self):
        out, base = [], 0
        for n in self.sequence_lengths:
            for s in range(0, n, self.chunk_size):
                out.append(list(range(base + s, base + min(s + self.chunk_size, n))))
            base += n
        return out

    def __iter__(self):
        order = torch.randperm(len(self.chunks), generator=self._gen()).tolist() if self.shuffle else range(len(self.chunks))
        return iter([i for ci in order for i in self.chunks[ci]])

    def __len__(self):
        return sum(self.sequence_lengths)


class AdaptiveSampler(_Seeded):
    """Uniform at first; after ``warmup_updates`` difficulty updates, samples with
    probability proportional to ``difficulty ** temperature`` (hard examples more)."""

    def __init__(self, dataset_size: int, temperature: float = 1.0, warmup_updates: int = 1, seed: int = 0):
        super().__init__(seed)
        self.n, self.temperature, self.warmup_updates = dataset_size, temperature, warmup_updates
        self.scores = torch.ones(dataset_size)
        self.updates = 0
        self.strategy = "uniform"

    def _create_base_sampler(self):
        return data.RandomSampler(range(self.n), generator=self._gen())

    def update_difficulty_scores(self, sample_indices: List[int], scores: List[float]) -> None:
        self.scores[torch.as_tensor(sample_indices)] = torch.as_tensor(scores, dtype=torch.float32).clamp_min(1e-6)
        self.updates += 1
        self.adapt_strategy()

    def adapt_strategy(self) -> None:
        self.strategy = "difficulty" if self.updates >= self.warmup_updates else "uniform"

    def __iter__(self):
        if self.strategy == "uniform":
            return iter(list(self._create_base_sampler()))
        w = self.scores.pow(self.temperature)
        return iter(torch.multinomial(w, self.n, True, generator=self._gen()).tolist())

    def __len__(self):
        return self.n

    def get_current_strategy(self) -> str:
        return self.strategy
