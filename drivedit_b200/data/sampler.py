"""Index samplers over sequence datasets with the reference's API (``data/sampler.py``):
``TemporalSampler`` (:15-131), ``BalancedSampler`` (:134-279), ``ChunkedSampler``
(:282-379), ``SequentialChunkSampler`` (:382-474) and ``AdaptiveSampler`` (:477-570).

Every sampler takes the dataset first. Sequence structure comes from the dataset's
``sequences`` (a list with ``num_frames``) and ``sequence_indices`` (``(sequence, start)``
per item), as :class:`~drivedit_b200.data.video_loader.VideoDataset` provides; without it
the dataset is one sequence. Randomness comes from one seeded ``torch.Generator`` (the
same order on every pass unless :meth:`set_epoch` changes it), or from the global
generator when ``seed`` is None.
"""
from __future__ import annotations

from collections import defaultdict
from typing import Any, Dict, Iterator, List, Optional, Tuple

import numpy as np
import torch
from torch.utils import data


class _Seeded(data.Sampler):
    def __init__(self, seed: Optional[int] = None):
        self.seed, self.epoch = seed, 0
        self.generator = torch.Generator().manual_seed(seed) if seed is not None else None

    def set_epoch(self, epoch: int):
        self.epoch = epoch

    def _gen(self) -> Optional[torch.Generator]:
        if self.seed is None:
            return None
        return torch.Generator().manual_seed(self.seed + 1009 * self.epoch)

    def _perm(self, n: int) -> List[int]:
        return torch.randperm(n, generator=self._gen()).tolist()


def _sequence_lengths(dataset) -> List[int]:
    seqs = getattr(dataset, "sequences", None)
    if seqs:
        return [s.get("num_frames", len(s.get("frame_paths", []))) if isinstance(s, dict) else len(s)
                for s in seqs]
    return [len(dataset)]


class TemporalSampler(_Seeded):
    """Windows ``(sequence, start)`` of ``sequence_length`` frames ``temporal_stride``
    apart: ``uniform`` starts every ``sequence_length // 2`` frames, ``dense`` at every
    frame, ``sparse`` every ``sequence_length`` frames, ``adaptive`` dense on short
    sequences (under two windows) and at least three evenly spread starts on long ones.
    Yields positions in ``temporal_indices``."""

    def __init__(self, dataset, sampling_strategy: str = "uniform", sequence_length: int = 16,
                 temporal_stride: int = 1, shuffle: bool = True, seed: Optional[int] = None):
        super().__init__(seed)
        if sampling_strategy not in ("uniform", "dense", "sparse", "adaptive"):
            raise ValueError(f"unknown sampling strategy {sampling_strategy!r}")
        self.dataset, self.sampling_strategy = dataset, sampling_strategy
        self.sequence_length, self.temporal_stride, self.shuffle = sequence_length, temporal_stride, shuffle
        self.temporal_indices = self._build_temporal_indices()

    def _build_temporal_indices(self) -> List[Tuple[int, int]]:
        return [t for si, n in enumerate(_sequence_lengths(self.dataset))
                for t in self._sample_from_sequence(n, si)]

    def _sample_from_sequence(self, num_frames: int, seq_idx: int) -> List[Tuple[int, int]]:
        L = self.sequence_length
        last = num_frames - (L - 1) * self.temporal_stride - 1   # last valid start
        if last < 0:
            return []
        s = self.sampling_strategy
        if s == "adaptive" and last == 0:
            return []
        if s == "dense" or (s == "adaptive" and num_frames < 2 * L):
            starts = range(last + 1)
        elif s == "sparse":
            starts = range(0, last + 1, max(1, L))
        elif s == "uniform":
            if last == 0:
                return []
            half = max(1, L // 2)
            starts = [i * half for i in range(max(1, last // half)) if i * half <= last]
        else:  # adaptive, long sequence
            n = max(3, num_frames // L)
            starts = [min(i * last // (n - 1), last) for i in range(n)]
        return [(seq_idx, int(st)) for st in starts]

    def __iter__(self) -> Iterator[int]:
        n = len(self.temporal_indices)
        return iter(self._perm(n) if self.shuffle else range(n))

    def __len__(self) -> int:
        return len(self.temporal_indices)


class BalancedSampler(_Seeded):
    """Equalises class counts: every class is resampled to the largest class's size
    (``oversample_minority``), the smallest's (``undersample_majority``) or the median's
    (both). Labels come from ``dataset.get_sequence_info(i)[class_key]`` or
    ``dataset[i][class_key]`` (``"unknown"`` when absent). Oversampling draws with
    replacement, or repeats cyclically without."""

    def __init__(self, dataset, class_key: str = "class_label", oversample_minority: bool = True,
                 undersample_majority: bool = False, replacement: bool = True, seed: Optional[int] = None):
        super().__init__(seed)
        self.dataset, self.class_key = dataset, class_key
        self.oversample_minority, self.undersample_majority = oversample_minority, undersample_majority
        self.replacement = replacement
        self.class_indices = self._build_class_indices()
        self.balanced_indices = self._create_balanced_indices()

    def _label(self, i: int):
        try:
            if hasattr(self.dataset, "get_sequence_info"):
                return self.dataset.get_sequence_info(i).get(self.class_key, "unknown")
            item = self.dataset[i]
            return item.get(self.class_key, "unknown") if isinstance(item, dict) else "unknown"
        except Exception:  # noqa: BLE001 - an unreadable item counts as unlabelled
            return "unknown"

    def _build_class_indices(self) -> Dict[Any, List[int]]:
        d: Dict[Any, List[int]] = defaultdict(list)
        for i in range(len(self.dataset)):
            d[self._label(i)].append(i)
        return dict(d)

    def _create_balanced_indices(self) -> List[int]:
        sizes = sorted(len(v) for v in self.class_indices.values())
        if not sizes or not (self.oversample_minority or self.undersample_majority):
            return list(range(len(self.dataset)))
        if self.oversample_minority and self.undersample_majority:
            target = sizes[len(sizes) // 2]
        else:
            target = sizes[-1] if self.oversample_minority else sizes[0]
        g = self._gen()
        out: List[int] = []
        for idx in self.class_indices.values():
            n = len(idx)
            if n == target:
                out += idx
            elif n < target:
                if self.replacement:
                    pick = torch.randint(n, (target,), generator=g).tolist()
                    out += [idx[j] for j in pick]
                else:
                    out += idx * (target // n) + idx[:target % n]
            else:
                out += [idx[j] for j in torch.randperm(n, generator=g)[:target].tolist()]
        return out

    def __iter__(self) -> Iterator[int]:
        order = self._perm(len(self.balanced_indices))
        return iter([self.balanced_indices[i] for i in order])

    def __len__(self) -> int:
        return len(self.balanced_indices)

    def get_class_distribution(self) -> Dict[Any, int]:
        """Items per class in the balanced index list."""
        cls = {i: c for c, idx in self.class_indices.items() for i in idx}
        out: Dict[Any, int] = defaultdict(int)
        for i in self.balanced_indices:
            out[cls[i]] += 1
        return dict(out)


class ChunkedSampler(_Seeded):
    """Contiguous chunks of ``chunk_size`` items, neighbours sharing ``overlap`` items
    (cache locality), in shuffled order; items inside a chunk optionally shuffled; a
    short last chunk dropped with ``drop_incomplete``."""

    def __init__(self, dataset, chunk_size: int = 32, overlap: int = 4, shuffle_chunks: bool = True,
                 shuffle_within_chunks: bool = False, drop_incomplete: bool = False, seed: Optional[int] = None):
        super().__init__(seed)
        assert 0 <= overlap < chunk_size
        self.dataset, self.chunk_size, self.overlap = dataset, chunk_size, overlap
        self.shuffle_chunks, self.shuffle_within_chunks = shuffle_chunks, shuffle_within_chunks
        self.drop_incomplete = drop_incomplete
        self.chunks = self._create_chunks()

    def _create_chunks(self) -> List[List[int]]:
        n, step = len(self.dataset), self.chunk_size - self.overlap
        chunks = [list(range(s, min(s + self.chunk_size, n))) for s in range(0, n, step)]
        return [c for c in chunks if len(c) == self.chunk_size or not self.drop_incomplete]

    def __iter__(self) -> Iterator[int]:
        order = self._perm(len(self.chunks)) if self.shuffle_chunks else range(len(self.chunks))
        g = self._gen()
        out: List[int] = []
        for ci in order:
            c = self.chunks[ci]
            if self.shuffle_within_chunks:
                c = [c[j] for j in torch.randperm(len(c), generator=g).tolist()]
            out += c
        return iter(out)

    def __len__(self) -> int:
        return sum(len(c) for c in self.chunks)

    def get_chunk_info(self) -> Dict[str, Any]:
        sizes = [len(c) for c in self.chunks]
        return {"num_chunks": len(sizes), "chunk_sizes": sizes,
                "avg_chunk_size": float(np.mean(sizes)) if sizes else 0.0, "total_samples": sum(sizes)}


class SequentialChunkSampler(_Seeded):
    """Items grouped by sequence (``dataset.sequence_indices``), in start order within a
    sequence when ``maintain_sequence_order``; consecutive sequences fill a chunk until it
    holds ``sequences_per_chunk`` items; chunk order optionally shuffled (for streaming,
    stateful training). Without sequence structure: plain chunks of that many items."""

    def __init__(self, dataset, sequences_per_chunk: int = 8, maintain_sequence_order: bool = True,
                 shuffle_sequences: bool = False, seed: Optional[int] = None):
        super().__init__(seed)
        self.dataset, self.sequences_per_chunk = dataset, sequences_per_chunk
        self.maintain_sequence_order, self.shuffle_sequences = maintain_sequence_order, shuffle_sequences
        self.sequence_chunks = self._create_sequence_chunks()

    def _create_sequence_chunks(self) -> List[List[int]]:
        si = getattr(self.dataset, "sequence_indices", None)
        k = self.sequences_per_chunk
        if not si:
            n = len(self.dataset)
            return [list(range(s, min(s + k, n))) for s in range(0, n, k)]
        groups: Dict[int, List[int]] = defaultdict(list)
        for i, (seq, _) in enumerate(si):
            groups[seq].append(i)
        chunks, cur = [], []
        for idx in groups.values():
            if self.maintain_sequence_order:
                idx = sorted(idx, key=lambda i: si[i][1])
            cur += idx
            if len(cur) >= k:
                chunks.append(cur)
                cur = []
        if cur:
            chunks.append(cur)
        return chunks

    def __iter__(self) -> Iterator[int]:
        n = len(self.sequence_chunks)
        order = self._perm(n) if self.shuffle_sequences else range(n)
        return iter([i for ci in order for i in self.sequence_chunks[ci]])

    def __len__(self) -> int:
        return sum(len(c) for c in self.sequence_chunks)


class AdaptiveSampler(_Seeded):
    """Starts with ``initial_strategy`` (``uniform``, ``balanced`` or ``temporal``) and,
    every ``adaptation_frequency`` items drawn once at least 100 difficulty scores are
    known, switches: ``balanced`` when the scores vary a lot (std above 0.3), ``temporal``
    when they are high (mean above 0.7), else ``uniform``. With
    ``difficulty`` as the strategy, items are drawn in proportion to their scores."""

    def __init__(self, dataset, initial_strategy: str = "uniform", adaptation_frequency: int = 1000,
                 difficulty_key: str = "difficulty", seed: Optional[int] = None):
        super().__init__(seed)
        self.dataset, self.current_strategy = dataset, initial_strategy
        self.adaptation_frequency, self.difficulty_key = adaptation_frequency, difficulty_key
        self.step_count = 0
        self.difficulty_scores: Dict[int, float] = {}
        self.base_sampler = self._create_base_sampler()

    def _create_base_sampler(self) -> data.Sampler:
        if self.current_strategy == "balanced":
            return BalancedSampler(self.dataset, seed=self.seed)
        if self.current_strategy == "temporal":
            return TemporalSampler(self.dataset, seed=self.seed)
        return data.RandomSampler(range(len(self.dataset)), generator=self._gen())

    def update_difficulty_scores(self, sample_indices: List[int], scores: List[float]) -> None:
        for i, s in zip(sample_indices, scores):
            self.difficulty_scores[int(i)] = float(s)

    def adapt_strategy(self) -> None:
        if len(self.difficulty_scores) < 100:
            return
        v = np.asarray(list(self.difficulty_scores.values()), dtype=np.float64)
        new = "balanced" if v.std() > 0.3 else "temporal" if v.mean() > 0.7 else "uniform"
        if new != self.current_strategy:
            self.current_strategy = new
            self.base_sampler = self._create_base_sampler()

    def __iter__(self) -> Iterator[int]:
        if self.current_strategy == "difficulty" and self.difficulty_scores:
            w = torch.full((len(self.dataset),), 1e-6)
            for i, s in self.difficulty_scores.items():
                w[i] = max(s, 1e-6)
            it = iter(torch.multinomial(w, len(self.dataset), True, generator=self._gen()).tolist())
        else:
            it = iter(self.base_sampler)
        for i in it:
            self.step_count += 1
            if self.step_count % self.adaptation_frequency == 0:
                self.adapt_strategy()
            yield i

    def __len__(self) -> int:
        return len(self.base_sampler) if self.current_strategy != "difficulty" else len(self.dataset)

    def get_current_strategy(self) -> str:
        return self.current_strategy
