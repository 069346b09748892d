"""Flat parameter storage: one fp32 master buffer, one fp32 gradient buffer and one bf16
compute copy for a group of parameters.

Every ``nn.Parameter`` of the group is re-pointed at a view of the flat master buffer
and its ``.grad`` at a view of the flat gradient buffer, so:
  * autograd accumulates ordinary gradients in place into the flat buffer;
  * fused kernels write weight gradients straight into ``p.grad`` (fp32 reductions);
  * the fused AdamW kernel updates the whole group in one pass and writes the bf16
    compute copy the next forward reads (no separate cast);
  * FSDP shards exactly these buffers (``drivedit_b200.parallel.fsdp``).

Segments are padded to 64 elements so every view starts 128-byte aligned in the bf16
copy (TMA needs 16) and weight-decay / no-decay parameters are grouped so the update
kernel receives one boundary instead of a mask.
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Tuple

import torch
import torch.nn as nn

ALIGN = 64


def _round(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class FlatParamGroup:
    def __init__(self, named_params: Iterable[Tuple[str, nn.Parameter]], device=None,
                 no_decay: Optional[Iterable[str]] = None, pad_to: int = 1,
                 compute_dtype: torch.dtype = torch.bfloat16, allocator=None):
        """``allocator(kind, numel, dtype)`` may supply the ``master`` / ``grad`` /
        ``compute`` buffers (e.g. in peer-mapped memory); they must be zero-filled."""
        named = list(named_params)
        nd = set(no_decay or [])
        decay = [(n, p) for n, p in named if n not in nd]
        nodecay = [(n, p) for n, p in named if n in nd]
        self.names: List[str] = []
        self.params: List[nn.Parameter] = []
        self.offsets: Dict[str, Tuple[int, int]] = {}
        off = 0
        self.decay_end = 0
        for i, (n, p) in enumerate(decay + nodecay):
            if i == len(decay):
                self.decay_end = off
            self.names.append(n)
            self.params.append(p)
            self.offsets[n] = (off, p.numel())
            off = _round(off + p.numel(), ALIGN)
        if not nodecay:
            self.decay_end = off
        self.numel = _round(off, ALIGN * max(pad_to, 1))
        dev = device if device is not None else (self.params[0].device if self.params else "cpu")
        self.device = torch.device(dev)
        if allocator is None:
            allocator = lambda kind, n, dt: torch.zeros(n, dtype=dt, device=self.device)
        self.master = allocator("master", self.numel, torch.float32)
        self.grad = allocator("grad", self.numel, torch.float32)
        # an fp32 compute copy would equal the master: alias it instead of copying
        self.compute = (self.master if compute_dtype == torch.float32
                        else allocator("compute", self.numel, compute_dtype))
        # groups whose parameters this one resolves views for too (rank-local expert
        # parameters under expert parallelism live in their own group)
        self.linked: List["FlatParamGroup"] = []
        self._pos = {id(p): i for i, p in enumerate(self.params)}
        with torch.no_grad():
            for n, p in zip(self.names, self.params):
                o, k = self.offsets[n]
                self.master[o:o + k].copy_(p.data.reshape(-1).float())
                p.data = self.master[o:o + k].view(p.shape)
                p.grad = self.grad[o:o + k].view(p.shape)
        self.refresh_compute()

    # ------------------------------------------------------------------ views
    def view(self, buf: torch.Tensor, p: nn.Parameter) -> torch.Tensor:
        n = self.names[self.index(p)]
        o, k = self.offsets[n]
        return buf[o:o + k].view(p.shape)

    def index(self, p: nn.Parameter) -> int:
        i = self._pos.get(id(p))
        if i is None or self.params[i] is not p:
            raise KeyError("parameter not in this group")
        return i

    def owns(self, p: nn.Parameter) -> bool:
        i = self._pos.get(id(p))
        return i is not None and self.params[i] is p

    def compute_view(self, p: nn.Parameter) -> torch.Tensor:
        if not self.owns(p):
            for g in self.linked:
                if g.owns(p):
                    return g.compute_view(p)
        return self.view(self.compute, p)

    def grad_view(self, p: nn.Parameter) -> torch.Tensor:
        return self.view(self.grad, p)

    # ------------------------------------------------------------------ updates
    def refresh_compute(self):
        if self.compute.data_ptr() != self.master.data_ptr():
            self.compute.copy_(self.master)
        for g in self.linked:
            g.refresh_compute()

    def zero_grad(self):
        for g in self.linked:
            g.zero_grad()
        self.grad.zero_()
        for n, p in zip(self.names, self.params):
            if p.grad is None or p.grad.data_ptr() != self.grad_view(p).data_ptr():
                p.grad = self.grad_view(p)

    def state_dict(self) -> Dict[str, torch.Tensor]:
        return {n: p.detach().clone() for n, p in zip(self.names, self.params)}
