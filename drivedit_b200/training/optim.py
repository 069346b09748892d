"""AdamW over a :class:`~drivedit_b200.parallel.flat.FlatParamGroup`.

One pass over the flat buffers updates master weights and moments and writes the bf16
compute copy the next forward reads (the reference uses ``torch.optim.AdamW(fused=True)``
plus a separate autocast cast, training/cuda_optimized.py:840-885). Decoupled weight
decay applies to ``[0, decay_end)`` only (the reference's decay / no-decay groups).
Optional global-norm gradient clipping takes the norm of the whole buffer (or, under
FSDP, the all-reduced squared norm of the shards).

On CUDA the update is the ``adamw_flat`` kernel (``csrc/fused/optim.cu``); on CPU the
same arithmetic runs in PyTorch.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from ..parallel.flat import FlatParamGroup


class FlatAdamW:
    def __init__(self, group: FlatParamGroup, lr: float = 1e-4, betas=(0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 0.01, grad_clip: float = 0.0,
                 master: Optional[torch.Tensor] = None, grad: Optional[torch.Tensor] = None,
                 compute: Optional[torch.Tensor] = None, decay_end: Optional[int] = None):
        self.group = group
        self.lr, self.betas, self.eps, self.wd = lr, tuple(betas), eps, weight_decay
        self.grad_clip = grad_clip
        # buffers to update (the full group, or this rank's shard under FSDP)
        self.master = group.master if master is None else master
        self.grad = group.grad if grad is None else grad
        self.compute = group.compute if compute is None else compute
        self.decay_end = group.decay_end if decay_end is None else decay_end
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.step_count = 0
        self.last_grad_norm = None

    def grad_sq_norm(self) -> torch.Tensor:
        if self.grad.is_cuda:
            from ..ops.fused import sq_norm

            return sq_norm(self.grad)
        return torch.dot(self.grad, self.grad)   # one BLAS pass on the CPU

    def step(self, grad_scale: float = 1.0, sq_norm: Optional[torch.Tensor] = None):
        """Apply one update. ``grad_scale`` multiplies the gradient (e.g. 1/world for a
        summed reduce-scatter); ``sq_norm`` is the (global) squared grad norm when
        clipping is on (computed here if not given)."""
        self.step_count += 1
        b1, b2 = self.betas
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        clip = torch.ones((), device=self.grad.device, dtype=torch.float32)
        if self.grad_clip and self.grad_clip > 0:
            if sq_norm is None:
                sq_norm = self.grad_sq_norm()
            norm = sq_norm.sqrt() * grad_scale
            self.last_grad_norm = norm
            clip = torch.clamp(self.grad_clip / (norm + 1e-6), max=1.0)
        if self.master.is_cuda:
            from ..ops.fused import adamw_flat

            adamw_flat(self.master, self.grad, self.m, self.v, self.compute, clip,
                       lr=self.lr, b1=b1, b2=b2, eps=self.eps, wd=self.wd,
                       bc1=bc1, bc2=bc2, grad_scale=grad_scale, decay_end=self.decay_end)
            return
        if hasattr(torch, "_fused_adamw_"):
            # PyTorch's fused CPU AdamW: one pass per segment (decay, no-decay); it divides
            # the gradient by its grad_scale argument, so pass the reciprocal of ours
            inv = (1.0 / (grad_scale * clip)).reshape(1).float()
            step = torch.tensor(float(self.step_count))
            for lo, hi, wd in ((0, self.decay_end, self.wd), (self.decay_end, self.master.numel(), 0.0)):
                if hi > lo:
                    torch._fused_adamw_([self.master[lo:hi]], [self.grad[lo:hi]], [self.m[lo:hi]],
                                        [self.v[lo:hi]], [], [step], lr=self.lr, beta1=b1,
                                        beta2=b2, weight_decay=wd, eps=self.eps, amsgrad=False,
                                        maximize=False, grad_scale=inv, found_inf=None)
        else:
            g = self.grad * (grad_scale * clip)
            self.m.mul_(b1).add_(g, alpha=1 - b1)
            self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
            upd = (self.m / bc1) / ((self.v / bc2).sqrt() + self.eps)
            if self.wd:
                self.master[: self.decay_end].mul_(1 - self.lr * self.wd)
            self.master.add_(upd, alpha=-self.lr)
        if self.compute.data_ptr() != self.master.data_ptr():
            self.compute.copy_(self.master)

    def state_dict(self):
        return {"m": self.m, "v": self.v, "step": self.step_count, "lr": self.lr,
                "betas": self.betas, "eps": self.eps, "wd": self.wd}

    def load_state_dict(self, sd):
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.step_count = int(sd["step"])


def cosine_lr(step: int, total: int, base_lr: float, warmup: int = 0, min_ratio: float = 0.1):
    """Linear warm-up then cosine decay to ``min_ratio * base_lr`` (reference
    training/cuda_optimized.py:888-904)."""
    if warmup and step < warmup:
        return base_lr * (step + 1) / warmup
    p = min(1.0, (step - warmup) / max(1, total - warmup))
    return base_lr * (min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * p)))
