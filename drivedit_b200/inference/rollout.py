"""Streaming autoregressive rollout of the causal world model (Self-Forcing++ style).

Frames are produced in chunks: for each chunk of ``chunk_frames`` latent frames, start
from Gaussian noise at flow time t=0 and take ``flow_steps`` Euler steps to t=1 with the
velocity predicted from the chunk and the cached keys/values of the previous
``window_frames`` frames (frame-causal inside the chunk); then run the finished chunk once
more at t=1 to put its clean keys/values into the rolling window. The context frames are
encoded the same way before the first chunk.

Re-design of the reference's ``StreamingRollout`` (inference/rollout.py:158-492: one frame
at a time, no denoising steps, a VAE re-encode of the whole window every frame, a token
contract that does not match its own model) from its working pieces: the Euler flow
sampler (blocks/flow_matching.py:228-281), the rolling KV window
(training/self_forcing_plus.py:29-145, here in frames) and the causal student.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional

import torch

from ..config import RolloutConfig
from ..models.world_dit import KVCacheSet, WorldDiT, forward_cached


@dataclass
class RolloutResult:
    frames: torch.Tensor          # [B, F_total, C, H, W] (context + generated)
    chunk_ms: List[float]         # device time per generated chunk
    total_ms: float

    @property
    def generated_frames(self) -> int:
        return len(self.chunk_ms)

    def frames_per_s(self, batch: int, chunk_frames: int) -> float:
        return batch * chunk_frames * len(self.chunk_ms) / (sum(self.chunk_ms) / 1000.0)

    def percentile_ms(self, q: float) -> float:
        xs = sorted(self.chunk_ms)
        if not xs:
            return 0.0
        i = min(len(xs) - 1, max(0, int(round(q / 100.0 * (len(xs) - 1)))))
        return xs[i]


class StreamingRollout:
    def __init__(self, model: WorldDiT, cfg: RolloutConfig, dtype: Optional[torch.dtype] = None):
        self.model = model
        self.cfg = cfg
        dev = next(model.parameters()).device
        self.device = dev
        self.dtype = dtype or (torch.bfloat16 if dev.type == "cuda" else torch.float32)

    def _timer(self):
        if self.device.type == "cuda":
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            return s, e
        return None, None

    @torch.no_grad()
    def run(self, context: torch.Tensor, actions: torch.Tensor, total_frames: Optional[int] = None,
            generator: Optional[torch.Generator] = None, extra_cond: Optional[torch.Tensor] = None,
            replace=None) -> RolloutResult:
        """``context [B, Fc, C, H, W]`` clean latent frames, ``actions [B, F_total, A]``
        for every frame (context included); returns context + generated frames.

        ``extra_cond [B, F_total, d]`` is added to each frame's conditioning. ``replace``
        (a callable ``(f0, n) -> chunk or None``) may supply the chunk of frames
        ``[f0, f0 + n)`` instead of generating it (e.g. the ground-truth frames in
        self-forcing training for chunks that are not self-generated)."""
        cfg = self.cfg
        m = self.model
        B, Fc = context.shape[:2]
        total = total_frames or cfg.total_frames
        chunk = cfg.chunk_frames
        cache = KVCacheSet(m, B, cfg.window_frames, chunk, self.device, self.dtype)
        out = [context.to(self.dtype)]
        ones = torch.ones(B, device=self.device)
        # context frames -> cache (clean, t = 1)
        for f0 in range(0, Fc, chunk):
            f1 = min(Fc, f0 + chunk)
            forward_cached(m, context[:, f0:f1].to(self.dtype), ones, actions[:, f0:f1], cache,
                           commit=True, extra_cond=None if extra_cond is None else extra_cond[:, f0:f1])
        ts = torch.linspace(0.0, 1.0, cfg.flow_steps + 1, device=self.device)
        chunk_ms: List[float] = []
        t_all0 = time.perf_counter()
        f = Fc
        shape = (B, chunk) + tuple(context.shape[2:])
        while f < total:
            n = min(chunk, total - f)
            a = actions[:, f:f + n]
            ec = None if extra_cond is None else extra_cond[:, f:f + n]
            s_ev, e_ev = self._timer()
            t0 = time.perf_counter()
            if s_ev is not None:
                s_ev.record()
            given = replace(f, n) if replace is not None else None
            if given is not None:
                x = given.to(self.dtype)
            else:
                x = torch.randn(shape[:1] + (n,) + shape[2:], device=self.device,
                                generator=generator, dtype=torch.float32).to(self.dtype)
                for i in range(cfg.flow_steps):
                    t = ts[i].expand(B)
                    v = forward_cached(m, x, t, a, cache, commit=False, extra_cond=ec)
                    x = (x.float() + (ts[i + 1] - ts[i]) * v.float()).to(self.dtype)
            forward_cached(m, x, ones, a, cache, commit=True, extra_cond=ec)
            if e_ev is not None:
                e_ev.record()
                e_ev.synchronize()
                chunk_ms.append(s_ev.elapsed_time(e_ev))
            else:
                chunk_ms.append((time.perf_counter() - t0) * 1000.0)
            out.append(x)
            f += n
        total_ms = (time.perf_counter() - t_all0) * 1000.0
        return RolloutResult(torch.cat(out, 1), chunk_ms, total_ms)
