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
from collections import defaultdict, deque
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from ..config import RolloutConfig
from ..models.world_dit import KVCacheSet, WorldDiT
from ..models.world_dit import forward_cached as _forward_cached


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


class MemoryBank:
    """Long-horizon memory of pooled frame features (reference ``inference/rollout.py:26-129``).

    ``update`` stores an 8x8 average-pooled summary of each frame, scored by its variance,
    and a 4x4 summary of frames with strong edges as object memory; ``get_memory_tokens``
    returns the ``top_k`` best-scored summaries (recency-weighted, temporal order kept)
    projected to ``d_model``. The projection is drawn once per feature width from a fixed
    seed; the reference draws a new random matrix on every call, so its tokens change
    between identical calls."""

    def __init__(self, d_model: int = 1024, max_spatial_memory: int = 2048, max_object_memory: int = 512,
                 decay_rate: float = 0.95, seed: int = 0):
        self.d_model, self.decay_rate, self.seed = d_model, decay_rate, seed
        self.max_spatial_memory, self.max_object_memory = max_spatial_memory, max_object_memory
        self.spatial_memory = deque(maxlen=max_spatial_memory)
        self.object_memory = deque(maxlen=max_object_memory)
        self.memory_scores = deque(maxlen=max_spatial_memory)
        self.frame_count = 0
        self._proj: Dict[int, torch.Tensor] = {}

    def update(self, frame: torch.Tensor, frame_idx: int = 0):
        self.spatial_memory.append(F.adaptive_avg_pool2d(frame, (8, 8)).flatten(1).detach())
        self.memory_scores.append(float(frame.float().var(dim=(2, 3)).mean()))
        edges = (frame[..., 1:] - frame[..., :-1]).abs().mean() + (frame[..., 1:, :] - frame[..., :-1, :]).abs().mean()
        if float(edges) > 0.1:
            self.object_memory.append(F.adaptive_avg_pool2d(frame, (4, 4)).flatten(1).detach())
        self.frame_count += 1

    def _projection(self, width: int, device) -> torch.Tensor:
        if width not in self._proj:
            g = torch.Generator().manual_seed(self.seed + width)
            self._proj[width] = torch.randn(self.d_model, width, generator=g) * 0.02
        return self._proj[width].to(device)

    def get_memory_tokens(self, top_k: int = 64) -> torch.Tensor:
        if not self.spatial_memory:
            return torch.zeros(1, 0, self.d_model)
        mem = torch.stack(list(self.spatial_memory), 0)              # [T, B, f]
        scores = torch.tensor(list(self.memory_scores))
        w = scores * torch.exp(-0.1 * torch.arange(len(scores), 0, -1, dtype=torch.float32))
        if len(w) > top_k:
            mem = mem[torch.sort(torch.topk(w, top_k).indices).values.to(mem.device)]
        flat = mem.reshape(-1, mem.shape[-1]).float()
        return F.linear(flat, self._projection(flat.shape[-1], flat.device)).unsqueeze(0)

    def clear(self):
        self.spatial_memory.clear()
        self.object_memory.clear()
        self.memory_scores.clear()
        self.frame_count = 0


class InferenceConfig:
    """Streaming-inference settings (reference ``inference/rollout.py:132-155``); maps onto
    :class:`~drivedit_b200.config.RolloutConfig` (``chunk_size`` -> chunk frames,
    ``context_window`` -> KV window frames, ``max_sequence_length`` -> total frames)."""

    def __init__(self, max_sequence_length: int = 300, context_window: int = 8, memory_limit: int = 2048,
                 temperature: float = 1.0, top_p: float = 0.9, use_kv_cache: bool = True,
                 mixed_precision: bool = True, chunk_size: int = 4, memory_offload_freq: int = 20,
                 flow_steps: int = 4):
        self.max_sequence_length, self.context_window, self.memory_limit = max_sequence_length, context_window, memory_limit
        self.temperature, self.top_p, self.use_kv_cache = temperature, top_p, use_kv_cache
        self.mixed_precision, self.chunk_size, self.memory_offload_freq = mixed_precision, chunk_size, memory_offload_freq
        self.flow_steps = flow_steps

    def to_rollout_config(self) -> RolloutConfig:
        return RolloutConfig(total_frames=self.max_sequence_length, chunk_frames=self.chunk_size,
                             flow_steps=self.flow_steps, window_frames=max(self.context_window, self.chunk_size))


class RolloutEvaluator:
    """Generated vs ground-truth frames: MSE, an edge-gradient L1 (perceptual proxy) and
    temporal-difference consistency (reference ``inference/rollout.py:495-546``)."""

    def __init__(self):
        self.metrics = defaultdict(list)

    @staticmethod
    def _compute_gradients(frames: torch.Tensor) -> torch.Tensor:
        gx = F.pad(frames[..., 1:] - frames[..., :-1], (0, 1))
        gy = F.pad(frames[..., 1:, :] - frames[..., :-1, :], (0, 0, 0, 1))
        return gx + gy

    def evaluate_sequence(self, generated_frames: torch.Tensor, ground_truth_frames: torch.Tensor) -> Dict[str, float]:
        g, t = generated_frames.float(), ground_truth_frames.float()
        m = {"mse": float(F.mse_loss(g, t)),
             "lpips_proxy": float(F.l1_loss(self._compute_gradients(g), self._compute_gradients(t)))}
        if g.shape[1] > 1:
            m["temporal_consistency"] = float(F.mse_loss(g[:, 1:] - g[:, :-1], t[:, 1:] - t[:, :-1]))
        for k, v in m.items():
            self.metrics[k].append(v)
        return m


class StreamingRollout:
    """Chunked flow-matching rollout of a :class:`WorldDiT` over a sliding KV window.

    Constructed as the reference's (``world_model, vae_model, config, device``,
    inference/rollout.py:158-197); ``StreamingRollout(model, config[, dtype])`` also
    works. ``config`` is a :class:`RolloutConfig` or an :class:`InferenceConfig`. With a
    VAE, :meth:`generate_sequence` takes and returns RGB frames (encoded to the model's
    latent grid, rolled out, decoded); :meth:`run` always works on latents."""

    def __init__(self, world_model: WorldDiT, vae_model=None, config=None, device=None,
                 dtype: Optional[torch.dtype] = None):
        if vae_model is not None and not isinstance(vae_model, torch.nn.Module):
            # (model, config[, dtype])
            vae_model, config, dtype = None, vae_model, (config if isinstance(config, torch.dtype) else dtype)
        if config is None:
            config = RolloutConfig()
        if isinstance(config, InferenceConfig):
            config = config.to_rollout_config()
        self.model = self.world_model = world_model
        self.vae_model = vae_model.eval() if vae_model is not None else None
        self.cfg = self.config = config
        dev = next(world_model.parameters()).device
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
        make_cache = getattr(m, "make_kv_cache", None)     # e.g. a tensor-parallel model
        fwd_chunk = getattr(m, "forward_cached_chunk", None)
        cache = (make_cache(B, cfg.window_frames, chunk, self.device, self.dtype) if make_cache is not None
                 else KVCacheSet(m, B, cfg.window_frames, chunk, self.device, self.dtype))

        def forward_cached(m_, x_, t_, a_, cache_, commit=False, extra_cond=None):
            if fwd_chunk is not None:
                return fwd_chunk(x_, t_, a_, cache_, commit, extra_cond)
            return _forward_cached(m_, x_, t_, a_, cache_, commit=commit, extra_cond=extra_cond)

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

    # ---------------------------------------------------------------- reference-style API
    def reset_state(self):
        """Rollouts keep no state between ``run`` calls (each builds its own KV window)."""

    def _encode_rgb(self, frames: torch.Tensor) -> torch.Tensor:
        """RGB ``[B, T, 3, H, W]`` in [0, 1] -> posterior-mean latents on the model's grid."""
        with torch.no_grad():
            mean, _ = self.vae_model.encode((frames.float() * 2 - 1).transpose(1, 2))
        lat = mean.transpose(1, 2).float()
        Hm, Wm = self.model.cfg.latent_h, self.model.cfg.latent_w
        lat = lat[..., :Hm, :Wm]
        return F.pad(lat, (0, Wm - lat.shape[-1], 0, Hm - lat.shape[-2]))

    def _decode_rgb(self, lat: torch.Tensor, hw) -> torch.Tensor:
        tc = getattr(self.vae_model.config, "temporal_compression", 1)
        z = lat.float().transpose(1, 2)
        with torch.no_grad():
            x = self.vae_model.decode(z, output_shape=(z.shape[2] * tc,) + tuple(hw))
        return ((x.float() + 1) / 2).clamp(0, 1).transpose(1, 2)

    def generate_sequence(self, context_frames: torch.Tensor, control_sequence: Optional[torch.Tensor] = None,
                          max_new_frames: Optional[int] = None, return_intermediates: bool = False, *,
                          controls: Optional[torch.Tensor] = None, num_frames: Optional[int] = None):
        """``context_frames [B, Fc, C, H, W]`` (latents, or RGB in [0, 1] with a VAE),
        per-frame controls ``[B, F_total, A]`` (zeros when omitted), ``max_new_frames``
        frames to generate. Returns the reference's keys (``context_frames``,
        ``generated_frames``, ``full_sequence``, ``metadata``, ``performance``) and
        ``frames`` (the generated latents), ``chunk_ms``, ``total_ms``."""
        controls = control_sequence if control_sequence is not None else controls
        n_new = max_new_frames if max_new_frames is not None else num_frames
        rgb = self.vae_model is not None and context_frames.shape[2] == 3
        lat = self._encode_rgb(context_frames.to(self.device)) if rgb else context_frames
        B, Fc = lat.shape[:2]
        total = Fc + (n_new if n_new is not None else self.cfg.total_frames - Fc)
        A = self.model.cfg.action_dim
        if controls is None:
            controls = torch.zeros(B, total, A, device=self.device)
        controls = controls.to(self.device).float()[..., :A]
        if controls.shape[1] < total:  # hold the last control
            controls = torch.cat([controls, controls[:, -1:].expand(-1, total - controls.shape[1], -1)], 1)
        res = self.run(lat, controls[:, :total], total)
        gen_lat = res.frames[:, Fc:]
        gen = self._decode_rgb(gen_lat, context_frames.shape[-2:]) if rgb else gen_lat
        n = max(gen_lat.shape[1], 1)
        mem = torch.cuda.max_memory_allocated(self.device) / 1e6 if self.device.type == "cuda" else 0.0
        out = {"context_frames": context_frames, "generated_frames": gen,
               "full_sequence": torch.cat([context_frames.to(gen.device, gen.dtype), gen], 1),
               "metadata": {"frame_times": [ms / 1e3 * len(res.chunk_ms) / n for ms in res.chunk_ms],
                            "chunk_ms": res.chunk_ms},
               "performance": {"avg_fps": 1e3 * n / res.total_ms if res.total_ms > 0 else 0.0,
                               "peak_memory_mb": mem, "avg_memory_mb": mem},
               "frames": gen_lat, "chunk_ms": res.chunk_ms, "total_ms": res.total_ms}
        if return_intermediates:
            out["all_frames"] = res.frames
        return out
