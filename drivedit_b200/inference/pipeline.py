"""End-to-end inference pipelines: RGB context frames -> VAE latents -> streaming
rollout of the world model -> VAE decode -> RGB frames.

API of the reference ``inference/pipeline.py``: ``PipelineConfig`` (:22-34),
``InferencePipeline`` (load models, preprocess, generate, postprocess, :37-302),
``BatchInferencePipeline`` (:305-369), ``RealtimeInferencePipeline`` (frame-by-frame
streaming with a rolling context, :372-458), ``MultiModelPipeline`` (ensembles,
:461-538) and ``create_pipeline`` (:541-575).

Built on this framework's pieces: ``WorldDiT`` + ``StreamingRollout`` (chunked Euler
flow sampling over a rolling KV window, fused kernels on CUDA) and ``VAE3D`` (causal
conv3d kernels on CUDA). Without a VAE the pipeline works on latents directly. Weights
come from checkpoints when paths are given (reference-format keys accepted), otherwise
random init. Timing uses CUDA events.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

import numpy as np
import torch

from ..config import RolloutConfig, get_config
from ..models.world_dit import WorldDiT
from .rollout import StreamingRollout


@dataclass
class PipelineConfig:
    """The reference's fields in its order (inference/pipeline.py:23-34), then this
    framework's settings. Of the reference's, ``max_sequence_length``, ``context_window``,
    ``temperature`` and ``cache_models`` are accepted and recorded only: the number of
    frames is the ``num_frames`` of each call, the KV window is ``window_frames``,
    sampling is the deterministic flow ODE and the models stay resident."""
    model_path: Optional[str] = None
    vae_path: Optional[str] = None
    device: str = "cuda"
    batch_size: int = 1
    max_sequence_length: int = 64
    context_window: int = 8
    temperature: float = 0.8
    use_mixed_precision: bool = True
    use_torch_compile: bool = False       # accepted for API parity; kernels are fused already
    cache_models: bool = True
    model_preset: str = "rollout_dit_b"
    model_overrides: List[str] = field(default_factory=list)
    use_vae: bool = True
    vae_hidden_dims: List[int] = field(default_factory=lambda: [128, 256, 512, 512])
    vae_use_attention: bool = True
    image_size: tuple = (256, 512)
    chunk_frames: int = 4
    flow_steps: int = 4
    window_frames: int = 32
    seed: int = 0


class InferencePipeline:
    def __init__(self, config: PipelineConfig):
        self.config = config
        dev = config.device if (config.device != "cuda" or torch.cuda.is_available()) else "cpu"
        self.device = torch.device(dev)
        self.dtype = torch.bfloat16 if (self.device.type == "cuda" and config.use_mixed_precision) else torch.float32
        self.cfg = get_config(config.model_preset, config.model_overrides)
        self.model = self._load_student_model(config.model_path)
        self.vae = self._load_vae_model(config.vae_path) if config.use_vae else None
        rc = RolloutConfig(total_frames=0, chunk_frames=config.chunk_frames, flow_steps=config.flow_steps,
                           window_frames=config.window_frames, context_frames=1, batch=config.batch_size)
        self.rollout = StreamingRollout(self.model, rc, self.dtype)
        self.gen = torch.Generator(device=self.device).manual_seed(config.seed)

    # ------------------------------------------------------------------ models
    def _load_student_model(self, model_path: Optional[str]) -> WorldDiT:
        torch.manual_seed(self.config.seed)
        m = WorldDiT(self.cfg.model)
        if model_path:
            sd = torch.load(model_path, map_location="cpu")
            sd = sd.get("model", sd.get("model_state_dict", sd))
            m.load_state_dict(self._create_model_from_state_dict(sd), strict=False)
        m.to(self.device).eval()
        if self.device.type == "cuda":
            from ..parallel.flat import FlatParamGroup

            m.enable_fused(group=FlatParamGroup(m.flat_layout(m.named_parameters()), self.device))
        return m

    @staticmethod
    def _create_model_from_state_dict(state_dict: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        """Strips wrapper prefixes (``module.``, ``_orig_mod.``)."""
        out = {}
        for k, v in state_dict.items():
            for p in ("module.", "_orig_mod."):
                if k.startswith(p):
                    k = k[len(p):]
            out[k] = v
        return out

    def _load_vae_model(self, vae_path: Optional[str]):
        from ..models.vae3d import VAE3D, VAE3DConfig

        vc = VAE3DConfig(latent_dim=self.cfg.model.latent_channels, hidden_dims=list(self.config.vae_hidden_dims),
                         use_attention=self.config.vae_use_attention, use_perceptual_loss=False,
                         use_gradient_checkpointing=False)
        vae = VAE3D(vc)
        if vae_path:
            sd = torch.load(vae_path, map_location="cpu")
            vae.load_state_dict(self._create_model_from_state_dict(sd.get("model", sd)), strict=False)
        return vae.to(self.device).eval()

    def _compile_models(self):
        """Kept for API parity: the CUDA path is hand-written kernels, nothing to trace."""
        return self

    # ------------------------------------------------------------------ io
    def preprocess_input(self, context_frames: torch.Tensor, controls: Optional[torch.Tensor] = None,
                         num_frames: int = 16) -> Dict[str, torch.Tensor]:
        """``context_frames``: RGB ``[B, T, H, W, 3]`` uint8 / ``[B, T, 3, H, W]`` float in
        [0, 1] (with a VAE) or latents ``[B, T, C, h, w]`` (without). ``controls``:
        ``[B, T_total, A]`` per-frame actions in [-1, 1] (zeros when omitted)."""
        x = context_frames.to(self.device)
        B = x.shape[0]
        if self.vae is not None:
            if x.dtype == torch.uint8:
                x = x.permute(0, 1, 4, 2, 3).float() / 255.0
            x = x.float() * 2 - 1                                   # [B, T, 3, H, W]
            self._img_hw = tuple(x.shape[-2:])
            with torch.no_grad():
                mean, _ = self.vae.encode(x.transpose(1, 2))
            lat = mean.transpose(1, 2).float()                      # [B, T', C, h, w]
            # the VAE's stride-2 / padding-2 downsampling yields h = H/8 + 1 style extents:
            # crop (or zero-pad) to the world model's latent grid; decode restores H x W
            Hm, Wm = self.cfg.model.latent_h, self.cfg.model.latent_w
            lat = lat[..., :Hm, :Wm]
            if lat.shape[-2:] != (Hm, Wm):
                lat = torch.nn.functional.pad(lat, (0, Wm - lat.shape[-1], 0, Hm - lat.shape[-2]))
        else:
            lat = x.float()
        tc = self.vae.config.temporal_compression if self.vae is not None else 1
        n_lat = lat.shape[1] + -(-num_frames // tc)
        A = self.cfg.model.action_dim
        if controls is None:
            act = torch.zeros(B, n_lat, A, device=self.device)
        else:
            c = controls.to(self.device).float()[..., :A]
            if c.shape[1] != n_lat:  # per-RGB-frame controls -> one per latent frame
                idx = torch.linspace(0, c.shape[1] - 1, n_lat, device=self.device).round().long()
                c = c[:, idx]
            act = c
        return {"latents": lat.to(self.dtype), "actions": act, "total_latent_frames": n_lat}

    def postprocess_output(self, result: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        out = {}
        for k in ("generated_frames", "context_frames"):
            v = result[k]
            if v.dim() == 5 and v.shape[2] == 3:
                v = (v.clamp(0, 1) * 255).round().to(torch.uint8).permute(0, 1, 3, 4, 2)
            out[k] = v.cpu().numpy()
        out["metadata"], out["performance"] = result["metadata"], result["performance"]
        return out

    def _decode(self, lat: torch.Tensor) -> torch.Tensor:
        if self.vae is None:
            return lat.float()
        tc = self.vae.config.temporal_compression
        H, W = getattr(self, "_img_hw", (lat.shape[-2] * self.vae.config.spatial_compression,
                                         lat.shape[-1] * self.vae.config.spatial_compression))
        z = lat.float().transpose(1, 2).to(torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        with torch.no_grad():
            x = self.vae.decode(z, output_shape=(z.shape[2] * tc, H, W))
        return ((x.float() + 1) / 2).clamp(0, 1).transpose(1, 2)

    @torch.no_grad()
    def generate(self, context_frames: torch.Tensor, controls: Optional[torch.Tensor] = None,
                 num_frames: int = 16, return_dict: bool = True, decode: bool = True) -> Dict[str, Any]:
        t0 = time.perf_counter()
        inp = self.preprocess_input(context_frames, controls, num_frames)
        lat, act = inp["latents"], inp["actions"]
        Fc = lat.shape[1]
        res = self.rollout.run(lat, act, total_frames=inp["total_latent_frames"], generator=self.gen)
        gen_lat = res.frames[:, Fc:]
        gen = self._decode(gen_lat) if decode else gen_lat.float()
        ctx = self._decode(lat) if decode else lat.float()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        wall = time.perf_counter() - t0
        n_out = gen.shape[1]
        result = {"generated_frames": gen, "context_frames": ctx, "generated_latents": gen_lat,
                  "metadata": {"num_context_frames": int(context_frames.shape[1]), "num_generated": int(n_out),
                               "latent_frames": int(gen_lat.shape[1]), "model": self.cfg.model.name},
                  "performance": {"total_ms": wall * 1000.0, "rollout_ms": float(sum(res.chunk_ms)),
                                  "fps": float(n_out * gen.shape[0] / max(wall, 1e-9)),
                                  "p50_chunk_ms": res.percentile_ms(50)}}
        return result if return_dict else gen


class BatchInferencePipeline(InferencePipeline):
    def generate_batch(self, context_list: Sequence[torch.Tensor], controls_list=None,
                       num_frames: int = 16) -> List[Dict[str, Any]]:
        """Independent requests batched ``batch_size`` at a time (same context shape)."""
        out = []
        bs = self.config.batch_size
        for i in range(0, len(context_list), bs):
            ctx = torch.cat([c if c.dim() == 5 else c[None] for c in context_list[i:i + bs]], 0)
            ctl = None
            if controls_list is not None:
                ctl = torch.cat([c if c.dim() == 3 else c[None] for c in controls_list[i:i + bs]], 0)
            r = self.generate(ctx, ctl, num_frames)
            for j in range(ctx.shape[0]):
                out.append({"generated_frames": r["generated_frames"][j:j + 1],
                            "metadata": r["metadata"], "performance": r["performance"]})
        return out


class RealtimeInferencePipeline(InferencePipeline):
    """Streaming: frames arrive one by one (RGB or latent); once ``context`` frames have
    been seen, each call returns the next predicted frame conditioned on the latest
    control (generated a chunk at a time, served frame by frame)."""

    def __init__(self, config: PipelineConfig, context: int = 4):
        super().__init__(config)
        self.context = context
        self.buffer: List[torch.Tensor] = []
        self.controls: List[torch.Tensor] = []
        self.pending: List[torch.Tensor] = []
        self.streaming = False

    def start_streaming(self):
        self.streaming = True
        self.buffer, self.controls, self.pending = [], [], []

    def stop_streaming(self):
        self.streaming = False
        self.buffer, self.controls, self.pending = [], [], []

    @torch.no_grad()
    def process_frame(self, frame, control=None):
        if not self.streaming:
            self.start_streaming()
        f = torch.as_tensor(np.asarray(frame)) if not torch.is_tensor(frame) else frame
        self.buffer.append(f)
        A = self.cfg.model.action_dim
        c = torch.zeros(A) if control is None else torch.as_tensor(np.asarray(control), dtype=torch.float32)[:A]
        self.controls.append(F_pad(c, A))
        if self.pending:
            return self.pending.pop(0)
        if len(self.buffer) < self.context:
            return None
        ctx = torch.stack(self.buffer[-self.context:])[None]
        ctl = torch.stack(self.controls[-self.context:])[None]  # resampled per latent frame
        r = self.generate(ctx, ctl, num_frames=self.config.chunk_frames)
        frames = r["generated_frames"][0]
        if frames.dim() == 4 and frames.shape[1] == 3:
            frames = (frames.clamp(0, 1) * 255).round().to(torch.uint8).permute(0, 2, 3, 1)
        self.pending = [fr.cpu().numpy() for fr in frames]
        return self.pending.pop(0)


def F_pad(c: torch.Tensor, n: int) -> torch.Tensor:
    return torch.nn.functional.pad(c.float(), (0, max(0, n - c.numel())))


class MultiModelPipeline:
    def __init__(self, model_configs: List[PipelineConfig]):
        self.pipelines = [InferencePipeline(c) for c in model_configs]

    @torch.no_grad()
    def generate_ensemble(self, context_frames, controls=None, num_frames: int = 16,
                          weights: Optional[Sequence[float]] = None) -> Dict[str, Any]:
        outs = [p.generate(context_frames, controls, num_frames) for p in self.pipelines]
        w = torch.tensor(weights if weights is not None else [1.0] * len(outs), dtype=torch.float32)
        w = w / w.sum()
        gen = sum(wi * o["generated_frames"].float().cpu() for wi, o in zip(w.tolist(), outs))
        return {"generated_frames": gen, "individual": outs,
                "performance": {"total_ms": sum(o["performance"]["total_ms"] for o in outs)}}


def create_pipeline(model_path: Optional[str] = None, vae_path: Optional[str] = None,
                    pipeline_type: str = "standard", device: str = "cuda", **kwargs):
    """``standard``, ``batch`` or ``realtime`` pipeline (inference/pipeline.py:541-575)."""
    if pipeline_type not in ("standard", "batch", "realtime"):
        raise ValueError(f"Unsupported pipeline type: {pipeline_type}")
    cfg = PipelineConfig(model_path=model_path, vae_path=vae_path, device=device,
                         **{k: v for k, v in kwargs.items() if k in PipelineConfig.__dataclass_fields__})
    if pipeline_type == "batch":
        return BatchInferencePipeline(cfg)
    if pipeline_type == "realtime":
        return RealtimeInferencePipeline(cfg)
    return InferencePipeline(cfg)
