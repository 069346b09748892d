"""Flow-matching trainer for the world models (single device, DP, FSDP, FSDP + EP).

One ``train_step(batch)`` = sample noise and flow time, build ``x_t``, predict the
velocity, MSE (+ MoE aux loss, + REPA when configured), backward, AdamW. Mirrors the
reference's ``FlowMatchingTrainer.train_step`` (blocks/flow_matching.py:424-491) and the
``UnifiedTrainer`` step (training/unified_trainer.py:1095-1152) with bf16 compute on
the sm_100a path instead of fp16 autocast + GradScaler.

Parameters live in a :class:`FlatParamGroup`; on CUDA the forward/backward of every
block runs through the fused kernels and the update is one fused AdamW pass that also
writes the bf16 weights of the next step. On a process group of more than one rank the
:class:`~drivedit_b200.parallel.sharded.ShardedDataParallel` engine owns the buffers
instead (sharded AdamW state, reduce-scatter / all-gather fused into the optimizer
kernel), and with ``parallel="fsdp_ep"`` :class:`~drivedit_b200.parallel.expert.ExpertParallel`
places the routed experts.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn

from ..config import TrainConfig
from ..data.synthetic import LatentBatch
from ..parallel.flat import FlatParamGroup
from .flow_matching import interpolate, sample_t
from .optim import FlatAdamW


class WorldModelTrainer:
    def __init__(self, model: nn.Module, cfg: TrainConfig, device=None, fused: Optional[bool] = None,
                 process_group=None):
        self.model = model
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else next(model.parameters()).device
        self.model.to(self.device)
        self.cuda = self.device.type == "cuda"
        self.compute_dtype = torch.bfloat16 if (self.cuda and cfg.dtype == "bf16") else torch.float32
        self.pg = process_group
        if self.cuda and getattr(cfg, "deterministic", False):
            from ..ops.debug import set_deterministic

            set_deterministic(True)
        self.engine = None
        self.ep = None
        world = torch.distributed.get_world_size(process_group) if process_group is not None else 1
        if world > 1:
            from ..parallel.sharded import ShardedDataParallel

            transport = "fused" if (self.cuda and cfg.fused_collectives) else "nccl"
            local = None
            moe_cfg = getattr(getattr(model, "cfg", None), "moe", None)
            if cfg.parallel == "fsdp_ep" and moe_cfg is not None:
                from ..parallel.expert import ExpertParallel

                # expert parallelism over the whole data-parallel group
                self.ep = ExpertParallel(process_group, moe_cfg.num_experts, transport, self.device)
                local = model.enable_expert_parallel(self.ep)
            self.engine = ShardedDataParallel(model, process_group, self.device, transport,
                                              cfg.lr, cfg.betas, cfg.eps, cfg.weight_decay,
                                              cfg.grad_clip, local_params=local,
                                              weight_gather=getattr(cfg, "shard_weights", False),
                                              overlap=getattr(cfg, "overlap_grad_reduce", False))
            self.group = self.engine.flat
            self.opt = None
        else:
            named = model.named_parameters()
            if hasattr(model, "flat_layout"):
                named = model.flat_layout(named)
            # on the CPU every op reads the fp32 master: no separate compute copy
            self.group = FlatParamGroup(named, self.device, no_decay=model.no_decay_names(),
                                        compute_dtype=torch.bfloat16 if self.cuda else torch.float32)
            self.opt = FlatAdamW(self.group, cfg.lr, cfg.betas, cfg.eps, cfg.weight_decay,
                                 cfg.grad_clip)
        self.fused = self.cuda if fused is None else fused
        if self.fused:
            model.enable_fused(group=self.group)
            model.fused.recompute = bool(getattr(cfg, "checkpoint_blocks", False))
            if self.engine is not None and self.engine.pieces is not None:
                model.fused.grad_ready = self.engine.bucket_ready
        self.gen = torch.Generator(device=self.device)
        self.gen.manual_seed(cfg.seed + 1)
        self.step_idx = 0
        self.teacher = None
        rp = getattr(getattr(model, "cfg", None), "repa", None)
        if rp is not None:
            self._build_teacher(rp)
        self.last_losses: Dict[str, torch.Tensor] = {}

    def _build_teacher(self, rp):
        """Frozen ViT teacher (the V-JEPA encoder with 2-D patches: tubelet 1, one frame
        per image) applied to every RGB frame; its layer ``rp.feature_layer`` (-1: last)
        patch features, frame-major like the DiT tokens, are what the DiT's
        layer-``rp.layer`` hidden states are aligned to (cosine, weight ``rp.weight``).
        Random-init unless weights are loaded into ``self.teacher``."""
        from ..models.vjepa import VJEPABackbone, VJEPAConfig

        tl = rp.feature_layer if rp.feature_layer >= 0 else rp.teacher_layers - 1
        self.teacher_layer = tl
        vcfg = VJEPAConfig(embed_dim=rp.teacher_dim, num_layers=rp.teacher_layers,
                           num_heads=rp.teacher_heads, patch_size=rp.teacher_patch,
                           tubelet_size=1, num_frames=1,
                           image_size=(rp.image_h, rp.image_w), extract_layers=[tl])
        g = torch.random.get_rng_state()
        torch.manual_seed(self.cfg.seed + 7)
        self.teacher = VJEPABackbone(vcfg).to(self.device)
        torch.random.set_rng_state(g)

    def loss(self, batch: LatentBatch) -> torch.Tensor:
        x1 = batch.latents.to(self.compute_dtype)
        B = x1.shape[0]
        x0 = torch.randn(x1.shape, device=x1.device, generator=self.gen, dtype=torch.float32)
        t = sample_t(B, self.cfg.t_sampling, x1.device, self.gen)
        x_t = interpolate(x0, x1.float(), t).to(self.compute_dtype)
        target = (x1.float() - x0)
        if self.teacher is None:
            v, aux = self.model(x_t, t, batch.actions, return_aux=True)
            mse = (v.float() - target).pow(2).mean()
            self.last_losses = {"mse": mse.detach(), "aux": aux.detach()}
            return mse + aux
        rp = self.model.cfg.repa
        v, aux, feats = self.model(x_t, t, batch.actions, return_aux=True,
                                   return_features=rp.layer)
        mse = (v.float() - target).pow(2).mean()
        with torch.no_grad():
            rgb = batch.rgb  # [B, F, 3, Hi, Wi] -> B*F single-frame clips [B*F, 3, 1, Hi, Wi]
            clips = rgb.reshape(-1, *rgb.shape[2:]).unsqueeze(2)
            tf = self.teacher(clips, max_layer=self.teacher_layer)["intermediate"]
            tfeat = tf[f"layer_{self.teacher_layer}"].reshape(B, -1, self.teacher.config.embed_dim)
        from .repa import alignment_loss

        proj = self.model.repa_head(feats.reshape(B, -1, feats.shape[-1]))
        repa = alignment_loss(proj, tfeat, "cosine")
        self.last_losses = {"mse": mse.detach(), "aux": aux.detach(), "repa": repa.detach()}
        return mse + aux + rp.weight * repa

    def train_step(self, batch: LatentBatch) -> torch.Tensor:
        self.group.zero_grad()
        loss = self.loss(batch)
        if self.engine is not None:
            self.engine.arm_overlap()  # one backward, then the step: buckets reduce as they finish
        loss.backward()
        if self.engine is not None:
            self.engine.step()
        else:
            self.opt.step()
        self.step_idx += 1
        return loss.detach()

    def close(self):
        """Release the symmetric (CUDA-IPC) buffers of the sharded and expert-parallel
        engines; every rank calls it at the same point."""
        if self.engine is not None:
            self.engine.close()
        if self.ep is not None:
            self.ep.close()

    def state_dict(self) -> Dict:
        if self.engine is not None:
            self.engine.gather_weights()   # weight-sharded mode: materialise full weights
        opt = self.opt.state_dict() if self.opt is not None else {
            "m": self.engine.m, "v": self.engine.v, "step": self.engine.step_count}
        if self.engine is not None and self.engine.local_opt is not None:
            opt["local"] = self.engine.local_opt.state_dict()   # this rank's experts
        return {"model": self.model.state_dict(), "optim": opt, "step": self.step_idx}

    def load_state_dict(self, sd: Dict):
        self.model.load_state_dict(sd["model"])
        self.group.refresh_compute()
        if self.opt is not None:
            self.opt.load_state_dict(sd["optim"])
        else:
            self.engine.m.copy_(sd["optim"]["m"])
            self.engine.v.copy_(sd["optim"]["v"])
            self.engine.step_count = int(sd["optim"]["step"])
            if self.engine.local_opt is not None and "local" in sd["optim"]:
                self.engine.local_opt.load_state_dict(sd["optim"]["local"])
        self.step_idx = int(sd["step"])
