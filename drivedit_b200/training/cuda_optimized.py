"""Generic GPU training helpers (the reference's ``training/cuda_optimized.py`` interface:
``CUDAOptimizedConfig``, ``CUDAStream``, ``AsyncPrefetcher``, ``CUDADataPipeline``,
``CUDAControlNormalizer``, ``GradientAccumulator``, ``MemoryOptimizer``,
``OptimizedTrainer``, ``setup_distributed``, ``cleanup_distributed``,
``create_optimized_optimizer``, ``create_cosine_scheduler``) for arbitrary ``nn.Module``s.

The world models train through :class:`~drivedit_b200.training.trainer.WorldModelTrainer`
(fused sm_100a engine, flat-buffer AdamW, peer-memory sharded optimizer); these helpers are
for other models a user brings. B200 choices: mixed precision is bf16 autocast (no loss
scaler; ``grad_scaler_enabled`` only matters for fp16); ``use_fsdp`` shards the optimizer
with :class:`~drivedit_b200.parallel.sharded.ShardedDataParallel` (the reference's
``SHARD_GRAD_OP`` schedule, ``:571-615``) instead of wrapping in torch FSDP; no tracing
compiler (``compile_mode`` is accepted and ignored); the H2D prefetcher copies the next
batch on side streams and the compute stream waits on an event, so copies overlap the step.
"""
from __future__ import annotations

import contextlib
import logging
import math
import queue
from dataclasses import dataclass
from typing import Any, Callable, Dict, Iterator, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.utils.data import DataLoader, Dataset

logger = logging.getLogger(__name__)


@dataclass
class CUDAOptimizedConfig:
    prefetch_batches: int = 2
    num_streams: int = 2
    pin_memory: bool = True
    persistent_workers: bool = True
    num_workers: int = 4
    compile_mode: str = "none"
    compile_fullgraph: bool = False
    compile_dynamic: bool = False
    use_amp: bool = True
    amp_dtype: torch.dtype = torch.bfloat16
    grad_scaler_enabled: bool = True
    grad_scaler_growth_interval: int = 2000
    gradient_accumulation_steps: int = 1
    gradient_clip_norm: float = 1.0
    gradient_checkpointing: bool = False
    checkpoint_every_n_layers: int = 2
    empty_cache_interval: int = 100
    max_memory_fraction: float = 0.95
    offload_to_cpu: bool = False
    use_fsdp: bool = False
    fsdp_sharding_strategy: str = "SHARD_GRAD_OP"
    fsdp_mixed_precision: bool = True
    fsdp_cpu_offload: bool = False
    fsdp_min_num_params: int = 1_000_000
    enable_profiling: bool = False
    profile_warmup_steps: int = 10
    profile_active_steps: int = 5


class CUDAStream:
    """Context manager making ``stream`` current (restores the previous stream on exit)."""

    def __init__(self, stream: Optional[torch.cuda.Stream] = None):
        self.stream = stream or torch.cuda.Stream()
        self._prev = None

    def __enter__(self):
        self._prev = torch.cuda.current_stream()
        torch.cuda.set_stream(self.stream)
        return self

    def __exit__(self, *args):
        torch.cuda.set_stream(self._prev)

    def synchronize(self):
        self.stream.synchronize()

    def wait_stream(self, other: "CUDAStream"):
        self.stream.wait_stream(other.stream)


def _to_device(obj, device, non_blocking=True):
    if torch.is_tensor(obj):
        return obj.to(device, non_blocking=non_blocking)
    if isinstance(obj, dict):
        return {k: _to_device(v, device, non_blocking) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_device(v, device, non_blocking) for v in obj)
    if hasattr(obj, "to"):
        return obj.to(device, non_blocking=non_blocking)
    return obj


def _record_stream(obj, stream):
    if torch.is_tensor(obj) and obj.is_cuda:
        obj.record_stream(stream)
    elif isinstance(obj, dict):
        for v in obj.values():
            _record_stream(v, stream)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            _record_stream(v, stream)


class AsyncPrefetcher:
    """Iterates a DataLoader with the next ``num_streams`` batches already copying to the
    GPU on side streams; each batch is handed out after the current stream waits for its
    copy event (and its memory is tied to the consuming stream)."""

    def __init__(self, dataloader, device: torch.device, num_streams: int = 2):
        self.dataloader, self.device = dataloader, torch.device(device)
        self.num_streams = max(1, num_streams)
        self.cuda = self.device.type == "cuda"
        self.streams = [torch.cuda.Stream(self.device) for _ in range(self.num_streams)] if self.cuda else []
        self.prefetch_queue: "queue.Queue" = queue.Queue()
        self.iterator: Optional[Iterator] = None
        self.exhausted = False
        self._i = 0

    def _to_cuda_async(self, batch):
        if not self.cuda:
            return batch, None
        s = self.streams[self._i % self.num_streams]
        self._i += 1
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            out = _to_device(batch, self.device)
            ev = torch.cuda.Event()
            ev.record(s)
        return out, ev

    def _prefetch_next(self):
        try:
            self.prefetch_queue.put(self._to_cuda_async(next(self.iterator)))
        except StopIteration:
            self.exhausted = True

    def __iter__(self):
        self.iterator = iter(self.dataloader)
        self.exhausted = False
        self.prefetch_queue = queue.Queue()
        for _ in range(self.num_streams):
            self._prefetch_next()
        return self

    def __next__(self):
        if self.prefetch_queue.empty():
            raise StopIteration
        batch, ev = self.prefetch_queue.get()
        if ev is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(ev)
            _record_stream(batch, cur)
        if not self.exhausted:
            self._prefetch_next()
        return batch

    def __len__(self):
        return len(self.dataloader)


class CUDADataPipeline:
    """Pinned-memory DataLoader + :class:`AsyncPrefetcher`; an optional ``gpu_transform``
    (e.g. the fused clip augmentation of :mod:`drivedit_b200.data.transforms`) runs on the
    device batch."""

    def __init__(self, dataset: Dataset, batch_size: int, config: CUDAOptimizedConfig,
                 device: Optional[torch.device] = None, gpu_transform: Optional[Callable] = None,
                 shuffle: bool = True):
        self.config = config
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        nw = config.num_workers
        self.dataloader = DataLoader(dataset, batch_size=batch_size, shuffle=shuffle, num_workers=nw,
                                     pin_memory=config.pin_memory and self.device.type == "cuda",
                                     persistent_workers=config.persistent_workers and nw > 0,
                                     drop_last=True, prefetch_factor=2 if nw > 0 else None)
        self.gpu_transform = gpu_transform
        self.prefetcher = AsyncPrefetcher(self.dataloader, self.device, config.num_streams)

    def __iter__(self) -> Iterator[Any]:
        for b in self.prefetcher:
            yield self.gpu_transform(b) if self.gpu_transform is not None else b

    def __len__(self) -> int:
        return len(self.dataloader)


class CUDAControlNormalizer(nn.Module):
    """Running-statistics normalisation of control vectors, ``(x - mean) / sqrt(var + eps)``,
    plus a homogeneous ego-frame transform of positions."""

    def __init__(self, control_dim: int, use_compile: bool = False, momentum: float = 0.1, eps: float = 1e-5):
        super().__init__()
        self.control_dim, self.momentum, self.eps = control_dim, momentum, eps
        self.register_buffer("running_mean", torch.zeros(control_dim))
        self.register_buffer("running_var", torch.ones(control_dim))
        self.register_buffer("num_batches_tracked", torch.tensor(0, dtype=torch.long))
        self.register_buffer("ego_transform", torch.eye(4))

    def forward(self, controls: torch.Tensor, update_stats: bool = True) -> torch.Tensor:
        flat = controls.reshape(-1, self.control_dim).float()
        if self.training and update_stats:
            with torch.no_grad():
                m = self.momentum
                self.running_mean.mul_(1 - m).add_(flat.mean(0), alpha=m)
                self.running_var.mul_(1 - m).add_(flat.var(0, unbiased=flat.shape[0] > 1), alpha=m)
                self.num_batches_tracked += 1
        out = (flat - self.running_mean) * torch.rsqrt(self.running_var + self.eps)
        return out.view_as(controls).to(controls.dtype)

    def transform_ego(self, positions: torch.Tensor) -> torch.Tensor:
        """``[..., 3]`` world positions -> ego frame through the 4x4 transform."""
        h = torch.cat([positions, torch.ones_like(positions[..., :1])], -1)
        return (h @ self.ego_transform.T.to(h.dtype))[..., :3]

    def set_ego_transform(self, transform_matrix: torch.Tensor):
        self.ego_transform.copy_(transform_matrix)


class GradientAccumulator:
    """Scales the loss by ``1 / steps`` and says when an optimizer step is due."""

    def __init__(self, accumulation_steps: int = 1, scaler=None):
        self.accumulation_steps = max(1, accumulation_steps)
        self.scaler = scaler
        self.current_step = 0

    def scale_loss(self, loss: torch.Tensor) -> torch.Tensor:
        loss = loss / self.accumulation_steps
        return self.scaler.scale(loss) if self.scaler is not None else loss

    def step(self) -> bool:
        self.current_step += 1
        return self.current_step % self.accumulation_steps == 0

    def reset(self):
        self.current_step = 0


class MemoryOptimizer:
    def __init__(self, config: CUDAOptimizedConfig):
        self.config = config
        self.step_count = 0

    def maybe_empty_cache(self):
        self.step_count += 1
        if torch.cuda.is_available() and self.config.empty_cache_interval and \
                self.step_count % self.config.empty_cache_interval == 0:
            torch.cuda.empty_cache()

    def get_memory_stats(self) -> Dict[str, float]:
        if not torch.cuda.is_available():
            return {}
        return {"allocated_gb": torch.cuda.memory_allocated() / 1e9,
                "reserved_gb": torch.cuda.memory_reserved() / 1e9,
                "max_allocated_gb": torch.cuda.max_memory_allocated() / 1e9}

    def enable_memory_efficient_attention(self, model: nn.Module):
        """This framework's attention layers are flash-style already (no S x S matrix)."""
        return model

    @contextlib.contextmanager
    def memory_checkpoint_context(self, model: nn.Module):
        """Turns on activation checkpointing for blocks that support it while inside."""
        flagged = []
        if self.config.gradient_checkpointing:
            for m in model.modules():
                if hasattr(m, "gradient_checkpointing") and not m.gradient_checkpointing:
                    m.gradient_checkpointing = True
                    flagged.append(m)
        try:
            yield
        finally:
            for m in flagged:
                m.gradient_checkpointing = False


class OptimizedTrainer:
    """bf16 autocast, gradient accumulation, clipping, periodic cache trimming, optional
    profiler; ``use_fsdp`` (with an initialised process group) shards the optimizer over
    the ranks through :class:`ShardedDataParallel` and its step replaces ``optimizer``'s."""

    def __init__(self, model: nn.Module, config: CUDAOptimizedConfig, device: Optional[torch.device] = None,
                 lr: float = 1e-4, weight_decay: float = 0.01):
        self.config = config
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda" if torch.cuda.is_available() else "cpu")
        self.engine = None
        self.model = self._setup_model(model, lr, weight_decay)
        on_cuda = self.device.type == "cuda"
        self.amp_context = (lambda: torch.autocast("cuda", dtype=config.amp_dtype)) if (config.use_amp and on_cuda) \
            else contextlib.nullcontext
        fp16 = config.amp_dtype == torch.float16 and config.use_amp and on_cuda
        self.scaler = torch.amp.GradScaler("cuda", growth_interval=config.grad_scaler_growth_interval) \
            if (fp16 and config.grad_scaler_enabled) else None
        self.accumulator = GradientAccumulator(config.gradient_accumulation_steps, self.scaler)
        self.memory_optimizer = MemoryOptimizer(config)
        self.profiler = self._setup_profiler() if config.enable_profiling else None
        self.global_step = 0
        self.compiled = False

    def _setup_model(self, model: nn.Module, lr: float, wd: float) -> nn.Module:
        model = model.to(self.device)
        if self.config.use_fsdp and dist.is_initialized() and dist.get_world_size() > 1:
            self.engine = self._wrap_fsdp(model, lr, wd)
        return model

    def _wrap_fsdp(self, model: nn.Module, lr: float, wd: float):
        from ..parallel.sharded import ShardedDataParallel

        transport = "fused" if self.device.type == "cuda" else "nccl"
        return ShardedDataParallel(model, device=self.device, transport=transport, lr=lr, weight_decay=wd,
                                   grad_clip=self.config.gradient_clip_norm)

    def _setup_profiler(self):
        acts = [torch.profiler.ProfilerActivity.CPU]
        if self.device.type == "cuda":
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        c = self.config
        p = torch.profiler.profile(activities=acts, schedule=torch.profiler.schedule(
            wait=0, warmup=c.profile_warmup_steps, active=c.profile_active_steps, repeat=1))
        p.start()
        return p

    def train_step(self, batch: Dict[str, torch.Tensor], optimizer: Optional[torch.optim.Optimizer],
                   loss_fn: Callable) -> Dict[str, float]:
        self.model.train()
        batch = _to_device(batch, self.device)
        with self.amp_context():
            outputs = self.model(**batch) if isinstance(batch, dict) else self.model(batch)
            losses = loss_fn(outputs, batch)
        loss = losses["total"] if isinstance(losses, dict) else losses
        self.accumulator.scale_loss(loss).backward()
        stepped = self.accumulator.step()
        gnorm = float("nan")
        if stepped:
            if self.engine is not None:
                self.engine.step()
                self.engine.zero_grad()
            else:
                if self.scaler is not None:
                    self.scaler.unscale_(optimizer)
                if self.config.gradient_clip_norm > 0:
                    gnorm = float(torch.nn.utils.clip_grad_norm_(self.model.parameters(),
                                                                 self.config.gradient_clip_norm))
                if self.scaler is not None:
                    self.scaler.step(optimizer)
                    self.scaler.update()
                else:
                    optimizer.step()
                optimizer.zero_grad(set_to_none=True)
        self.global_step += 1
        self.memory_optimizer.maybe_empty_cache()
        if self.profiler is not None:
            self.profiler.step()
        out = {"loss": float(loss.detach()), "stepped": float(stepped), "grad_norm": gnorm}
        if isinstance(losses, dict):
            out.update({k: float(v.detach()) for k, v in losses.items() if torch.is_tensor(v) and v.dim() == 0})
        return out

    @torch.no_grad()
    def validate_step(self, batch: Dict[str, torch.Tensor], loss_fn: Callable) -> Dict[str, float]:
        self.model.eval()
        batch = _to_device(batch, self.device)
        with self.amp_context():
            outputs = self.model(**batch) if isinstance(batch, dict) else self.model(batch)
            losses = loss_fn(outputs, batch)
        loss = losses["total"] if isinstance(losses, dict) else losses
        return {"val_loss": float(loss)}

    def train_epoch(self, dataloader, optimizer, loss_fn: Callable, scheduler=None) -> Dict[str, float]:
        tot, n = 0.0, 0
        for batch in dataloader:
            m = self.train_step(batch, optimizer, loss_fn)
            if scheduler is not None and m["stepped"]:
                scheduler.step()
            tot += m["loss"]
            n += 1
        return {"loss": tot / max(n, 1), "steps": n}

    def save_checkpoint(self, path: str, optimizer=None, scheduler=None, **extra):
        from pathlib import Path

        from .distributed import _atomic_save

        ck = {"model": self.model.state_dict(), "global_step": self.global_step, **extra}
        if optimizer is not None:
            ck["optimizer"] = optimizer.state_dict()
        if scheduler is not None:
            ck["scheduler"] = scheduler.state_dict()
        if self.engine is not None:
            ck["sharded_m"], ck["sharded_v"] = self.engine.m, self.engine.v
            ck["sharded_step"] = self.engine.step_count
        _atomic_save(ck, Path(path))

    def load_checkpoint(self, path: str, optimizer=None, scheduler=None) -> Dict[str, Any]:
        from pathlib import Path

        from .distributed import _verified_load

        ck = _verified_load(Path(path))
        self.model.load_state_dict(ck["model"])
        if optimizer is not None and "optimizer" in ck:
            optimizer.load_state_dict(ck["optimizer"])
        if scheduler is not None and "scheduler" in ck:
            scheduler.load_state_dict(ck["scheduler"])
        if self.engine is not None and "sharded_m" in ck:
            self.engine.m.copy_(ck["sharded_m"])
            self.engine.v.copy_(ck["sharded_v"])
            self.engine.step_count = ck["sharded_step"]
            self.engine.flat.refresh_compute()
        self.global_step = ck.get("global_step", 0)
        return ck


def setup_distributed(rank: int, world_size: int, backend: str = "nccl"):
    from .distributed import DistributedManager

    m = DistributedManager()
    m.setup(rank, world_size, backend)
    return m


def cleanup_distributed():
    if dist.is_initialized():
        dist.destroy_process_group()


def create_optimized_optimizer(model: nn.Module, lr: float = 1e-4, weight_decay: float = 0.01,
                               betas: Tuple[float, float] = (0.9, 0.999), use_fused: bool = True
                               ) -> torch.optim.Optimizer:
    """AdamW with biases, norms and embeddings excluded from weight decay."""
    decay, no_decay = [], []
    for n, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (no_decay if ("bias" in n or "norm" in n or "embedding" in n) else decay).append(p)
    groups = [{"params": decay, "weight_decay": weight_decay}, {"params": no_decay, "weight_decay": 0.0}]
    on_cuda = any(p.is_cuda for p in model.parameters())
    return torch.optim.AdamW(groups, lr=lr, betas=betas, fused=bool(use_fused and on_cuda))


def create_cosine_scheduler(optimizer: torch.optim.Optimizer, total_steps: int, warmup_steps: int,
                            min_lr: float = 1e-6):
    """Linear warm-up then cosine decay, floored at ``min_lr``."""
    base = optimizer.defaults["lr"]

    def lr_lambda(step: int) -> float:
        if step < warmup_steps:
            return step / max(1, warmup_steps)
        prog = min(1.0, (step - warmup_steps) / max(1, total_steps - warmup_steps))
        return max(min_lr / base, 0.5 * (1.0 + math.cos(math.pi * prog)))

    return torch.optim.lr_scheduler.LambdaLR(optimizer, lr_lambda)
