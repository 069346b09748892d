"""Distributed runtime helpers, memory monitoring, checkpointing and failure detection.

API of the reference ``training/distributed.py``: ``DistributedManager`` (:21-73),
``MemoryMonitor`` (:76-119), ``CheckpointManager`` (``checkpoint_step_{N}.pt`` /
``best_checkpoint.pt`` with ``{epoch, step, model_state_dict, optimizer_state_dict, loss,
metrics, [scheduler_state_dict]}``, keep-N, latest-by-step, :122-228),
``distributed_context`` / ``setup_distributed_model`` / ``create_distributed_dataloader``
/ ``reduce_dict`` / ``get_available_port`` / ``launch_distributed`` (:232-325).

Additions for the sharded engines and for failure detection:

* process groups are created with a timeout, so a rank whose peers died ends its next
  collective with an error instead of waiting forever;
* checkpoints are written atomically (temporary file + rename) and carry a SHA-256 of
  the payload; ``load_checkpoint`` verifies it and falls back to the previous checkpoint
  when the newest one is corrupt or truncated;
* sharded optimizer state is saved per rank (``..._rank{r}.pt``) and a resume refuses a
  checkpoint whose shard set is incomplete;
* ``Heartbeat`` publishes a per-rank timestamp in the process-group store; ranks check
  their peers between steps and raise ``PeerFailure`` naming the silent rank;
* ``export_reference_checkpoint`` writes the reference's dict layout and key names
  (per-expert MoE keys) from a model in this framework's layout.
"""
from __future__ import annotations

import contextlib
import datetime
import gc
import hashlib
import io
import logging
import os
import socket
import time
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist

logger = logging.getLogger(__name__)


class PeerFailure(RuntimeError):
    """A peer rank stopped publishing heartbeats (crashed, hung or exited)."""


class DistributedManager:
    def __init__(self):
        self.is_initialized = False
        self.rank, self.world_size, self.local_rank = 0, 1, 0
        self.is_master = True

    def setup(self, rank: int, world_size: int, backend: str = "nccl", timeout_s: float = 120.0) -> None:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "12355")
        if backend == "nccl" and not torch.cuda.is_available():
            backend = "gloo"
        dist.init_process_group(backend, rank=rank, world_size=world_size,
                                timeout=datetime.timedelta(seconds=timeout_s))
        self.rank, self.world_size = rank, world_size
        self.local_rank = int(os.environ.get("LOCAL_RANK", rank % max(torch.cuda.device_count(), 1)))
        self.is_master = rank == 0
        self.is_initialized = True
        if backend == "nccl":
            torch.cuda.set_device(self.local_rank)

    def cleanup(self) -> None:
        if self.is_initialized:
            dist.destroy_process_group()
            self.is_initialized = False

    def barrier(self) -> None:
        if self.is_initialized:
            dist.barrier()

    def all_reduce(self, tensor: torch.Tensor, op=dist.ReduceOp.SUM) -> torch.Tensor:
        if self.is_initialized and self.world_size > 1:
            dist.all_reduce(tensor, op)
        return tensor

    def gather(self, tensor: torch.Tensor) -> Optional[list]:
        if not self.is_initialized or self.world_size == 1:
            return [tensor] if self.is_master else None
        out = [torch.zeros_like(tensor) for _ in range(self.world_size)] if self.is_master else None
        dist.gather(tensor, out, dst=0)
        return out


class MemoryMonitor:
    def __init__(self, max_memory_gb: float = 12.0):
        self.max_memory_gb = max_memory_gb
        self.peak_memory = self.allocated_memory = 0.0
        self.cleanup_threshold = max_memory_gb * 0.8

    def update(self) -> Dict[str, float]:
        if torch.cuda.is_available():
            self.allocated_memory = torch.cuda.memory_allocated() / 2 ** 30
            self.peak_memory = max(self.peak_memory, torch.cuda.max_memory_allocated() / 2 ** 30)
        return {"allocated_gb": self.allocated_memory, "peak_gb": self.peak_memory,
                "usage_percent": 100.0 * self.allocated_memory / self.max_memory_gb}

    def should_cleanup(self) -> bool:
        return self.allocated_memory > self.cleanup_threshold

    def cleanup(self) -> float:
        if not torch.cuda.is_available():
            return 0.0
        before = torch.cuda.memory_allocated() / 2 ** 30
        gc.collect()
        torch.cuda.empty_cache()
        self.allocated_memory = torch.cuda.memory_allocated() / 2 ** 30
        return before - self.allocated_memory

    def reset_peak(self) -> None:
        if torch.cuda.is_available():
            torch.cuda.reset_peak_memory_stats()
        self.peak_memory = 0.0


# ----------------------------------------------------------------------------- checkpoints
def _atomic_save(obj: Any, path: Path) -> str:
    """Serialise to bytes, write ``path.tmp`` + fsync, rename; returns the SHA-256."""
    buf = io.BytesIO()
    torch.save(obj, buf)
    data = buf.getvalue()
    digest = hashlib.sha256(data).hexdigest()
    tmp = path.with_suffix(path.suffix + ".tmp")
    with open(tmp, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)
    path.with_suffix(path.suffix + ".sha256").write_text(digest)
    return digest


def _verified_load(path: Path, map_location="cpu") -> Any:
    data = path.read_bytes()
    sha = path.with_suffix(path.suffix + ".sha256")
    if sha.exists() and hashlib.sha256(data).hexdigest() != sha.read_text().strip():
        raise IOError(f"checkpoint {path} is corrupt (checksum mismatch)")
    return torch.load(io.BytesIO(data), map_location=map_location, weights_only=False)


class CheckpointManager:
    def __init__(self, checkpoint_dir: str, keep_checkpoints: int = 5, rank: int = 0, world_size: int = 1):
        self.checkpoint_dir = Path(checkpoint_dir)
        self.checkpoint_dir.mkdir(parents=True, exist_ok=True)
        self.keep_checkpoints = keep_checkpoints
        self.rank, self.world_size = rank, world_size

    def _path(self, step: int, rank: Optional[int] = None) -> Path:
        return self.checkpoint_dir / (f"checkpoint_step_{step}.pt" if rank is None
                                      else f"checkpoint_step_{step}_rank{rank}.pt")

    def save_checkpoint(self, model, optimizer, scheduler, epoch: int, step: int, loss: float,
                        metrics: Optional[Dict[str, float]] = None, is_best: bool = False,
                        optimizer_shard: Optional[Dict[str, Any]] = None, config: Optional[Dict] = None) -> str:
        """Rank 0 writes the model (replicated weights) and the optimizer state; with
        ``optimizer_shard`` every rank also writes its own shard file."""
        if optimizer_shard is not None:
            _atomic_save({"step": step, "rank": self.rank, "world_size": self.world_size,
                          "optimizer_shard": optimizer_shard}, self._path(step, self.rank))
        path = self._path(step)
        if self.rank == 0:
            ck = {"epoch": epoch, "step": step, "model_state_dict": model.state_dict(),
                  "optimizer_state_dict": optimizer.state_dict() if optimizer is not None else None,
                  "loss": float(loss), "metrics": metrics or {}, "world_size": self.world_size,
                  "sharded_optimizer": optimizer_shard is not None, "config": config}
            if scheduler is not None:
                ck["scheduler_state_dict"] = scheduler.state_dict()
            _atomic_save(ck, path)
            if is_best:
                _atomic_save(ck, self.checkpoint_dir / "best_checkpoint.pt")
            self._cleanup_old_checkpoints()
        return str(path)

    def _steps(self) -> List[int]:
        out = []
        for p in self.checkpoint_dir.glob("checkpoint_step_*.pt"):
            stem = p.stem[len("checkpoint_step_"):]
            if stem.isdigit():
                out.append(int(stem))
        return sorted(out)

    def _get_latest_checkpoint(self) -> Optional[str]:
        s = self._steps()
        return str(self._path(s[-1])) if s else None

    def _cleanup_old_checkpoints(self) -> None:
        for s in self._steps()[:-self.keep_checkpoints] if self.keep_checkpoints > 0 else []:
            for p in self.checkpoint_dir.glob(f"checkpoint_step_{s}*"):
                p.unlink(missing_ok=True)

    def load_checkpoint(self, model, optimizer=None, scheduler=None, checkpoint_path: Optional[str] = None,
                        load_best: bool = False, strict: bool = True) -> Dict[str, Any]:
        """Newest valid checkpoint (checksum verified, shard set complete); corrupt or
        incomplete ones are skipped with a warning. Returns ``{}`` when none is usable."""
        if checkpoint_path is not None or load_best:
            cands = [Path(checkpoint_path) if checkpoint_path else self.checkpoint_dir / "best_checkpoint.pt"]
        else:
            cands = [self._path(s) for s in reversed(self._steps())]
        for path in cands:
            if not path.exists():
                continue
            try:
                ck = _verified_load(path)
                shard = None
                if ck.get("sharded_optimizer"):
                    sp = self._path(ck["step"], self.rank)
                    if not sp.exists() or ck.get("world_size") != self.world_size:
                        raise IOError(f"optimizer shard {sp.name} missing or world size changed")
                    shard = _verified_load(sp)["optimizer_shard"]
            except Exception as e:  # noqa: BLE001 - try the next older checkpoint
                logger.warning("skipping checkpoint %s: %s", path, e)
                continue
            model.load_state_dict(ck["model_state_dict"], strict=strict)
            if optimizer is not None and ck.get("optimizer_state_dict") is not None:
                optimizer.load_state_dict(ck["optimizer_state_dict"])
            if scheduler is not None and "scheduler_state_dict" in ck:
                scheduler.load_state_dict(ck["scheduler_state_dict"])
            return {"epoch": ck["epoch"], "step": ck["step"], "loss": ck["loss"], "metrics": ck.get("metrics", {}),
                    "optimizer_shard": shard, "path": str(path), "config": ck.get("config")}
        return {}


def export_reference_checkpoint(model, path: str, epoch: int = 0, step: int = 0, loss: float = 0.0,
                                optimizer_state: Optional[Dict] = None) -> Dict[str, torch.Tensor]:
    """Model state in the reference's checkpoint dict and key layout: MoE FFNs expand
    to ``router.gate.weight`` / ``experts.N.{w_gate,w_value,w_out}.weight`` /
    ``shared_experts.N.*`` / ``shared_gate.weight``; everything else keeps its name."""
    from ..layers.moe import MoEFFN

    sd = dict(model.state_dict())
    for name, mod in model.named_modules():
        if isinstance(mod, MoEFFN):
            pre = name + "." if name else ""
            for k in list(sd):
                if k.startswith(pre) and k[len(pre):] in ("router_weight", "expert_bias", "expert_load_ema",
                                                           "w13", "w2"):
                    del sd[k]
            sd.update(mod.reference_state_dict(pre))
    torch.save({"epoch": epoch, "step": step, "model_state_dict": sd, "optimizer_state_dict": optimizer_state or {},
                "loss": float(loss), "metrics": {}}, path)
    return sd


# ----------------------------------------------------------------------------- failure detection
class Heartbeat:
    """Per-rank liveness through the process group's key-value store: ``beat()`` after
    every step writes this rank's wall time; ``check()`` raises ``PeerFailure`` when a
    peer's last beat is older than ``timeout_s`` (or never came)."""

    def __init__(self, store, rank: int, world_size: int, timeout_s: float = 30.0, prefix: str = "hb"):
        self.store, self.rank, self.world_size = store, rank, world_size
        self.timeout_s, self.prefix = timeout_s, prefix
        self.started = time.time()

    def beat(self, step: int = 0) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", f"{time.time():.6f}:{step}")

    def check(self) -> Dict[int, float]:
        now, ages = time.time(), {}
        for r in range(self.world_size):
            if r == self.rank:
                continue
            key = f"{self.prefix}/{r}"
            try:
                self.store.wait([key], datetime.timedelta(seconds=0.05))
                ts = float(self.store.get(key).decode().split(":")[0])
            except Exception:  # noqa: BLE001 - key absent: never beat
                ts = self.started
            ages[r] = now - ts
            if ages[r] > self.timeout_s:
                raise PeerFailure(f"rank {r} silent for {ages[r]:.1f}s (timeout {self.timeout_s}s)")
        return ages


def check_finite(*tensors: torch.Tensor, names: Optional[List[str]] = None) -> None:
    """NaN / Inf sentinel (one host sync for all tensors)."""
    flags = torch.stack([torch.isfinite(t.detach()).all() for t in tensors])
    if not bool(flags.all()):
        bad = [(names[i] if names else str(i)) for i, ok in enumerate(flags.tolist()) if not ok]
        raise FloatingPointError(f"non-finite values in {bad}")


# ----------------------------------------------------------------------------- launch helpers
@contextlib.contextmanager
def distributed_context(rank: int, world_size: int, backend: str = "nccl", timeout_s: float = 120.0):
    m = DistributedManager()
    m.setup(rank, world_size, backend, timeout_s)
    try:
        yield m
    finally:
        m.cleanup()


def setup_distributed_model(model: torch.nn.Module, local_rank: int, find_unused_parameters: bool = False):
    """DDP wrapper (the baseline data-parallel path; the framework's own engines are
    :class:`~drivedit_b200.parallel.sharded.ShardedDataParallel` and the MoE EP path)."""
    from torch.nn.parallel import DistributedDataParallel as DDP

    if torch.cuda.is_available():
        model = model.cuda(local_rank)
        return DDP(model, device_ids=[local_rank], find_unused_parameters=find_unused_parameters)
    return DDP(model, find_unused_parameters=find_unused_parameters)


def create_distributed_dataloader(dataset, batch_size: int, shuffle: bool = True, num_workers: int = 4,
                                  pin_memory: bool = True, drop_last: bool = True,
                                  rank: Optional[int] = None, world_size: Optional[int] = None, **kw):
    """A loader over this rank's share of ``dataset`` (the reference's arguments,
    training/distributed.py:256-274); without a process group (or with one rank) it
    shuffles the whole dataset itself. Pinned memory only when CUDA is present."""
    from torch.utils.data import DataLoader, DistributedSampler

    if world_size is None:
        world_size = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
    sampler = DistributedSampler(dataset, world_size, rank, shuffle=shuffle) if world_size > 1 else None
    return DataLoader(dataset, batch_size=batch_size, shuffle=shuffle and sampler is None, sampler=sampler,
                      num_workers=num_workers, pin_memory=pin_memory and torch.cuda.is_available(),
                      drop_last=drop_last, **kw)


def reduce_dict(input_dict: Dict[str, torch.Tensor], world_size: int, average: bool = True) -> Dict[str, float]:
    """One all-reduce for all values (stacked), then one host transfer."""
    if not input_dict:
        return {}
    keys = sorted(input_dict)
    vals = torch.stack([torch.as_tensor(input_dict[k], dtype=torch.float32).reshape(()) for k in keys])
    if world_size > 1 and dist.is_initialized():
        if dist.get_backend() == "nccl":
            vals = vals.cuda()
        dist.all_reduce(vals)
        if average:
            vals = vals / world_size
    return dict(zip(keys, vals.cpu().tolist()))


def get_available_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch_distributed(train_func, world_size: int, backend: str = "nccl", master_addr: str = "127.0.0.1",
                       master_port: Optional[str] = None, *args) -> None:
    """Spawns ``world_size`` processes running ``train_func(rank, world_size, *args)``
    inside a ``distributed_context`` (rendezvous at ``master_addr``, a free port unless
    ``master_port`` is given)."""
    import torch.multiprocessing as mp

    fn = train_func
    os.environ["MASTER_ADDR"] = master_addr
    os.environ["MASTER_PORT"] = str(master_port or get_available_port())
    mp.spawn(_launch_entry, args=(world_size, backend, fn, args), nprocs=world_size, join=True)


def _launch_entry(rank, world_size, backend, fn, args):
    with distributed_context(rank, world_size, backend):
        fn(rank, world_size, *args)
