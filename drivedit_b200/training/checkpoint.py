"""Per-rank (sharded) training checkpoints, resume, and consolidation to the reference
checkpoint format.

The reference saves one file with the whole model and optimizer from rank 0
(``training/distributed.py:122-228``). Under this framework's sharded data parallelism
and expert parallelism that would lose state: every rank owns 1/W of the AdamW moments,
and each rank holds only its own routed experts (and their AdamW state). So every rank
writes its own file per checkpoint:

``step_<N>/rank<r>.pt``
    ``local``: this rank's rank-local parameters (expert-parallel experts) and the range
    of experts they cover; ``optim``: this rank's optimizer state (its shard of the
    sharded AdamW moments plus the full AdamW state of its local experts, or the whole
    AdamW state in a single process); ``rng``: the trainer's noise generator; rank 0 also
    writes ``replicated``: every parameter and buffer that all ranks share (weights
    gathered first when the block GEMM weights are sharded) and the config.
``step_<N>/COMPLETE``
    written by rank 0 after every rank's file is on disk (a barrier): world size, step
    and each file's SHA-256. A directory without it is an interrupted save and is
    ignored by :func:`latest_step`.

Files are written atomically (temporary file, fsync, rename) with a checksum beside
them. :func:`load_distributed` restores a trainer bit-exactly on the same world size;
:func:`consolidate` merges the rank files into one full single-process state dict (all
experts), and :func:`export_reference` writes it in the reference's key layout
(``experts.N.{w_gate,w_value,w_out}.weight``, ...).
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist

from .distributed import _atomic_save, _verified_load


def _step_dir(directory, step: int) -> Path:
    return Path(directory) / f"step_{step:08d}"


def _is_local(name: str, local_names) -> bool:
    return name in local_names


def _world_rank(trainer):
    pg = trainer.pg
    if pg is None or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(pg), dist.get_rank(pg)


def _expert_ranges(model) -> Dict[str, List[int]]:
    out = {}
    for i, blk in enumerate(getattr(model, "blocks", [])):
        moe = getattr(blk, "moe", None)
        if moe is not None and getattr(moe, "ep", None) is not None:
            out[f"blocks.{i}.moe."] = list(moe.ep.local_range())
    return out


def _cpu(obj):
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().clone()
    if isinstance(obj, dict):
        return {k: _cpu(v) for k, v in obj.items()}
    return obj


def _optimizer_state(trainer) -> Dict[str, Any]:
    if trainer.engine is None:
        return {"kind": "flat_adamw", "state": _cpu(trainer.opt.state_dict())}
    eng = trainer.engine
    st = {"kind": "sharded", "m": eng.m.detach().cpu().clone(), "v": eng.v.detach().cpu().clone(),
          "step_count": eng.step_count, "shard_off": eng.shard_off, "shard_len": eng.shard_len,
          "layout": list(eng.flat.names)}
    if eng.local_opt is not None:
        st["local"] = _cpu(eng.local_opt.state_dict())
    return st


def save_distributed(trainer, directory: str, step: int, config: Optional[Dict] = None) -> Path:
    """Every rank of the trainer's group calls this at the same step."""
    world, rank = _world_rank(trainer)
    if trainer.engine is not None:
        trainer.engine.gather_weights()
    model = trainer.model
    local_names = set(model.expert_parameter_names()) if hasattr(model, "expert_parameter_names") \
        and trainer.ep is not None else set()
    sd = model.state_dict()
    d = _step_dir(directory, step)
    d.mkdir(parents=True, exist_ok=True)
    payload = {
        "step": step, "rank": rank, "world": world,
        "local": {k: v.detach().cpu().clone() for k, v in sd.items() if _is_local(k, local_names)},
        "expert_ranges": _expert_ranges(model),
        "optim": _optimizer_state(trainer),
        "rng": trainer.gen.get_state(),
        "trainer_step": trainer.step_idx,
    }
    if rank == 0:
        payload["replicated"] = {k: v.detach().cpu().clone() for k, v in sd.items()
                                 if not _is_local(k, local_names)}
        payload["config"] = config
    _atomic_save(payload, d / f"rank{rank}.pt")
    if world > 1:
        dist.barrier(group=trainer.pg)
    if rank == 0:
        files = {f"rank{r}.pt": (d / f"rank{r}.pt.sha256").read_text().strip() for r in range(world)}
        (d / "COMPLETE").write_text(json.dumps({"step": step, "world": world, "files": files}))
    if world > 1:
        dist.barrier(group=trainer.pg)
    return d


def latest_step(directory: str, world: Optional[int] = None) -> Optional[int]:
    """Newest step whose save completed (and, if given, was written by ``world`` ranks)."""
    best = None
    for d in Path(directory).glob("step_*"):
        marker = d / "COMPLETE"
        if not marker.exists():
            continue
        try:
            meta = json.loads(marker.read_text())
        except json.JSONDecodeError:
            continue
        if world is not None and meta.get("world") != world:
            continue
        best = max(best or -1, int(meta["step"]))
    return best


def _read(d: Path, rank: int) -> Dict[str, Any]:
    meta = json.loads((d / "COMPLETE").read_text())
    path = d / f"rank{rank}.pt"
    data = path.read_bytes()
    if hashlib.sha256(data).hexdigest() != meta["files"][f"rank{rank}.pt"]:
        raise IOError(f"checkpoint file {path} does not match its recorded checksum")
    return _verified_load(path)


def load_distributed(trainer, directory: str, step: Optional[int] = None) -> Optional[int]:
    """Restore the trainer from the newest complete checkpoint (or ``step``); returns the
    step, or ``None`` when there is none. Every rank of the group calls it."""
    world, rank = _world_rank(trainer)
    step = latest_step(directory, world) if step is None else step
    if step is None:
        return None
    d = _step_dir(directory, step)
    mine = _read(d, rank)
    rep = mine if rank == 0 else _read(d, 0)
    if mine["world"] != world:
        raise IOError(f"checkpoint written by {mine['world']} ranks, loading on {world}")
    if mine["expert_ranges"] != _expert_ranges(trainer.model):
        raise IOError("the expert placement differs from the checkpoint's")
    state = dict(rep["replicated"])
    state.update(mine["local"])
    trainer.model.load_state_dict(state, strict=True)
    trainer.group.refresh_compute()
    opt = mine["optim"]
    if opt["kind"] == "flat_adamw":
        trainer.opt.load_state_dict(opt["state"])
    else:
        eng = trainer.engine
        if opt["layout"] != list(eng.flat.names) or opt["shard_len"] != eng.shard_len:
            raise IOError("the flat parameter layout differs from the checkpoint's")
        eng.m.copy_(opt["m"].to(eng.m.device))
        eng.v.copy_(opt["v"].to(eng.v.device))
        eng.step_count = int(opt["step_count"])
        if eng.local_opt is not None:
            eng.local_opt.load_state_dict(opt["local"])
    trainer.gen.set_state(mine["rng"])
    trainer.step_idx = int(mine["trainer_step"])
    if world > 1:
        dist.barrier(group=trainer.pg)
    return step


def consolidate(directory: str, step: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """One full, single-process state dict from a sharded checkpoint (CPU): every rank's
    routed experts in expert order, shared experts appended behind them (the
    unsharded layout ``[E + n_shared, ...]``)."""
    step = latest_step(directory) if step is None else step
    if step is None:
        raise FileNotFoundError(f"no complete checkpoint under {directory}")
    d = _step_dir(directory, step)
    world = json.loads((d / "COMPLETE").read_text())["world"]
    files = [_read(d, r) for r in range(world)]
    sd = dict(files[0]["replicated"])
    for prefix in files[0]["expert_ranges"]:
        for name in ("w13", "w2"):
            parts = sorted(((f["expert_ranges"][prefix][0], f["local"][prefix + name]) for f in files),
                           key=lambda t: t[0])
            routed = torch.cat([p for _, p in parts], 0)
            shared = sd.pop(prefix + name + "_shared", None)
            sd[prefix + name] = routed if shared is None else torch.cat([routed, shared], 0)
    return sd


def export_reference(directory: str, out_path: str, model_config, step: Optional[int] = None):
    """Consolidate, load into an unsharded model on the CPU and write the reference's
    checkpoint dict and key layout."""
    from ..models.world_dit import WorldDiT
    from .distributed import export_reference_checkpoint

    sd = consolidate(directory, step)
    model = WorldDiT(model_config)
    model.load_state_dict(sd, strict=True)
    return export_reference_checkpoint(model, out_path, step=step or latest_step(directory) or 0)
