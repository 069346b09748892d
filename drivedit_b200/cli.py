"""Command-line entry points (the reference's ``scripts/``: ``train.py``, ``process_data.py``,
``profile_codebase.py``).

``python -m drivedit_b200.cli train --config dit_b --steps 100 [key=value ...]``
    trains a world-model preset on synthetic latents, one process per GPU under
    ``torchrun`` (NCCL; sharded optimizer and, for MoE presets, expert parallelism),
    logging JSONL metrics and writing atomic checkpoints every ``--ckpt-every`` steps;
    ``--resume`` continues from the newest valid checkpoint.
``python -m drivedit_b200.cli process-data INPUT_DIR [--cache-dir D]``
    builds uint8 memmap caches of every video under INPUT_DIR in parallel.
``python -m drivedit_b200.cli ingest INPUT_DIR``
    large-scale ingestion (quality gate, chunks, dedup, sqlite), see
    :mod:`drivedit_b200.data.large_scale`.
``python -m drivedit_b200.cli profile step|deadcode ...``
    see :mod:`drivedit_b200.profiling`.

The reference's ``scripts/train.py`` trains a three-convolution placeholder network
(``:86-92``); this one trains the real models.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from concurrent.futures import ProcessPoolExecutor
from pathlib import Path


def _train(a) -> int:
    import torch
    import torch.distributed as dist

    from .config import get_config
    from .data.synthetic import make_batch
    from .models.world_dit import WorldDiT
    from .config import to_dict
    from .training.checkpoint import load_distributed, save_distributed
    from .training.trainer import WorldModelTrainer
    from .utils.observability import MetricsLogger

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cuda = torch.cuda.is_available()
    if ws > 1:
        import datetime

        if cuda:
            torch.cuda.set_device(local)
        dist.init_process_group("nccl" if cuda else "gloo", timeout=datetime.timedelta(seconds=a.pg_timeout))
    dev = torch.device("cuda", local) if cuda else torch.device("cpu")
    cfg = get_config(a.config, a.override)
    if not cuda:
        cfg.train.dtype = "fp32"
    torch.manual_seed(cfg.train.seed)
    model = WorldDiT(cfg.model)
    tr = WorldModelTrainer(model, cfg.train, dev, process_group=dist.group.WORLD if ws > 1 else None)
    ckdir = str(Path(a.out) / "checkpoints")
    start = 0
    if a.resume:  # per-rank files: sharded optimizer state, each rank's experts, RNG
        start = load_distributed(tr, ckdir) or 0
    log = MetricsLogger(a.out, rank, ws, config={"preset": a.config, "overrides": a.override})
    rgb = cfg.train.frames if cfg.model.repa is not None else 0
    tokens = cfg.train.batch_per_gpu * cfg.train.frames * cfg.model.tokens_per_frame
    t0 = time.perf_counter()
    for step in range(start, a.steps):
        # the synthetic stream is a function of (step, rank), so a resumed run sees the
        # same batches as an uninterrupted one
        gen = torch.Generator().manual_seed(1000 + 7919 * step + rank)
        batch = make_batch(cfg, generator=gen, pin=cuda, rgb_frames=rgb).to(dev, non_blocking=True)
        loss = tr.train_step(batch)
        if (step + 1) % a.log_every == 0:
            if cuda:
                torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            t0 = time.perf_counter()
            log.log(step + 1, {"loss": float(loss), "tok_per_s": ws * tokens * a.log_every / dt,
                               **{k: float(v) for k, v in tr.last_losses.items()}})
        if a.ckpt_every and (step + 1) % a.ckpt_every == 0:
            save_distributed(tr, ckdir, step + 1, config=to_dict(cfg))
    if ws > 1:
        dist.barrier()
        if tr.engine is not None:
            tr.engine.close()
        if tr.ep is not None:
            tr.ep.close()
        dist.destroy_process_group()
    return 0


def _cache_one(args):
    from .data.pipeline import VideoMemoryMap

    path, cache = args
    try:
        m = VideoMemoryMap(path, cache)
        return path, m.frame_count, None
    except Exception as e:  # noqa: BLE001 - reported per video
        return path, 0, str(e)


def _process_data(a) -> int:
    vids = sorted(str(p) for p in Path(a.input_dir).rglob("*")
                  if p.suffix.lower() in (".mp4", ".avi", ".mov", ".mkv", ".webm"))
    cache = a.cache_dir or str(Path(a.input_dir) / "cache")
    with ProcessPoolExecutor(a.workers) as ex:
        res = list(ex.map(_cache_one, [(v, cache) for v in vids]))
    print(json.dumps({"videos": len(vids), "frames": sum(r[1] for r in res),
                      "errors": {r[0]: r[2] for r in res if r[2]}}, indent=2))
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="drivedit_b200", description=__doc__.split("\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    t = sub.add_parser("train")
    t.add_argument("--config", default="tiny")
    t.add_argument("--steps", type=int, default=100)
    t.add_argument("--out", default="./runs/train")
    t.add_argument("--log-every", type=int, default=10)
    t.add_argument("--ckpt-every", type=int, default=0)
    t.add_argument("--resume", action="store_true")
    t.add_argument("--pg-timeout", type=float, default=300.0)
    t.add_argument("override", nargs="*")
    p = sub.add_parser("process-data")
    p.add_argument("input_dir")
    p.add_argument("--cache-dir", default=None)
    p.add_argument("--workers", type=int, default=4)
    g = sub.add_parser("ingest")
    g.add_argument("rest", nargs=argparse.REMAINDER)
    f = sub.add_parser("profile")
    f.add_argument("rest", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    if a.cmd == "train":
        return _train(a)
    if a.cmd == "process-data":
        return _process_data(a)
    if a.cmd == "ingest":
        from .data.large_scale import main as ingest_main

        return ingest_main(a.rest)
    from .profiling import main as prof_main

    return prof_main(a.rest)


if __name__ == "__main__":
    sys.exit(main())
