"""Large-scale video ingestion (the reference's ``data/large_scale_processing.py``:
``StorageTier``, ``DatasetMetadata``, ``ProcessingConfig``, ``HierarchicalStorageManager``,
``DatasetDatabase`` (sqlite), ``LargeScaleProcessor``, ``create_large_scale_config``,
``main``).

A directory of videos becomes quality-filtered, deduplicated, overlapping chunks cached as
uint8 memmaps (:class:`~drivedit_b200.data.pipeline.VideoMemoryMap`), tracked in a sqlite
database and placed on the fastest storage tier with room. Quality = mean of a sharpness
score (variance of the Laplacian, saturating) and a motion score (mean absolute frame
difference) over sampled frames; videos below ``min_quality_score`` are skipped. Videos are
processed by a process pool, ``max_concurrent_videos`` at a time.
"""
from __future__ import annotations

import hashlib
import json
import logging
import multiprocessing as mp
import shutil
import sqlite3
import time
from concurrent.futures import ProcessPoolExecutor, as_completed
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np

logger = logging.getLogger(__name__)
VIDEO_EXT = (".mp4", ".avi", ".mov", ".mkv", ".webm")


@dataclass
class StorageTier:
    name: str
    path: str
    capacity_gb: float
    access_speed: str          # "fast" | "medium" | "slow"
    cost_per_gb: float
    retention_days: int


@dataclass
class DatasetMetadata:
    dataset_id: str
    source: str
    total_hours: float
    total_size_gb: float
    fps: float
    resolution: Tuple[int, int]
    num_sequences: int
    quality_score: float
    processing_date: str
    storage_tier: str


@dataclass
class ProcessingConfig:
    num_workers: int = max(1, mp.cpu_count() // 2)
    max_concurrent_videos: int = 100
    chunk_size_gb: float = 10.0
    storage_tiers: Optional[List[StorageTier]] = None
    min_quality_score: float = 0.7
    max_blur_ratio: float = 0.3
    min_motion_score: float = 0.01
    organize_by_quality: bool = True
    organize_by_scenario: bool = True
    organize_by_time_of_day: bool = True
    enable_deduplication: bool = True
    enable_compression: bool = True
    compression_quality: int = 85
    use_database: bool = True
    database_path: str = "./dataset_metadata.db"
    chunk_seconds: float = 300.0
    overlap_seconds: float = 30.0
    output_root: str = "./processed"


class HierarchicalStorageManager:
    """Places files on the fastest tier with capacity; promotes hot files."""

    def __init__(self, config: ProcessingConfig):
        self.config = config
        self.tiers = config.storage_tiers or self._create_default_tiers()
        self.usage_gb: Dict[str, float] = {t.name: 0.0 for t in self.tiers}
        self.access_tracker: Dict[str, int] = {}
        self.placement: Dict[str, str] = {}

    def _create_default_tiers(self) -> List[StorageTier]:
        root = Path(self.config.output_root)
        return [StorageTier("hot", str(root / "hot"), 2000.0, "fast", 0.10, 30),
                StorageTier("warm", str(root / "warm"), 10000.0, "medium", 0.05, 90),
                StorageTier("cold", str(root / "cold"), 100000.0, "slow", 0.01, 365)]

    def _check_tier_capacity(self, tier: StorageTier, required_gb: float) -> bool:
        return self.usage_gb[tier.name] + required_gb <= tier.capacity_gb

    def allocate_storage(self, file_size_gb: float, priority: str = "medium") -> StorageTier:
        order = {"high": ["fast", "medium", "slow"], "medium": ["medium", "fast", "slow"],
                 "low": ["slow", "medium", "fast"]}.get(priority, ["medium", "fast", "slow"])
        for speed in order:
            for t in self.tiers:
                if t.access_speed == speed and self._check_tier_capacity(t, file_size_gb):
                    self.usage_gb[t.name] += file_size_gb
                    Path(t.path).mkdir(parents=True, exist_ok=True)
                    return t
        raise RuntimeError(f"no storage tier has {file_size_gb:.2f} GB free")

    def promote_file(self, file_path: str, target_tier: str) -> str:
        tier = next(t for t in self.tiers if t.name == target_tier)
        Path(tier.path).mkdir(parents=True, exist_ok=True)
        dst = Path(tier.path) / Path(file_path).name
        if Path(file_path).resolve() != dst.resolve():
            shutil.move(str(file_path), dst)
        self.placement[str(dst)] = target_tier
        return str(dst)

    def _update_access_tracker(self, file_path: str):
        self.access_tracker[file_path] = self.access_tracker.get(file_path, 0) + 1


class DatasetDatabase:
    def __init__(self, db_path: str):
        self.db_path = db_path
        self._init_database()

    def _init_database(self):
        with sqlite3.connect(self.db_path) as c:
            c.execute("""CREATE TABLE IF NOT EXISTS datasets (id TEXT PRIMARY KEY, source TEXT, total_hours REAL,
                         total_size_gb REAL, fps REAL, resolution TEXT, num_sequences INTEGER, quality_score REAL,
                         processing_date TEXT, storage_tier TEXT, metadata TEXT)""")
            c.execute("""CREATE TABLE IF NOT EXISTS video_files (id TEXT PRIMARY KEY, dataset_id TEXT,
                         file_path TEXT, file_size_gb REAL, duration_seconds REAL, quality_score REAL,
                         processing_status TEXT, chunk_ids TEXT, created_at TIMESTAMP DEFAULT CURRENT_TIMESTAMP,
                         FOREIGN KEY (dataset_id) REFERENCES datasets (id))""")
            c.execute("""CREATE TABLE IF NOT EXISTS processing_jobs (id TEXT PRIMARY KEY, job_type TEXT, status TEXT,
                         input_files TEXT, output_files TEXT, started_at TIMESTAMP, completed_at TIMESTAMP,
                         error_message TEXT)""")
            for stmt in ("CREATE INDEX IF NOT EXISTS idx_dataset_source ON datasets(source)",
                         "CREATE INDEX IF NOT EXISTS idx_video_dataset ON video_files(dataset_id)",
                         "CREATE INDEX IF NOT EXISTS idx_video_status ON video_files(processing_status)",
                         "CREATE INDEX IF NOT EXISTS idx_job_status ON processing_jobs(status)"):
                c.execute(stmt)

    def insert_dataset(self, m: DatasetMetadata):
        with sqlite3.connect(self.db_path) as c:
            c.execute("INSERT OR REPLACE INTO datasets VALUES (?,?,?,?,?,?,?,?,?,?,?)",
                      (m.dataset_id, m.source, m.total_hours, m.total_size_gb, m.fps, json.dumps(list(m.resolution)),
                       m.num_sequences, m.quality_score, m.processing_date, m.storage_tier, json.dumps(asdict(m))))

    def insert_video_file(self, video_id: str, dataset_id: str, file_path: str, file_size_gb: float,
                          duration_seconds: float, quality_score: float):
        with sqlite3.connect(self.db_path) as c:
            c.execute("""INSERT OR REPLACE INTO video_files (id, dataset_id, file_path, file_size_gb, duration_seconds,
                         quality_score, processing_status, chunk_ids) VALUES (?,?,?,?,?,?,?,?)""",
                      (video_id, dataset_id, file_path, file_size_gb, duration_seconds, quality_score, "pending", "[]"))

    def update_processing_status(self, video_id: str, status: str, chunk_ids: Optional[List[str]] = None):
        with sqlite3.connect(self.db_path) as c:
            c.execute("UPDATE video_files SET processing_status = ?, chunk_ids = ? WHERE id = ?",
                      (status, json.dumps(chunk_ids or []), video_id))

    def get_pending_videos(self, limit: int = 100) -> List[Tuple]:
        with sqlite3.connect(self.db_path) as c:
            return c.execute("SELECT id, file_path FROM video_files WHERE processing_status = 'pending' LIMIT ?",
                             (limit,)).fetchall()

    def get_dataset_stats(self) -> Dict:
        with sqlite3.connect(self.db_path) as c:
            n_ds, hours, size = c.execute("SELECT COUNT(*), COALESCE(SUM(total_hours),0), "
                                          "COALESCE(SUM(total_size_gb),0) FROM datasets").fetchone()
            by_status = dict(c.execute("SELECT processing_status, COUNT(*) FROM video_files "
                                       "GROUP BY processing_status").fetchall())
            by_source = dict(c.execute("SELECT source, COUNT(*) FROM datasets GROUP BY source").fetchall())
        return {"num_datasets": n_ds, "total_hours": hours, "total_size_gb": size, "videos_by_status": by_status,
                "datasets_by_source": by_source}


# ----------------------------------------------------------------------------- per video (worker side)
def _sample_frames(path: str, n: int = 10):
    import cv2

    cap = cv2.VideoCapture(path)
    count = int(cap.get(cv2.CAP_PROP_FRAME_COUNT))
    fps = cap.get(cv2.CAP_PROP_FPS) or 30.0
    frames = []
    for i in np.linspace(0, max(count - 1, 0), min(n, max(count, 1))).astype(int):
        cap.set(cv2.CAP_PROP_POS_FRAMES, int(i))
        ok, f = cap.read()
        if ok:
            frames.append(f)
    cap.release()
    return frames, count, fps


def assess_quality(frames: List[np.ndarray]) -> float:
    """0.5 * sharpness (Laplacian variance / 100, capped at 1) + 0.5 * motion (mean
    absolute difference of consecutive samples / 10, capped at 1)."""
    import cv2

    if not frames:
        return 0.0
    grey = [cv2.cvtColor(f, cv2.COLOR_BGR2GRAY).astype(np.float32) for f in frames]
    sharp = np.mean([min(1.0, cv2.Laplacian(g, cv2.CV_32F).var() / 100.0) for g in grey])
    motion = np.mean([min(1.0, np.abs(a - b).mean() / 10.0) for a, b in zip(grey[1:], grey[:-1])]) if len(grey) > 1 else 0.0
    return float(0.5 * sharp + 0.5 * motion)


def process_video(video_path: str, out_dir: str, cfg: Dict) -> Dict:
    """Quality gate, overlapping chunks cached as memmaps; returns a result record."""
    import cv2

    from .pipeline import VideoMemoryMap

    try:
        frames, count, fps = _sample_frames(video_path)
        q = assess_quality(frames)
        vid = hashlib.sha1(str(Path(video_path).resolve()).encode()).hexdigest()[:16]
        if q < cfg["min_quality_score"]:
            return {"success": False, "video_id": vid, "quality_score": q,
                    "error": f"quality {q:.3f} below {cfg['min_quality_score']}"}
        step = max(1, int(round((cfg["chunk_seconds"] - cfg["overlap_seconds"]) * fps)))
        length = max(1, int(round(cfg["chunk_seconds"] * fps)))
        cap = cv2.VideoCapture(video_path)
        allf = []
        while True:
            ok, f = cap.read()
            if not ok:
                break
            allf.append(f[:, :, ::-1])
        cap.release()
        chunks = []
        vdir = Path(out_dir) / vid
        vdir.mkdir(parents=True, exist_ok=True)
        for k, s in enumerate(range(0, max(len(allf) - 1, 1), step)):
            seg = np.stack(allf[s:s + length]) if allf[s:s + length] else None
            if seg is None:
                break
            name = f"{vid}_chunk{k:04d}"
            VideoMemoryMap(str(vdir / f"{name}.mp4"), str(vdir), frames=seg)
            h = hashlib.sha1(np.ascontiguousarray(seg[:: max(1, len(seg) // 8)]).tobytes()).hexdigest()
            chunks.append({"name": name, "path": str(vdir / f"{name}.u8"), "frames": len(seg),
                           "duration": len(seg) / fps, "hash": h})
            if s + length >= len(allf):
                break
        return {"success": True, "video_id": vid, "quality_score": q, "chunks": chunks, "fps": fps,
                "resolution": tuple(allf[0].shape[:2]) if allf else (0, 0),
                "size_gb": Path(video_path).stat().st_size / 1024 ** 3}
    except Exception as e:  # noqa: BLE001 - one record per video
        return {"success": False, "error": str(e), "video_id": None}


class LargeScaleProcessor:
    def __init__(self, config: ProcessingConfig):
        self.config = config
        self.storage = HierarchicalStorageManager(config)
        self.database = DatasetDatabase(config.database_path) if config.use_database else None
        self.stats = {"processed": 0, "failed": 0, "skipped_quality": 0, "chunks": 0, "duplicates": 0}

    def _discover_video_files(self, input_path: Path) -> List[Path]:
        return sorted(p for p in Path(input_path).rglob("*") if p.suffix.lower() in VIDEO_EXT)

    def _estimate_total_hours(self, videos: List[Path]) -> float:
        import cv2

        total = 0.0
        for v in videos:
            cap = cv2.VideoCapture(str(v))
            n, fps = cap.get(cv2.CAP_PROP_FRAME_COUNT), cap.get(cv2.CAP_PROP_FPS) or 30.0
            cap.release()
            total += n / fps / 3600.0
        return total

    def _create_processing_batches(self, videos: List[Path]) -> List[List[Path]]:
        """Batches of at most ``max_concurrent_videos`` and ``chunk_size_gb`` on disk."""
        out, cur, size = [], [], 0.0
        for v in videos:
            s = v.stat().st_size / 1024 ** 3
            if cur and (len(cur) >= self.config.max_concurrent_videos or size + s > self.config.chunk_size_gb):
                out.append(cur)
                cur, size = [], 0.0
            cur.append(v)
            size += s
        if cur:
            out.append(cur)
        return out

    def _deduplicate_chunks(self, chunks: List[Dict], seen: set) -> List[Dict]:
        out = []
        for c in chunks:
            if c["hash"] in seen:
                self.stats["duplicates"] += 1
                Path(c["path"]).unlink(missing_ok=True)
                continue
            seen.add(c["hash"])
            out.append(c)
        return out

    @staticmethod
    def _generate_dataset_id(source: str, name: str) -> str:
        return f"{source}_{hashlib.sha1(f'{source}:{name}:{time.time()}'.encode()).hexdigest()[:12]}"

    def process_dataset_directory(self, input_dir: str, dataset_source: str = "custom") -> str:
        videos = self._discover_video_files(Path(input_dir))
        ds_id = self._generate_dataset_id(dataset_source, Path(input_dir).name)
        hours = self._estimate_total_hours(videos) if videos else 0.0
        size_gb = sum(v.stat().st_size for v in videos) / 1024 ** 3
        tier = self.storage.allocate_storage(max(size_gb, 1e-6), "high" if hours < 100 else "medium")
        out_dir = Path(tier.path) / ds_id
        out_dir.mkdir(parents=True, exist_ok=True)
        cfg = {"min_quality_score": self.config.min_quality_score, "chunk_seconds": self.config.chunk_seconds,
               "overlap_seconds": self.config.overlap_seconds}
        seen: set = set()
        qualities, n_seq, fps, res = [], 0, 0.0, (0, 0)
        for batch in self._create_processing_batches(videos):
            with ProcessPoolExecutor(max_workers=min(self.config.num_workers, len(batch)),
                                     mp_context=mp.get_context("spawn")) as ex:
                futs = {ex.submit(process_video, str(v), str(out_dir), cfg): v for v in batch}
                for f in as_completed(futs):
                    r = f.result()
                    v = futs[f]
                    if not r["success"]:
                        self.stats["skipped_quality" if "quality" in r.get("error", "") else "failed"] += 1
                        continue
                    chunks = self._deduplicate_chunks(r["chunks"], seen) if self.config.enable_deduplication \
                        else r["chunks"]
                    self.stats["processed"] += 1
                    self.stats["chunks"] += len(chunks)
                    qualities.append(r["quality_score"])
                    n_seq += len(chunks)
                    fps, res = r["fps"], r["resolution"]
                    if self.database:
                        self.database.insert_video_file(r["video_id"], ds_id, str(v), r["size_gb"],
                                                        sum(c["duration"] for c in chunks), r["quality_score"])
                        self.database.update_processing_status(r["video_id"], "completed", [c["name"] for c in chunks])
        meta = DatasetMetadata(ds_id, dataset_source, hours, size_gb, fps, res, n_seq,
                               float(np.mean(qualities)) if qualities else 0.0,
                               time.strftime("%Y-%m-%d %H:%M:%S"), tier.name)
        if self.database:
            self.database.insert_dataset(meta)
        (out_dir / "dataset_metadata.json").write_text(json.dumps(asdict(meta), indent=2))
        return ds_id

    def get_processing_status(self) -> Dict:
        out = dict(self.stats)
        if self.database:
            out["database"] = self.database.get_dataset_stats()
        out["storage_usage_gb"] = dict(self.storage.usage_gb)
        return out


def create_large_scale_config(**kw) -> ProcessingConfig:
    return ProcessingConfig(**kw)


def main(argv=None):
    import argparse

    ap = argparse.ArgumentParser(description="ingest a directory of driving videos")
    ap.add_argument("input_dir")
    ap.add_argument("--source", default="custom")
    ap.add_argument("--output-root", default="./processed")
    ap.add_argument("--db", default="./dataset_metadata.db")
    ap.add_argument("--workers", type=int, default=max(1, mp.cpu_count() // 2))
    ap.add_argument("--min-quality", type=float, default=0.7)
    a = ap.parse_args(argv)
    p = LargeScaleProcessor(ProcessingConfig(num_workers=a.workers, output_root=a.output_root, database_path=a.db,
                                             min_quality_score=a.min_quality))
    ds = p.process_dataset_directory(a.input_dir, a.source)
    print(json.dumps({"dataset_id": ds, **p.get_processing_status()}, indent=2, default=str))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
