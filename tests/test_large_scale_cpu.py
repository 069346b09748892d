"""Video ingestion: quality gate, overlapping memmap chunks, dedup, sqlite tracking (CPU)."""
import numpy as np
import pytest

cv2 = pytest.importorskip("cv2")

from drivedit_b200.data.large_scale import (DatasetDatabase, HierarchicalStorageManager, LargeScaleProcessor,
                                            ProcessingConfig)


def _video(path, n=40, fps=10.0, static=False, seed=0):
    rng = np.random.default_rng(seed)
    w = cv2.VideoWriter(str(path), cv2.VideoWriter_fourcc(*"MJPG"), fps, (64, 48))
    base = rng.integers(0, 255, (48, 64, 3), dtype=np.uint8)
    for i in range(n):
        f = base if static else np.roll(base, 3 * i, axis=1)
        w.write(f)
    w.release()


def test_ingest_directory(tmp_path):
    src = tmp_path / "videos"
    src.mkdir()
    _video(src / "a.avi", seed=0)
    _video(src / "b.avi", static=True, seed=1)           # no motion -> low quality
    _video(src / "c.avi", seed=0)                        # duplicate content of a
    cfg = ProcessingConfig(num_workers=2, output_root=str(tmp_path / "out"), database_path=str(tmp_path / "m.db"),
                           min_quality_score=0.6, chunk_seconds=2.0, overlap_seconds=0.5)
    p = LargeScaleProcessor(cfg)
    ds = p.process_dataset_directory(str(src), "custom")
    st = p.get_processing_status()
    assert st["processed"] == 2 and st["skipped_quality"] == 1
    assert st["duplicates"] >= 1 and st["chunks"] >= 2
    db = st["database"]
    assert db["num_datasets"] == 1 and db["videos_by_status"]["completed"] == 2
    chunks = list((tmp_path / "out").rglob("*.u8"))
    assert len(chunks) == st["chunks"]
    assert ds.startswith("custom_")


def test_storage_tiers_and_db(tmp_path):
    cfg = ProcessingConfig(output_root=str(tmp_path))
    sm = HierarchicalStorageManager(cfg)
    assert sm.allocate_storage(1.0, "high").access_speed == "fast"
    assert sm.allocate_storage(5000.0, "high").access_speed == "medium"   # hot tier full
    f = tmp_path / "x.bin"
    f.write_bytes(b"1")
    assert sm.promote_file(str(f), "cold").endswith("cold/x.bin")
    db = DatasetDatabase(str(tmp_path / "d.db"))
    db.insert_video_file("v1", "d", "/x", 0.1, 2.0, 0.9)
    assert db.get_pending_videos() == [("v1", "/x")]
    db.update_processing_status("v1", "completed", ["c0"])
    assert db.get_pending_videos() == []
