"""Scene-aware video chunking (reference ``data/video_chunking.py``) on synthetic clips."""
import json

import numpy as np
import pytest

from drivedit_b200.data.video_chunking import (ChunkConfig, ChunkedVideoDataset, QualityFilter,
                                               SceneDetector, VideoChunker, histogram_correlation,
                                               hsv_histograms, laplacian_variance, rgb_to_hsv)


def _clip(n=300, h=48, w=64, seed=0):
    """Two scenes (reddish then bluish), textured, with a moving stripe pattern."""
    rng = np.random.default_rng(seed)
    base = rng.integers(0, 60, size=(h, w, 3))
    frames = np.empty((n, h, w, 3), np.uint8)
    xs = np.arange(w)
    for i in range(n):
        tint = np.array([180, 60, 40]) if i < n // 2 else np.array([30, 70, 190])
        stripe = (((xs + 3 * i) // 4) % 2 * 60)[None, :, None]
        frames[i] = np.clip(base + tint + stripe, 0, 255)
    return frames


def test_hsv_matches_opencv():
    cv2 = pytest.importorskip("cv2")
    f = np.random.default_rng(1).integers(0, 256, size=(1, 16, 16, 3), dtype=np.uint8)
    ours = rgb_to_hsv(f)[0]
    ref = cv2.cvtColor(f[0], cv2.COLOR_RGB2HSV).astype(np.float32)
    assert np.abs(ours[..., 1:] - ref[..., 1:]).max() <= 1.0
    dh = np.abs(ours[..., 0] - ref[..., 0])
    assert np.minimum(dh, 180 - dh).max() <= 1.0


def test_scene_cut_and_quality(tmp_path):
    frames = _clip()
    chunker = VideoChunker(ChunkConfig(chunk_duration=4, overlap_duration=1, min_chunk_duration=2,
                                       target_fps=10, scene_threshold=0.3,
                                       blur_threshold=50.0, min_quality=0.3))
    from drivedit_b200.data.pipeline import VideoMemoryMap

    v = VideoMemoryMap(str(tmp_path / "drive.mp4"), str(tmp_path / "c"), frames=frames)
    cuts = SceneDetector(0.3).cut_frames(v)
    assert cuts == [150]
    q = QualityFilter(blur_threshold=50.0)
    assert q.assess_quality(frames[:10]) > 0.5
    still = np.repeat(frames[:1], 5, 0)
    assert q._assess_motion(still) == 0.0
    blurry = np.full((3, 32, 32, 3), 128, np.uint8)
    assert laplacian_variance(blurry).max() == 0.0 and q._assess_sharpness(blurry) == 0.0
    h = hsv_histograms(frames[[0, 1, 200]])
    c = histogram_correlation(h[[0, 0]], h[[1, 2]])
    assert c[0] > 0.9 and c[1] < 0.7


def test_boundaries_terminate_and_respect_scenes():
    c = VideoChunker(ChunkConfig(chunk_duration=300, overlap_duration=30, min_chunk_duration=60))
    uni = c._generate_chunk_boundaries(1000.0, [])
    assert uni[0] == (0.0, 300.0) and uni[1][0] == 270.0 and uni[-1][1] == 1000.0
    sc = c._generate_chunk_boundaries(1000.0, [200.0, 900.0])
    assert sc[0] == (0.0, 200.0)          # runs to the cut
    assert sc[1][0] == 170.0              # the next chunk starts one overlap earlier
    assert all(e - s <= 450 for s, e in sc) and sc[-1][1] == 1000.0


def test_chunk_video_writes_index_and_dataset_reads_it(tmp_path):
    frames = _clip()
    for strategy in ("uniform", "adaptive", "scene_aware"):
        out = tmp_path / strategy
        chunker = VideoChunker(ChunkConfig(chunk_duration=4, overlap_duration=1,
                                           min_chunk_duration=2, target_fps=10,
                                           blur_threshold=50.0, min_quality=0.3,
                                           sampling_strategy=strategy))
        chunks = chunker.chunk_video(str(tmp_path / "drive.mp4"), str(out),
                                     cache_dir=str(tmp_path / "cache"), frames=frames)
        assert chunks, strategy
        index = json.loads((out / "drive_chunks.json").read_text())
        assert index["total_chunks"] == len(chunks)
        for ch in chunks:
            assert {"name", "path", "start_time", "end_time", "num_frames",
                    "quality_score", "frame_indices"} <= set(ch)
            idx = np.array(ch["frame_indices"])
            assert (np.diff(idx) > 0).all() and ch["start_frame"] <= idx[0] < idx[-1] < ch["end_frame"]
        if strategy == "scene_aware":
            assert any(150 in ch["frame_indices"] for ch in chunks)
        ds = ChunkedVideoDataset(str(out), sequence_length=8, seed=0)
        item = ds[0]
        assert item["frames"].shape == (8, 3, 48, 64) and float(item["frames"].max()) <= 1.0
