"""Native depth loading, background frame service, scene graphs and session discovery (CPU)."""
import json

import numpy as np
import pytest
import torch
from PIL import Image

from drivedit_b200.data.depth import DepthLoader, DepthLoaderConfig, depth_gradient, fill_invalid, log_depth
from drivedit_b200.data.frame_service import FrameLoaderService, FrameRingBuffer
from drivedit_b200.data.native import available
from drivedit_b200.data.scene import BoundingBox3D, EntityClass, SceneParser
from drivedit_b200.data.session import DatasetConfig, SessionMetadata, find_sessions

pytestmark = pytest.mark.skipif(not available(), reason="native data runtime not built")


def _ref_process(a, tw, th, lo=None, hi=None, invert=False):
    a = a.astype(np.float32)
    if lo is None:
        f = a[np.isfinite(a)]
        lo, hi = float(f.min()), float(f.max())
    H, W = a.shape
    ys = np.arange(th) * (H / th)
    xs = np.arange(tw) * (W / tw)
    y0 = np.floor(ys).astype(int)
    x0 = np.floor(xs).astype(int)
    y1 = np.minimum(y0 + 1, H - 1)
    x1 = np.minimum(x0 + 1, W - 1)
    fy = (ys - y0)[:, None]
    fx = (xs - x0)[None]
    top = a[y0][:, x0] * (1 - fx) + a[y0][:, x1] * fx
    bot = a[y1][:, x0] * (1 - fx) + a[y1][:, x1] * fx
    v = top * (1 - fy) + bot * fy
    n = (np.clip(v, lo, hi) - lo) / (hi - lo)
    return 1 - n if invert else n


def test_depth_formats_match_reference_math(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.uniform(1, 80, (30, 50)).astype(np.float32)
    np.save(tmp_path / "d.npy", a)
    np.savez(tmp_path / "s.npz", depth=a)
    np.savez_compressed(tmp_path / "c.npz", other=a * 0, depth=a)
    u16 = (a * 100).astype(np.uint16)
    Image.fromarray(u16).save(tmp_path / "d.png")
    cfg = DepthLoaderConfig(target_width=20, target_height=12)
    want = _ref_process(a, 20, 12)
    for name in ("d.npy", "s.npz", "c.npz"):
        m = DepthLoader(cfg).load(tmp_path / name)
        np.testing.assert_allclose(m.data.numpy(), want, rtol=1e-5, atol=1e-5)
        assert abs(m.original_min - a.min()) < 1e-4
    m = DepthLoader(cfg).load(tmp_path / "d.png")
    np.testing.assert_allclose(m.data.numpy(), _ref_process(u16, 20, 12), rtol=1e-5, atol=1e-5)
    inv = DepthLoader(DepthLoaderConfig(20, 12, 0.0, 100.0, invert_depth=True)).load(tmp_path / "d.npy")
    np.testing.assert_allclose(inv.data.numpy(), _ref_process(a, 20, 12, 0.0, 100.0, True), rtol=1e-5, atol=1e-5)
    batch = DepthLoader(cfg).load_batch_contiguous([tmp_path / "d.npy", tmp_path / "c.npz"], threads=2)
    assert batch.shape == (2, 12, 20) and torch.allclose(batch[0], batch[1])
    with pytest.raises(RuntimeError):
        DepthLoader(DepthLoaderConfig(npz_array_name="missing")).load(tmp_path / "s.npz")
    assert log_depth(torch.tensor([1.0, 10.0]), 1.0, 10.0).tolist() == [0.0, 1.0]
    d = torch.ones(5, 5)
    d[2, 2] = 0
    assert float(fill_invalid(d)[2, 2]) == 1.0 and float(depth_gradient(d).abs().sum()) > 0


def test_frame_service_cache_and_errors(tmp_path):
    rng = np.random.default_rng(1)
    paths = []
    for i in range(4):
        p = tmp_path / f"f{i}.png"
        Image.fromarray(rng.integers(0, 256, (16, 24, 3), dtype=np.uint8)).save(p)
        paths.append(p)
    svc = FrameLoaderService(threads=2, cache_frames=8)
    r1 = svc.submit(paths, 16, 24)
    r2 = svc.submit(paths[::-1], 8, 12)
    out = r1.result()
    assert out.shape == (4, 16, 24, 3)
    assert np.array_equal(out[2].numpy(), np.asarray(Image.open(paths[2])))
    assert r2.result().shape == (4, 8, 12, 3)
    svc.load(paths[:2], 16, 24)
    assert svc.cache_stats()["hits"] >= 2
    with pytest.raises(RuntimeError):
        svc.load([tmp_path / "missing.png"], 16, 24)
    rb = FrameRingBuffer(3)
    for i in range(5):
        rb.push(torch.full((2,), float(i)))
    assert rb.is_full() and rb.latest(2)[:, 0].tolist() == [3.0, 4.0]


def test_scene_graph_queries_and_transforms():
    js = {"frame_id": 1, "timestamp": 1.0,
          "ego_pose": {"position": [10, 0, 0], "rotation": [0.7071068, 0, 0, 0.7071068]},
          "entities": [{"id": 1, "class": "car", "position": [20, 0, 0], "velocity": [1, 0, 0]},
                       {"id": 2, "class": "person", "position": [10, 5, 0]},
                       {"id": 3, "class": "tree", "position": [-50, 0, 0], "confidence": 0.2}]}
    sp = SceneParser()
    sc = sp.parse_str(json.dumps(js))
    assert [e.entity_class for e in sc.entities] == [EntityClass.CAR, EntityClass.PEDESTRIAN, EntityClass.VEGETATION]
    assert len(sc.get_dynamic()) == 2 and len(sc.get_static()) == 1
    assert [e.id for e in sc.get_within_distance([10, 0, 0], 10.5)] == [1, 2]
    assert [e.id for e in sc.get_in_fov(90, 30)] == [1, 2]
    ego = SceneParser.transform_to_ego(sc)       # ego at (10,0,0) facing +y
    np.testing.assert_allclose(ego.get_entity(1).position, [0, -10, 0], atol=1e-5)
    np.testing.assert_allclose(ego.get_entity(2).position, [5, 0, 0], atol=1e-5)
    sc2 = sp.parse_str(json.dumps({**js, "timestamp": 1.5, "entities": [
        {"id": 11, "class": "car", "position": [21, 0, 0]}, {"id": 12, "class": "person", "position": [10, 6, 0]}]}))
    m = SceneParser.match_entities(sc, sc2, 3.0)
    assert m == [(1, 11), (2, 12)]
    SceneParser.compute_velocities(sc, sc2, m)
    np.testing.assert_allclose(sc2.get_entity(11).velocity, [2, 0, 0], atol=1e-5)
    SceneParser.filter_by_confidence(sc, 0.5)
    assert len(sc) == 2 and SceneParser.to_feature_vector(sc, 4).shape == (4, 16)
    b = BoundingBox3D((0, 0, 0), (2, 2, 2))
    assert b.contains((0.9, 0.9, 0.9)) and not b.contains((1.1, 0, 0))
    assert abs(b.iou_approx(BoundingBox3D((1, 0, 0), (2, 2, 2))) - 4 / 12) < 1e-6
    rot = BoundingBox3D((0, 0, 0), (4, 2, 2), (0.7071068, 0, 0, 0.7071068))
    assert np.allclose(np.abs(rot.corners()).max(0), [1, 2, 1], atol=1e-5)


def test_sessions_and_presets(tmp_path):
    for name in ("s1", "nested/s2"):
        d = tmp_path / name / "frames"
        d.mkdir(parents=True)
        Image.fromarray(np.zeros((6, 10, 3), np.uint8)).save(d / "frame_000000.png")
        Image.fromarray(np.zeros((6, 10, 3), np.uint8)).save(d / "frame_000001.png")
    (tmp_path / "s1" / "telemetry.csv").write_text("t\n")
    found = find_sessions(tmp_path)
    assert [p.name for p in found] == ["s2", "s1"] or [p.name for p in found] == ["s1", "s2"]
    md = SessionMetadata.from_dir(tmp_path / "s1")
    assert (md.num_frames, md.width, md.height, md.has_telemetry) == (2, 10, 6, True)
    assert DatasetConfig.minimal().image_width == 128 and DatasetConfig.production().load_flow


def test_native_batch_loader_matches_dataset(tmp_path):
    import numpy as np
    import torch
    from PIL import Image

    from drivedit_b200.data import native_loader as nl

    if not nl.check_native_available():
        pytest.skip("data runtime not built")
    rng = np.random.default_rng(0)
    for s in range(3):
        d = tmp_path / f"session_{s:04d}"
        (d / "frames").mkdir(parents=True)
        for i in range(8):
            Image.fromarray(rng.integers(0, 256, (20, 36, 3), dtype=np.uint8)).save(d / "frames" / f"frame_{i:06d}.png")
        rows = ["timestamp_ms,steering,throttle,brake,speed_kmh"]
        rows += [f"{i * 100},{np.sin(i):.3f},0.5,0.0,{30 + i}" for i in range(8)]
        (d / "telemetry.csv").write_text("\n".join(rows) + "\n")
    cfg = nl.RustDatasetConfig(sequence_length=3, frame_skip=2, image_height=16, image_width=24, load_depth=False,
                               num_workers=2)
    ds = nl.RustEnfusionDataset(tmp_path, cfg)
    assert len(ds) == 3 * 4
    loader = nl.RustBatchLoader(ds, batch_size=5, shuffle=False, drop_last=False)
    batches = list(loader)
    assert len(batches) == len(loader) == 3
    assert [b["frames"].shape[0] for b in batches] == [5, 5, 2]
    b0 = batches[0]
    assert b0["frames"].shape == (5, 3, 3, 16, 24) and b0["controls"].shape == (5, 3, 6)
    for j in range(5):
        ref = ds[j]
        torch.testing.assert_close(b0["frames"][j], ref["frames"], atol=0, rtol=0)
        torch.testing.assert_close(b0["controls"][j], ref["controls"])
        assert b0["anchor_mask"][j].tolist() == ref["anchor_mask"].tolist()
    tr, va = nl.create_rust_dataloaders(tmp_path, cfg, batch_size=2, val_fraction=0.34)
    assert len(tr.dataset) + len(va.dataset) == len(ds)
    hcfg = dict(sequence_length=3, frame_skip=2, image_size=(16, 24), load_depth=False, num_workers=0)
    hy = nl.get_best_loader(tmp_path, 2, **{k: v for k, v in hcfg.items() if k != "sequence_length"},
                            sequence_length=3)
    assert hy.backend == "rust" and hy.is_rust
    n = sum(1 for _ in hy)
    assert n == len(hy) and hy.get_performance_stats()["batch_count"] == n
    py = nl.HybridDataLoader(tmp_path, nl.HybridLoaderConfig(prefer_rust=False, batch_size=2, **hcfg))
    assert py.backend == "python" and next(iter(py))["frames"].shape == (2, 3, 3, 16, 24)
    tr, va, te = nl.create_hybrid_dataloaders(tmp_path, nl.HybridLoaderConfig(batch_size=2, **hcfg),
                                              train_ratio=0.34, val_ratio=0.34, seed=0)
    assert sum(len(l._loader.dataset) for l in (tr, va, te)) == len(ds)
    r = nl.benchmark_rust_vs_python(tmp_path, cfg, batch_size=2, num_batches=2)
    assert r["native_batches_per_s"] > 0 and r["python_batches_per_s"] > 0
    assert nl.get_rust_version()
