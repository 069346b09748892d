"""Native data runtime (ENFCAP, telemetry, PNG frames) and the Enfusion dataset (CPU)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from drivedit_b200.data.enfcap import ENFCAPReader, ENFCAPWriter, FrameFlags, read_enfcap_py
from drivedit_b200.data.native import native
from drivedit_b200.data.telemetry import ControlNormalizer, TelemetryParser


def _write_capture(path, n=12, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = ENFCAPWriter(str(path), start_timestamp=1234.5, flags=16)
    frames = []
    for i in range(n):
        ne, nr = i % 4, (i * 3) % 5
        f = dict(frame_id=i, timestamp=0.2 * i, ego_transform=torch.randn(3, 4, generator=g),
                 vehicle_state=torch.randn(10, generator=g),
                 entity_type=torch.randint(0, 8, (ne,), generator=g),
                 entity_pos=torch.randn(ne, 3, generator=g), road_points=torch.randn(nr, 3, generator=g),
                 flags=int(FrameFlags.ANCHOR) if i % 5 == 0 else 0)
        w.write_frame(**f)
        frames.append(f)
    w.finalize()
    return frames


def test_enfcap_roundtrip_native_and_python(tmp_path):
    p = tmp_path / "capture.enfcap"
    frames = _write_capture(p)
    r = ENFCAPReader(str(p))
    assert r.frame_count == 12 and abs(r.start_timestamp - 1234.5) < 1e-3
    py = read_enfcap_py(str(p))
    assert py["frame_count"] == 12
    for i, f in enumerate(frames):
        d = r.read_frame(i)
        assert d["frame_id"] == i and d["flags"] == f["flags"]
        assert torch.equal(d["ego_transform"], f["ego_transform"])
        assert torch.equal(d["entity_pos"], f["entity_pos"])
        assert torch.equal(d["road_points"], f["road_points"])
        assert np.array_equal(py["frames"][i]["vehicle_state"], f["vehicle_state"].numpy())
    b = r.read_frames(2, 9, threads=3)
    assert b["ego_transform"].shape == (7, 3, 4)
    eo = b["entity_offsets"]
    assert torch.equal(b["entity_pos"][eo[3]:eo[4]], frames[5]["entity_pos"])
    ok, msg = r.validate()
    assert ok == 12 and msg == ""
    with pytest.raises(Exception):
        r.read_frame(12)


def test_png_decode_and_resize(tmp_path):
    from PIL import Image
    rng = np.random.default_rng(0)
    img = rng.integers(0, 256, (37, 53, 3), dtype=np.uint8)
    p = tmp_path / "f.png"
    Image.fromarray(img).save(p)
    dec = native().decode_png(p.read_bytes())
    assert np.array_equal(dec.numpy(), img)
    rgba = rng.integers(0, 256, (20, 30, 4), dtype=np.uint8)
    Image.fromarray(rgba, "RGBA").save(tmp_path / "a.png")
    assert np.array_equal(native().decode_png((tmp_path / "a.png").read_bytes()).numpy(), rgba[..., :3])
    out = native().load_frames([str(p)] * 3, 24, 32, 2)
    ref = F.interpolate(torch.from_numpy(img).permute(2, 0, 1)[None].float(), size=(24, 32),
                        mode="bilinear", align_corners=False)[0].permute(1, 2, 0)
    assert out.shape == (3, 24, 32, 3)
    assert (out[1].float() - ref).abs().max() <= 1.0


def test_telemetry_parse_and_normalize(tmp_path):
    csv = ("Timestamp,Lat,lng,alt,Heading,speed,steer,gas,braking,rpm\n"
           "0,1.0,2.0,3.0,10,36,0.5,0.7,0.0,2000\n"
           "200,1.1,2.1,3.0,20,72,-2.0,0.0,0.4,2500\n"
           "bad,row,,,,,,,,\n"
           "400,1.2,2.2,3.0,30,18,0.1,0.2,0.1,2100\n")
    p = tmp_path / "telemetry.csv"
    p.write_text(csv)
    raw = TelemetryParser.parse_raw(p)
    assert int(raw["_rows"]) == 3
    assert torch.allclose(raw["speed_ms"], torch.tensor([10.0, 20.0, 5.0], dtype=torch.float64))
    tel = TelemetryParser().parse_csv(p)
    py = ControlNormalizer().normalize_controls(tel)
    nat = ControlNormalizer.normalize_native(raw)
    assert torch.allclose(py, nat, atol=1e-6)
    assert py[1, 0] == -1.0 and abs(float(py[0, 1]) - 0.7) < 1e-6 and abs(float(py[1, 5]) - 0.4) < 1e-6
    up = TelemetryParser.interpolate_to_frame_rate(tel, 5)
    assert up["speed"].shape == (5,) and abs(up["speed"][2] - 20.0) < 1e-5
    T = TelemetryParser.compute_ego_transform(tel["position"], tel["rotation"])
    assert T.shape == (3, 4, 4) and np.allclose(T[:, 3, 3], 1.0)
    assert np.allclose(T[0, :3, :3] @ T[0, :3, :3].T, np.eye(3), atol=1e-5)


def test_enfusion_dataset(tmp_path):
    from PIL import Image
    from drivedit_b200.data.enfusion import (EnfusionCollator, EnfusionDataset, EnfusionDatasetConfig,
                                             create_enfusion_dataloaders)
    rng = np.random.default_rng(1)
    for s in range(2):
        d = tmp_path / f"session_{s:04d}"
        (d / "frames").mkdir(parents=True)
        for i in range(10):
            Image.fromarray(rng.integers(0, 256, (24, 40, 3), dtype=np.uint8)).save(d / "frames" / f"frame_{i:06d}.png")
        rows = ["timestamp_ms,steering,throttle,brake,speed_kmh"]
        rows += [f"{i * 200},{np.sin(i):.3f},0.5,0.0,{30 + i}" for i in range(6)]
        (d / "telemetry.csv").write_text("\n".join(rows) + "\n")
        (d / "session_info.txt").write_text("map: everon\nweather: clear\n")
        _write_capture(d / "capture.enfcap", n=10, seed=s)
    cfg = EnfusionDatasetConfig(sequence_length=4, frame_skip=2, image_size=(16, 32), load_depth=False,
                                augment=False)
    ds = EnfusionDataset(tmp_path, cfg)
    assert len(ds) == 2 * (10 - 7 + 1)
    x = ds[0]
    assert x["frames"].shape == (4, 3, 16, 32) and 0 <= float(x["frames"].min()) and float(x["frames"].max()) <= 1
    assert x["controls"].shape == (4, 6) and x["ego_transform"].shape == (4, 4, 4)
    assert x["anchor_mask"].tolist() == [True, False, False, False]   # ENFCAP anchor flags (0, 2, 4, 6)
    assert x["metadata"]["map"] == "everon"
    b = EnfusionCollator()([ds[0], ds[1]])
    assert b["frames"].shape == (2, 4, 3, 16, 32)
    tr, va, te = create_enfusion_dataloaders(tmp_path, cfg, batch_size=2, num_workers=0, pin_memory=False,
                                             train_ratio=0.5, val_ratio=0.0, seed=0, device="cpu")
    assert len(tr.dataset) + len(va.dataset) + len(te.dataset) == len(ds) and len(va.dataset) == 0
    from drivedit_b200.data.enfusion import EnfusionToDriveDiTAdapter
    ad = EnfusionToDriveDiTAdapter(8)(next(iter(tr)))
    assert ad["controls"].shape[-1] == 8 and "anchor_mask" in ad
    from drivedit_b200.data.enfusion import EnfusionDataLoader
    dl = EnfusionDataLoader(ds, batch_size=3, num_workers=0, device="cpu")
    batches = list(dl)
    assert len(dl) == len(batches) == len(ds) // 3
    assert batches[0]["frames"].shape == (3, 4, 3, 16, 32) and "scene_entities" not in batches[0]
    from drivedit_b200.data.enfusion_preprocessing import EnfusionQualityFilter
    ranked = EnfusionQualityFilter().filter_sessions(sorted(tmp_path.iterdir()), min_quality=0.0)
    assert len(ranked) == 2 and ranked[0][1] >= ranked[1][1]


def test_transforms_collate_samplers(tmp_path):
    from drivedit_b200.data.collate import ChunkedBatchCollator, MemoryEfficientCollator, VideoCollator
    from drivedit_b200.data.pipeline import DatasetSplitter, DrivingDataset, VideoMemoryMap
    from drivedit_b200.data.sampler import (AdaptiveSampler, BalancedSampler, ChunkedSampler,
                                            SequentialChunkSampler, TemporalSampler)
    from drivedit_b200.data.transforms import (AugmentationPipeline, FrameTransforms, VideoTransforms,
                                               clip_augment_reference)
    torch.manual_seed(0)
    v = torch.rand(6, 3, 20, 24)
    assert torch.allclose(FrameTransforms.denormalize(FrameTransforms.normalize(v)), v, atol=1e-6)
    assert FrameTransforms.center_crop(v, (10, 12)).shape == (6, 3, 10, 12)
    assert torch.allclose(FrameTransforms.hue(v[0], 0.0), v[0].clamp(0, 1), atol=1e-5)
    assert VideoTransforms.temporal_subsample(v, 2).shape[0] == 3
    out = AugmentationPipeline.create_training_pipeline((16, 16))(v)
    assert out.shape == (6, 3, 16, 16)
    x = torch.rand(2, 3, 3, 4, 5)
    y = clip_augment_reference(x, torch.tensor([1, 0]), torch.tensor([0.1, 0.0]), torch.tensor([1.0, 1.0]))
    assert torch.allclose(y[0], (x[0].flip(-1) + 0.1).clamp(0, 1)) and torch.allclose(y[1], x[1])
    batch = [{"frames": torch.rand(n, 3, 4, 4), "controls": torch.rand(n, 6), "id": n} for n in (3, 5)]
    b = VideoCollator()(batch)
    assert b["frames"].shape == (2, 5, 3, 4, 4) and b["sequence_mask"].sum() == 8 and b["id"] == [3, 5]
    assert ChunkedBatchCollator(chunk_size=2, overlap=1)(batch)["frames"].shape[1] == 2
    assert len(MemoryEfficientCollator(frame_memory_limit_mb=1e-4)(batch)["id"]) == 1
    assert len(MemoryEfficientCollator(max_batch_frames=10 ** 6)(batch)["id"]) == len(batch)
    class _Seqs(torch.utils.data.Dataset):      # sequence structure as VideoDataset exposes it
        sequences = [{"num_frames": 10}, {"num_frames": 3}, {"num_frames": 20}]
        sequence_indices = [(0, 0), (0, 4), (2, 0), (2, 4), (2, 8), (2, 12)]

        def __len__(self):
            return len(self.sequence_indices)

        def __getitem__(self, i):
            return {"class_label": "a" if i < 5 else "b"}
    ds_s = _Seqs()
    ts = TemporalSampler(ds_s, "sparse", sequence_length=4, seed=0)
    assert ts.temporal_indices == [(0, 0), (0, 4), (2, 0), (2, 4), (2, 8), (2, 12), (2, 16)]
    assert sorted(ts) == list(range(7)) and list(ts) == list(ts)        # seeded: repeatable
    assert len(TemporalSampler(ds_s, "dense", sequence_length=4)) == 7 + 17
    bs = BalancedSampler(ds_s, seed=0)
    assert {k: len(v) for k, v in bs.class_indices.items()} == {"a": 5, "b": 1}
    assert bs.get_class_distribution() == {"a": 5, "b": 5} and len(bs) == 10
    assert sorted(ChunkedSampler(ds_s, chunk_size=3, overlap=1, shuffle_chunks=False)) == [0, 1, 2, 2, 3, 4, 4, 5]
    sc = list(SequentialChunkSampler(ds_s, sequences_per_chunk=2))
    assert sc == [0, 1, 2, 3, 4, 5]
    ad = AdaptiveSampler(ds_s, adaptation_frequency=1, seed=0)
    ad.update_difficulty_scores(list(range(100)), [0.0, 1.0] * 50)
    list(ad)
    assert ad.get_current_strategy() == "balanced"
    frames = np.random.default_rng(0).integers(0, 256, (12, 8, 10, 3), dtype=np.uint8)
    vm = VideoMemoryMap(str(tmp_path / "clip.mp4"), frames=frames)
    vm2 = VideoMemoryMap(str(tmp_path / "clip.mp4"))  # reopens the cache
    assert torch.allclose(vm2.get_batch([3])[0], torch.from_numpy(frames[3]).permute(2, 0, 1).float() / 255)
    ds = DrivingDataset([vm], sequence_length=4, image_size=(8, 10), augment=False,
                        controls=[np.arange(72, dtype=np.float32).reshape(12, 6)])
    assert len(ds) == 9 and ds[0]["controls"].shape == (4, 6)
    parts = DatasetSplitter.split(ds, (0.5, 0.5))
    assert len(parts[0]) + len(parts[1]) == 9
    ds2 = DrivingDataset([vm], 4, (4, 5), None, 3, False, [np.arange(12, dtype=np.float32)[:, None]])
    x = ds2[1]                     # frames 1, 4, 7, 10 resized to 4 x 5
    assert len(ds2) == 12 - 9 and x["frames"].shape == (4, 3, 4, 5) and x["controls"][:, 0].tolist() == [1, 4, 7, 10]
    tr, va, te = DatasetSplitter.split_by_video([f"v{i}" for i in range(10)], 0.6, 0.2, seed=0)
    assert (len(tr), len(va), len(te)) == (6, 2, 2) and not set(tr) & set(te)
    from drivedit_b200.data.pipeline import StreamingDataLoader
    sl = StreamingDataLoader(ds, batch_size=2, num_workers=0, device="cpu")
    assert len(sl) == 4 and next(iter(sl))["frames"].shape == (2, 4, 3, 8, 10)
