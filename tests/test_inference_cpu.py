"""Inference pipelines and the headless HTTP / WebSocket server (CPU, tiny models)."""
import numpy as np
import pytest
import torch

from drivedit_b200.inference.pipeline import (BatchInferencePipeline, InferencePipeline, PipelineConfig,
                                              RealtimeInferencePipeline)


def _cfg(**kw):
    base = dict(device="cpu", model_preset="tiny", model_overrides=["model.n_layers=2"],
                vae_hidden_dims=[32, 64, 64, 64], vae_use_attention=False, chunk_frames=1, flow_steps=2)
    base.update(kw)
    return PipelineConfig(**base)


@pytest.fixture(scope="module")
def pipe():
    return InferencePipeline(_cfg())


def test_generate_rgb_roundtrip(pipe):
    ctx = torch.randint(0, 256, (1, 4, 128, 128, 3), dtype=torch.uint8)
    r = pipe.generate(ctx, torch.rand(1, 12, 3) * 2 - 1, num_frames=8)
    assert r["generated_frames"].shape == (1, 8, 3, 128, 128)
    assert r["metadata"]["latent_frames"] == 2 and r["performance"]["fps"] > 0
    post = pipe.postprocess_output(r)
    assert post["generated_frames"].dtype == np.uint8 and post["generated_frames"].shape == (1, 8, 128, 128, 3)


def test_latent_only_and_batch():
    p = BatchInferencePipeline(_cfg(use_vae=False, batch_size=2))
    ctx = [torch.randn(1, 2, 16, 16, 16) for _ in range(3)]
    outs = p.generate_batch(ctx, num_frames=3)
    assert len(outs) == 3 and outs[0]["generated_frames"].shape == (1, 3, 16, 16, 16)


def test_realtime_stream():
    p = RealtimeInferencePipeline(_cfg(), context=4)
    frames = [np.random.randint(0, 256, (128, 128, 3), dtype=np.uint8) for _ in range(6)]
    outs = [p.process_frame(f, [0.1, 0.0, 0.2]) for f in frames]
    assert outs[:3] == [None] * 3
    assert all(o is not None and o.shape == (128, 128, 3) for o in outs[3:])


def test_http_and_websocket_server(pipe):
    from fastapi.testclient import TestClient
    from drivedit_b200.inference.server import MultiModalServer, decode_image, encode_image
    rt = RealtimeInferencePipeline(_cfg(), context=2)
    srv = MultiModalServer(pipeline=pipe, realtime_pipeline=rt, device="cpu")
    c = TestClient(srv.app)
    assert c.get("/health").json()["status"] == "healthy"
    assert c.get("/info").json()["model"] == "tiny"
    img = np.random.randint(0, 256, (128, 128, 3), dtype=np.uint8)
    assert np.array_equal(decode_image(encode_image(img)), img)
    r = c.post("/generate", json={"context_frames": [encode_image(img)] * 4, "num_frames": 4}).json()
    assert r["success"], r.get("error")
    assert len(r["generated_frames"]) == 4 and decode_image(r["generated_frames"][0]).shape == (128, 128, 3)
    bad = c.post("/generate", json={"context_frames": ["not-an-image"], "num_frames": 4}).json()
    assert not bad["success"] and bad["error"]
    with c.websocket_connect("/stream") as ws:
        assert ws.receive_json()["type"] == "connected"
        ws.send_json({"type": "ping", "data": {}})
        assert ws.receive_json()["type"] == "pong"
        ws.send_json({"type": "frame", "data": {"image": encode_image(img)}})
        assert ws.receive_json()["type"] == "buffering"
        ws.send_json({"type": "frame", "data": {"image": encode_image(img), "control": [0.0, 0.5, 0.0]}})
        m = ws.receive_json()
        assert m["type"] == "result" and decode_image(m["data"]["generated_frame"]).shape == (128, 128, 3)
