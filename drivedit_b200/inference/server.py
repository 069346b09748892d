"""Headless HTTP / WebSocket serving of the inference pipelines (FastAPI).

Endpoints and message models of the reference ``inference/server.py``:
``InferenceRequest`` / ``InferenceResponse`` / ``StreamingMessage`` (:30-53),
``InferenceServer`` (base64 image codec, request processing, :56-206), ``HTTPServer``
(``GET /health``, ``POST /generate``, ``GET /info``, :209-269), ``WebSocketServer``
(``/stream``: ``frame`` / ``control`` / ``ping`` messages, :272-414),
``MultiModalServer`` (all routes on one app, :417-499) and ``create_server``
(:502-530). Images travel as base64 PNG (or JPEG) strings; no display or graphics stack
is involved. ``InferenceServer`` accepts an already-built pipeline (tests, embedding).
"""
from __future__ import annotations

import base64
import json
import time
from typing import Any, Dict, List, Optional, Union

import numpy as np
import torch

try:
    from fastapi import FastAPI, WebSocket, WebSocketDisconnect
    from fastapi.middleware.cors import CORSMiddleware
    from pydantic import BaseModel

    FASTAPI_AVAILABLE = True
except ImportError:  # pragma: no cover - the image ships FastAPI
    FASTAPI_AVAILABLE = False
    BaseModel = object

from .pipeline import InferencePipeline, PipelineConfig, RealtimeInferencePipeline


class InferenceRequest(BaseModel):
    context_frames: List[str]
    controls: Optional[List[List[float]]] = None
    num_frames: int = 16
    temperature: float = 0.8
    return_intermediates: bool = False


class InferenceResponse(BaseModel):
    generated_frames: List[str]
    context_frames: List[str]
    metadata: Dict[str, Any]
    performance: Dict[str, float]
    success: bool = True
    error: Optional[str] = None


class StreamingMessage(BaseModel):
    type: str
    data: Union[str, Dict[str, Any]]
    timestamp: float


def encode_image(arr: np.ndarray, fmt: str = ".png") -> str:
    import cv2

    a = np.asarray(arr)
    if a.dtype != np.uint8:
        a = (np.clip(a, 0, 1) * 255).round().astype(np.uint8)
    if a.ndim == 3 and a.shape[0] == 3 and a.shape[-1] != 3:
        a = a.transpose(1, 2, 0)
    ok, buf = cv2.imencode(fmt, a[:, :, ::-1] if a.ndim == 3 else a)
    if not ok:
        raise ValueError("Failed to encode image")
    return base64.b64encode(buf.tobytes()).decode("ascii")


def decode_image(b64: str) -> np.ndarray:
    import cv2

    raw = np.frombuffer(base64.b64decode(b64), dtype=np.uint8)
    img = cv2.imdecode(raw, cv2.IMREAD_COLOR)
    if img is None:
        raise ValueError("Failed to decode image")
    return img[:, :, ::-1].copy()


class InferenceServer:
    def __init__(self, model_path: Optional[str] = None, vae_path: Optional[str] = None, device: str = "cuda",
                 max_batch_size: int = 4, enable_optimization: bool = True,
                 pipeline: Optional[InferencePipeline] = None, realtime_pipeline=None, **config_kw):
        self.device, self.max_batch_size = device, max_batch_size
        if pipeline is None:
            cfg = PipelineConfig(model_path=model_path, vae_path=vae_path, device=device,
                                 batch_size=max_batch_size, use_torch_compile=enable_optimization, **config_kw)
            pipeline = InferencePipeline(cfg)
            realtime_pipeline = realtime_pipeline or RealtimeInferencePipeline(cfg)
        self.pipeline = pipeline
        self.realtime_pipeline = realtime_pipeline
        self.active_connections: List[Any] = []
        self.is_running = False

    _decode_image = staticmethod(decode_image)
    _encode_image = staticmethod(encode_image)

    def process_inference_request(self, request: InferenceRequest) -> InferenceResponse:
        try:
            ctx = np.stack([decode_image(f) for f in request.context_frames])       # [T, H, W, 3]
            ctx_t = torch.from_numpy(ctx)[None]
            ctl = torch.tensor(request.controls, dtype=torch.float32)[None] if request.controls else None
            r = self.pipeline.generate(ctx_t, ctl, num_frames=request.num_frames)
            post = self.pipeline.postprocess_output(r)
            gen = [encode_image(f) for f in post["generated_frames"][0]]
            ctx_out = [encode_image(f) for f in post["context_frames"][0]]
            return InferenceResponse(generated_frames=gen, context_frames=ctx_out, metadata=r["metadata"],
                                     performance={k: float(v) for k, v in r["performance"].items()})
        except Exception as e:  # noqa: BLE001 - reported to the client
            return InferenceResponse(generated_frames=[], context_frames=[], metadata={}, performance={},
                                     success=False, error=str(e))

    # ------------------------------------------------------------------ streaming
    async def handle_streaming_session(self, websocket):
        frame_count = 0
        while True:
            try:
                msg = json.loads(await websocket.receive_text())
                kind = msg.get("type")
                if kind == "frame":
                    d = msg["data"]
                    arr = decode_image(d["image"])
                    ctl = np.asarray(d["control"], dtype=np.float32) if "control" in d else None
                    t0 = time.perf_counter()
                    out = self.realtime_pipeline.process_frame(arr, ctl)
                    if out is not None:
                        await websocket.send_text(StreamingMessage(
                            type="result", data={"generated_frame": encode_image(out), "frame_id": frame_count,
                                                 "processing_time_ms": (time.perf_counter() - t0) * 1000.0},
                            timestamp=time.time()).model_dump_json())
                        frame_count += 1
                    else:
                        await websocket.send_text(StreamingMessage(
                            type="buffering", data={"frames_received": len(self.realtime_pipeline.buffer)},
                            timestamp=time.time()).model_dump_json())
                elif kind == "control":
                    await websocket.send_text(StreamingMessage(type="control_ack", data={"received": True},
                                                               timestamp=time.time()).model_dump_json())
                elif kind == "ping":
                    await websocket.send_text(StreamingMessage(type="pong", data={"server_time": time.time()},
                                                               timestamp=time.time()).model_dump_json())
                else:
                    await websocket.send_text(StreamingMessage(type="error", data=f"unknown type {kind!r}",
                                                               timestamp=time.time()).model_dump_json())
            except WebSocketDisconnect:
                break
            except Exception as e:  # noqa: BLE001
                await websocket.send_text(StreamingMessage(type="error", data=str(e),
                                                           timestamp=time.time()).model_dump_json())

    def _add_http_routes(self, app):
        @app.get("/health")
        async def health_check():
            return {"status": "healthy", "device": str(self.pipeline.device), "timestamp": time.time()}

        @app.post("/generate", response_model=InferenceResponse)
        async def generate_video(request: InferenceRequest):
            return self.process_inference_request(request)

        @app.get("/info")
        async def server_info():
            return {"device": str(self.pipeline.device), "max_batch_size": self.max_batch_size,
                    "model_loaded": True, "model": self.pipeline.cfg.model.name,
                    "capabilities": {"batch_inference": True, "streaming": self.realtime_pipeline is not None,
                                     "mixed_precision": self.pipeline.dtype == torch.bfloat16}}

    def _add_ws_routes(self, app):
        @app.websocket("/stream")
        async def websocket_endpoint(websocket: WebSocket):
            await websocket.accept()
            self.active_connections.append(websocket)
            if self.realtime_pipeline is not None:
                self.realtime_pipeline.start_streaming()
            await websocket.send_text(StreamingMessage(type="connected", data={"status": "ready"},
                                                       timestamp=time.time()).model_dump_json())
            try:
                await self.handle_streaming_session(websocket)
            finally:
                if websocket in self.active_connections:
                    self.active_connections.remove(websocket)

    def _make_app(self, title: str):
        if not FASTAPI_AVAILABLE:
            raise ImportError("FastAPI is required for the servers")
        app = FastAPI(title=title, description="Driving world-model video generation API", version="1.0.0")
        app.add_middleware(CORSMiddleware, allow_origins=["*"], allow_credentials=True, allow_methods=["*"],
                           allow_headers=["*"])
        return app


class HTTPServer(InferenceServer):
    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.app = self._make_app("DriveDiT-B200 Inference API")
        self._add_http_routes(self.app)

    def run(self, host: str = "127.0.0.1", port: int = 8000):
        import uvicorn

        uvicorn.run(self.app, host=host, port=port)


class WebSocketServer(InferenceServer):
    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.app = self._make_app("DriveDiT-B200 Streaming API")
        self._add_ws_routes(self.app)

    def run(self, host: str = "127.0.0.1", port: int = 8001):
        import uvicorn

        uvicorn.run(self.app, host=host, port=port)


class MultiModalServer(InferenceServer):
    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.app = self._make_app("DriveDiT-B200 Multi-Modal API")
        self._add_http_routes(self.app)
        self._add_ws_routes(self.app)

    def run(self, host: str = "127.0.0.1", port: int = 8000):
        import uvicorn

        uvicorn.run(self.app, host=host, port=port)


def create_server(server_type: str = "http", model_path: Optional[str] = None,
                  vae_path: Optional[str] = None, **kwargs) -> InferenceServer:
    """``http``, ``websocket`` or ``multimodal`` (inference/server.py:502-527)."""
    kinds = {"http": HTTPServer, "websocket": WebSocketServer, "multimodal": MultiModalServer}
    if server_type not in kinds:
        raise ValueError(f"Unknown server type: {server_type}")
    return kinds[server_type](model_path, vae_path, **kwargs)


def main():
    import argparse

    p = argparse.ArgumentParser(description="headless DriveDiT-B200 inference server")
    p.add_argument("--type", default="multimodal", choices=["http", "websocket", "multimodal"])
    p.add_argument("--model-path")
    p.add_argument("--vae-path")
    p.add_argument("--device", default="cuda")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--preset", default="rollout_dit_b")
    a = p.parse_args()
    create_server(a.type, model_path=a.model_path, vae_path=a.vae_path, device=a.device,
                  model_preset=a.preset).run(a.host, a.port)


if __name__ == "__main__":
    main()
