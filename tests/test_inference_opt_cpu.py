"""Inference helpers on CPU: rollout memory bank / evaluator / config mapping, the
optimisation module's benchmark, profiler and streaming wrappers."""
import torch
import torch.nn as nn

from drivedit_b200.config.presets import ModelConfig
from drivedit_b200.inference.optimization import (BenchmarkResult, CompileMode, InferenceOptimizer,
                                                  MemoryTracker, ModelCompiler, OptimizationConfig,
                                                  StreamingInference, benchmark_inference,
                                                  optimize_for_deployment, profile_bottlenecks)
from drivedit_b200.inference.rollout import (InferenceConfig, MemoryBank, RolloutEvaluator,
                                             StreamingRollout)
from drivedit_b200.models.world_dit import WorldDiT


def test_memory_bank_is_deterministic_and_bounded():
    mb = MemoryBank(d_model=32, max_spatial_memory=5)
    for i in range(8):
        mb.update(torch.rand(2, 3, 16, 16) * (i + 1), i)
    a, b = mb.get_memory_tokens(top_k=3), mb.get_memory_tokens(top_k=3)
    assert a.shape == (1, 6, 32) and torch.equal(a, b)
    assert len(mb.spatial_memory) == 5
    mb.clear()
    assert mb.get_memory_tokens().shape == (1, 0, 32)


def test_rollout_evaluator_and_generate_sequence():
    ev = RolloutEvaluator()
    g = torch.rand(1, 4, 3, 8, 8)
    m = ev.evaluate_sequence(g, g)
    assert m["mse"] == 0 and m["lpips_proxy"] == 0 and m["temporal_consistency"] == 0
    torch.manual_seed(0)
    model = WorldDiT(ModelConfig(n_layers=2, d_model=64, n_heads=2, mlp_hidden=128, latent_channels=4,
                                 latent_h=8, latent_w=8)).eval()
    ro = StreamingRollout(model, InferenceConfig(max_sequence_length=8, context_window=4, chunk_size=2,
                                                 flow_steps=2))
    out = ro.generate_sequence(torch.randn(1, 2, 4, 8, 8), None, num_frames=4)
    assert out["frames"].shape == (1, 4, 4, 8, 8) and len(out["chunk_ms"]) == 2
    # the reference's construction: (world_model, vae_model, config, device), RGB in and out
    from drivedit_b200.models.vae3d import VAE3DConfig, VAE3Dv2
    vae = VAE3Dv2(VAE3DConfig(latent_dim=4, hidden_dims=[16, 16, 16, 16], num_res_blocks=1,
                              use_attention=False, temporal_compression=1, spatial_compression=8,
                              use_perceptual_loss=False))
    ro = StreamingRollout(model, vae, InferenceConfig(max_sequence_length=8, context_window=4,
                                                      chunk_size=2, flow_steps=2), "cpu")
    rgb = torch.rand(1, 2, 3, 64, 64)
    out = ro.generate_sequence(rgb, torch.zeros(1, 6, 6), 4)
    assert out["generated_frames"].shape == (1, 4, 3, 64, 64)
    assert out["full_sequence"].shape == (1, 6, 3, 64, 64) and out["performance"]["avg_fps"] > 0
    si = StreamingInference(model, OptimizationConfig(chunk_size=2, target_fps=1.0), device="cpu")
    si.initialize(num_layers=2)
    frames = [f for f, _ in si.generate_stream(torch.randn(1, 2, 4, 8, 8), torch.zeros(1, 6, 2), 4)]
    assert len(frames) == 4 and frames[0].shape == (1, 4, 8, 8)
    assert si.get_streaming_stats()["frames"] == 4


def test_benchmark_profile_and_deployment_cpu():
    net = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 16))
    r = benchmark_inference(net, (4, 16), device="cpu", num_warmup=2, num_iterations=5, use_autocast=False)
    assert isinstance(r, BenchmarkResult) and r.avg_latency_ms > 0 and r.to_dict()["config"]["batch_size"] == 4
    assert "Latency" in r.summary()
    p = profile_bottlenecks(net, torch.randn(4, 16), device="cpu", num_iterations=2)
    assert p["top_operations"]
    opt, rep = optimize_for_deployment(net, torch.randn(4, 16), "minimal")
    assert rep["optimizations_applied"] == ["eval"] and rep["speedup"] > 0
    comp = ModelCompiler(OptimizationConfig(compile_mode=CompileMode.NONE))
    assert comp.compile(net, (torch.randn(2, 16),)) is net
    io = InferenceOptimizer()
    q = torch.randn(1, 2, 10, 8)
    full = torch.nn.functional.scaled_dot_product_attention(q, q, q, is_causal=True)
    torch.testing.assert_close(io.chunked_attention(q, q, q, chunk_size=3, causal=True), full)
    assert io.initialize_kv_cache(2) is io.get_kv_cache()
    mt = MemoryTracker()
    mt.record("x")
    assert mt.get_report()["samples"] == 1


def test_reference_factories_and_signatures():
    """The inference factories and configs take the reference's positional arguments."""
    from drivedit_b200.inference.optimization import CompileMode, FrameMetrics, ModelCompiler
    from drivedit_b200.inference.pipeline import InferencePipeline, PipelineConfig, create_pipeline
    from drivedit_b200.inference.server import InferenceServer, create_server

    cfg = PipelineConfig(None, None, "cpu", 1, 16, 4, 0.8, False)
    assert cfg.device == "cpu" and cfg.max_sequence_length == 16 and not cfg.use_mixed_precision
    assert ModelCompiler(CompileMode.REDUCE_OVERHEAD, False, False, "inductor", True).disable_cudagraphs
    assert FrameMetrics(0, 1.0, 2.0, 3.0, 5).kv_cache_length == 5
    p = create_pipeline(None, None, "standard", "cpu", model_preset="tiny", use_vae=False)
    assert isinstance(p, InferencePipeline) and p.device.type == "cpu"
    srv = create_server("http", None, None, device="cpu", model_preset="tiny", use_vae=False)
    assert isinstance(srv, InferenceServer)
