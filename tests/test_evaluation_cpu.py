"""Evaluation metrics, closed-loop evaluator, benchmarks and evaluators (CPU)."""
import math

import torch

from drivedit_b200.evaluation.metrics import (ControlMetrics, LatentMetrics, PerceptualMetrics, PhysicsMetrics,
                                              TemporalConsistencyMetrics, VideoMetrics, compute_all_metrics)


def test_video_and_perceptual_metrics():
    torch.manual_seed(0)
    x = torch.rand(2, 3, 3, 32, 32)
    assert VideoMetrics.psnr(x, x) > 100 and abs(float(VideoMetrics.ssim(x, x)) - 1) < 1e-5
    y = (x + 0.1 * torch.randn_like(x)).clamp(0, 1)
    assert 15 < float(VideoMetrics.psnr(y, x)) < 30 and float(VideoMetrics.ssim(y, x)) < 0.99
    assert float(VideoMetrics.lpips_proxy(y, x)) > float(VideoMetrics.lpips_proxy(x, x))
    a, b = torch.randn(2000, 8), torch.randn(2000, 8)
    assert float(PerceptualMetrics.frechet_distance(a, b)) < 0.2
    assert float(PerceptualMetrics.frechet_distance(a, b + 3)) > 60
    assert abs(float(PerceptualMetrics.inception_score(torch.full((10, 5), 0.2))) - 1.0) < 1e-5
    m = compute_all_metrics(y, x, torch.zeros(2, 3, 6), torch.zeros(2, 3, 6))
    assert set(["psnr", "ssim", "temporal_mse", "warping_error", "steering_accuracy"]) <= set(m)


def test_temporal_control_physics_metrics():
    f = torch.rand(1, 1, 3, 16, 16).expand(1, 4, 3, 16, 16)
    assert float(TemporalConsistencyMetrics.temporal_mse(f)) == 0
    assert float(TemporalConsistencyMetrics.frame_warping_error(f)) < 1e-6
    c = torch.linspace(0, 1, 10).view(1, 10, 1).expand(1, 10, 6)
    assert float(ControlMetrics.control_smoothness(c)) < 1e-10
    line = torch.stack([torch.arange(10.0), torch.zeros(10)], -1)[None]
    assert float(PhysicsMetrics.trajectory_smoothness(line)) == 0
    th = torch.linspace(0, math.pi, 20)
    circle = torch.stack([5 * th.cos(), 5 * th.sin()], -1)[None]
    assert float(PhysicsMetrics.turning_radius_validity(circle, 4.0)) == 1.0
    assert float(PhysicsMetrics.turning_radius_validity(circle, 6.0)) == 0.0
    z = torch.randn(4, 3, 8)
    assert abs(float(LatentMetrics.latent_cosine_similarity(z, z)) - 1) < 1e-6


def test_closed_loop_benchmarks_evaluators():
    from drivedit_b200.config import get_config
    from drivedit_b200.evaluation.benchmarks import PerformanceBenchmark, WorldModelBenchmark
    from drivedit_b200.evaluation.closed_loop import (ClosedLoopEvaluator, EvaluationConfig,
                                                      create_emergency_stop_task, create_obstacle_avoidance_task)
    from drivedit_b200.evaluation.evaluators import BatchEvaluator, RealTimeEvaluator, SequenceEvaluator
    from drivedit_b200.models.world_dit import WorldDiT
    torch.manual_seed(0)
    m = WorldDiT(get_config("tiny", ["model.n_layers=2"]).model)
    ev = ClosedLoopEvaluator(m, EvaluationConfig(flow_steps=1, num_trajectory_samples=6, planning_horizon=6,
                                                 replan_frequency=2), device="cpu")
    stop = ev.evaluate_episode(create_emergency_stop_task(), torch.randn(2, 16, 16, 16), {"speed": 3.0})
    assert stop.task_success and stop.task_duration_steps >= 5
    obs = ev.evaluate_episode(create_obstacle_avoidance_task((2.0, 0.0)), torch.randn(2, 16, 16, 16),
                              {"speed": 6.0})
    assert obs.predictions.shape[1] == 2 and obs.avg_inference_time_ms > 0
    scaling = ev.evaluate_with_inference_scaling(create_emergency_stop_task(), torch.randn(1, 16, 16, 16),
                                                 {"speed": 2.0}, (1, 2))
    assert scaling[2].planning_iterations_used >= scaling[1].planning_iterations_used
    perf = PerformanceBenchmark(m, "cpu", batch_sizes=(1, 2), frames=2).run_performance_suite()
    assert perf["latency"]["p99_ms"] >= perf["latency"]["p50_ms"] > 0
    data = {"latents": torch.randn(2, 4, 16, 16, 16), "actions": torch.rand(2, 4, 2)}
    res = WorldModelBenchmark(m, "cpu").run_full_benchmark(data)
    assert len(res["long_sequences"]["error_growth"]) == 4
    assert "mse" in SequenceEvaluator(m, "cpu").evaluate_sequence(data["latents"], data["actions"])
    assert BatchEvaluator(m, "cpu", frames=2).find_optimal_batch_size((1, 2)) in (1, 2)
    rt = RealTimeEvaluator(m, "cpu").evaluate_real_time_performance(target_fps=1.0, frames=4, chunk_frames=2,
                                                                    flow_steps=1)
    assert rt["fps"] > 0


def test_reference_constructor_forms():
    from drivedit_b200.evaluation.benchmarks import WorldModelBenchmark
    from drivedit_b200.evaluation.closed_loop import (create_emergency_stop_task, create_lane_following_task,
                                                      create_obstacle_avoidance_task)
    from drivedit_b200.evaluation.evaluators import SequenceEvaluator
    m = torch.nn.Linear(2, 2)
    b = WorldModelBenchmark(m, None, "cpu", None)
    assert b.device.type == "cpu" and b.vae_model is None
    assert SequenceEvaluator(m, None, "cpu", False).device.type == "cpu"
    assert create_lane_following_task("lf", 120).max_duration_steps == 120
    assert create_obstacle_avoidance_task((5.0, 1.0), "oa").goal_position == (15.0, 1.0)
    t = create_emergency_stop_task("es")
    assert t.name == "es" and t.goal_speed == 0.0 and t.max_duration_steps == 50
