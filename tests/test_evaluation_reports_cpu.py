"""Evaluation report builders and the comparison / ablation evaluators on the tiny
preset (CPU)."""
import torch

from drivedit_b200.config import get_config
from drivedit_b200.evaluation.evaluators import (AblationEvaluator, ComparisonEvaluator,
                                                 RealTimeEvaluator)
from drivedit_b200.evaluation.visualization import (ComparisonVisualizer, MetricsVisualizer,
                                                    SequenceVisualizer, create_comparison_plots,
                                                    create_evaluation_plots, lower_is_better,
                                                    sparkline)
from drivedit_b200.models.world_dit import WorldDiT


def _model(**over):
    cfg = get_config("tiny", [f"model.{k}={v}" for k, v in over.items()])
    torch.manual_seed(0)
    return WorldDiT(cfg.model).eval(), cfg


def _batches(cfg, n=1):
    m = cfg.model
    g = torch.Generator().manual_seed(1)
    return [{"latents": torch.randn(1, 4, m.latent_channels, m.latent_h, m.latent_w, generator=g),
             "actions": torch.rand(1, 4, m.action_dim, generator=g)} for _ in range(n)]


def test_visualizers_render_and_save(tmp_path):
    mv = MetricsVisualizer(str(tmp_path))
    txt = mv.plot_metrics_over_time({"loss": [3.0, 2.0, 1.0], "acc": [0.1, 0.5, 0.9]},
                                    save_name="hist")
    assert "█" in txt and (tmp_path / "hist.txt").exists()
    assert sparkline([0, 1, 2, 3, 4]) == "▁▂▄▆█"
    tab = mv.create_comparison_table({"a": {"mse": 0.1, "psnr": 30.0}, "b": {"mse": 0.2, "psnr": 31.0}})
    rows = {ln.split("|")[1].strip(): ln for ln in tab.splitlines() if ln.startswith("| ")}
    assert rows["mse"].rstrip(" |").endswith("a") and rows["psnr"].rstrip(" |").endswith("b")
    assert lower_is_better("val_loss") and not lower_is_better("psnr")
    seq = torch.randn(2, 5, 3, 8, 8)
    sv = SequenceVisualizer()
    assert "Channel 2" in sv.analyze_sequence_statistics(seq)
    fd = sv.create_frame_difference_analysis(seq, seq + 0.1)
    assert "Mean Absolute Error: 0.1000" in fd and "#" in fd
    assert "Consistency score" in sv.create_temporal_consistency_report(seq)
    cv = ComparisonVisualizer()
    perf = cv.create_performance_comparison({"x": {"latency_ms": 5.0}, "y": {"latency_ms": 9.0}})
    assert "x" in perf.split("★")[0].splitlines()[-1]
    plots = create_evaluation_plots({"metrics": {"a": {"b": 1.0}}, "training_history": {"l": [1, 2]}})
    assert set(plots) == {"metrics_summary", "training_progress"}
    assert set(create_comparison_plots({"m": {"mse": 1.0}})) == {"model_comparison",
                                                               "performance_comparison"}


def test_comparison_and_ablation_evaluators():
    base, cfg = _model()
    other, _ = _model(n_layers=2)
    data = _batches(cfg)
    cmp = ComparisonEvaluator({"four": base, "two": other}, device="cpu", context_frames=2,
                              flow_steps=1).compare_models(data)
    assert set(cmp["individual_results"]) == {"four", "two"}
    assert cmp["comparison_summary"]["mse"]["best_model"] in ("four", "two")
    abl = AblationEvaluator(base, device="cpu", context_frames=2, flow_steps=1)
    res = abl.evaluate_component_ablation(data, [{"name": "shallow", "overrides": {"n_layers": 2}}])
    a = res["analysis"]["shallow"]["mse"]
    assert set(a) == {"absolute_change", "relative_change", "improved"}
    txt = ComparisonVisualizer().create_ablation_summary(res)
    assert "Improvement rate" in txt
    # shared weights were copied into the ablated model
    m2 = abl._create_ablated_model({"overrides": {"n_layers": 2}})
    k = next(n for n, _ in m2.named_parameters() if n.startswith("blocks.0"))
    assert torch.equal(dict(m2.named_parameters())[k], dict(base.named_parameters())[k])


def test_streaming_performance_cpu():
    model, _ = _model()
    r = RealTimeEvaluator(model, device="cpu").evaluate_streaming_performance(
        total_duration_s=0.3, chunk_frames=2, source_fps=20, flow_steps=1)
    assert r["total_chunks"] == 3 and r["real_time_factor"] > 0
