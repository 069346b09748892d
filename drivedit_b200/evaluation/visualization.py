"""Text reports of evaluation results (the reference's ``evaluation/visualization.py``
builds tables and summaries without a plotting library; the same here, headless):
markdown tables and metric summaries, plus the reference's visualiser classes."""
from __future__ import annotations

import math
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence

import torch


def format_table(rows: Sequence[Dict[str, Any]], columns: Sequence[str] = None, floatfmt: str = ".4g") -> str:
    rows = list(rows)
    if not rows:
        return ""
    cols = list(columns or rows[0].keys())
    fmt = lambda v: format(v, floatfmt) if isinstance(v, float) else str(v)
    cells = [[fmt(r.get(c, "")) for c in cols] for r in rows]
    w = [max(len(c), *(len(x[i]) for x in cells)) for i, c in enumerate(cols)]
    line = lambda xs: "| " + " | ".join(x.ljust(w[i]) for i, x in enumerate(xs)) + " |"
    return "\n".join([line(cols), "|" + "|".join("-" * (n + 2) for n in w) + "|"] + [line(x) for x in cells])


def summarize_metrics(metrics: Dict[str, Any], title: str = "metrics") -> str:
    flat: List[Dict[str, Any]] = []

    def walk(prefix, d):
        for k, v in d.items():
            key = f"{prefix}.{k}" if prefix else k
            if isinstance(v, dict):
                walk(key, v)
            elif isinstance(v, (int, float, bool, str)):
                flat.append({"metric": key, "value": float(v) if isinstance(v, (int, float)) and not isinstance(v, bool) else v})
            elif hasattr(v, "item") and getattr(v, "numel", lambda: 0)() == 1:
                flat.append({"metric": key, "value": float(v.item())})

    walk("", metrics)
    return f"## {title}\n\n" + format_table(flat, ["metric", "value"])


def comparison_table(results: Dict[str, Dict[str, float]], metrics: Sequence[str]) -> str:
    return format_table([{"model": name, **{m: r.get(m, float("nan")) for m in metrics}}
                         for name, r in results.items()], ["model", *metrics])


def episode_report(result) -> str:
    d = result.to_dict() if hasattr(result, "to_dict") else dict(result)
    keys = ["task_success", "task_completion_ratio", "trajectory_controllability", "average_displacement_error",
            "lateral_deviation_mean", "comfort_score", "physics_violation_ratio", "avg_inference_time_ms"]
    return format_table([{k: d[k] for k in keys if k in d}])


# --------------------------------------------------------------------------- report builders
# Class surface of the reference's evaluation/visualization.py (MetricsVisualizer :13-197,
# SequenceVisualizer :200-400, ComparisonVisualizer :403-539, create_evaluation_plots
# :542-580, create_comparison_plots :583-612): headless text reports, optionally saved
# as .txt files. Statistics are computed with batched tensor reductions.
_LOWER_IS_BETTER = ("loss", "error", "mse", "mae", "time", "latency", "lpips", "fvd", "ms")
_SPARK = "▁▂▄▆█"


def lower_is_better(metric: str) -> bool:
    """Metric-direction rule shared by every comparison: errors, losses and times."""
    m = metric.lower()
    return any(w in m for w in _LOWER_IS_BETTER)


def sparkline(values: Sequence[float]) -> str:
    """Five-level bar glyphs of values normalised to their own range."""
    if not values:
        return ""
    lo, hi = min(values), max(values)
    span = hi - lo
    return "".join(_SPARK[min(4, int(5 * (v - lo) / span)) if span > 0 else 2] for v in values)


def _flatten(d: Dict[str, Any], prefix: str = "") -> Dict[str, Any]:
    out: Dict[str, Any] = {}
    for k, v in d.items():
        key = f"{prefix}.{k}" if prefix else str(k)
        if isinstance(v, dict):
            out.update(_flatten(v, key))
        elif torch.is_tensor(v) and v.numel() == 1:
            out[key] = float(v.item())
        else:
            out[key] = v
    return out


class _Saver:
    def __init__(self, save_dir: Optional[str] = None):
        self.save_dir = Path(save_dir) if save_dir else None
        if self.save_dir:
            self.save_dir.mkdir(parents=True, exist_ok=True)

    def _emit(self, text: str, save_name: Optional[str]) -> str:
        if save_name and self.save_dir:
            (self.save_dir / f"{save_name}.txt").write_text(text)
        return text


def _title(title: str) -> List[str]:
    return ["", title, "=" * len(title)]


class MetricsVisualizer(_Saver):
    def plot_metrics_over_time(self, metrics_history: Dict[str, List[float]],
                               title: str = "Metrics Over Time",
                               save_name: Optional[str] = None) -> str:
        if not metrics_history:
            return "No metrics to plot"
        lines = _title(title)
        for name, vals in metrics_history.items():
            if vals:
                lines.append(f"{name:15} | {sparkline(vals)} | {min(vals):.3f} - {max(vals):.3f}")
        return self._emit("\n".join(lines), save_name)

    def create_metrics_table(self, metrics_dict: Dict[str, Any], title: str = "Metrics Summary",
                             save_name: Optional[str] = None) -> str:
        flat = _flatten(metrics_dict)
        w = max((len(k) for k in flat), default=0)
        fmt = lambda v: f"{v:.4f}" if isinstance(v, float) else str(v)
        lines = _title(title) + [f"{k:<{w}} | {fmt(v)}" for k, v in flat.items()]
        return self._emit("\n".join(lines), save_name)

    def create_comparison_table(self, comparison_results: Dict[str, Dict[str, float]],
                                title: str = "Model Comparison",
                                save_name: Optional[str] = None) -> str:
        if not comparison_results:
            return "No comparison data available"
        metrics = sorted({m for r in comparison_results.values() for m in r})
        rows = []
        for m in metrics:
            vals = {n: r[m] for n, r in comparison_results.items()
                    if isinstance(r.get(m), (int, float)) and not isinstance(r.get(m), bool)}
            row = {"metric": m, **{n: comparison_results[n].get(m, "N/A") for n in comparison_results}}
            if vals:
                pick = min if lower_is_better(m) else max
                row["best"] = pick(vals, key=vals.get)
            rows.append(row)
        text = "\n".join(_title(title)) + "\n" + format_table(
            rows, ["metric", *comparison_results, "best"])
        return self._emit(text, save_name)


class SequenceVisualizer(_Saver):
    """Statistics of ``[B, T, C, H, W]`` sequences (latents or frames)."""

    def analyze_sequence_statistics(self, sequences: torch.Tensor,
                                    title: str = "Sequence Analysis") -> str:
        x = sequences.detach().float()
        B, T, C, H, W = x.shape
        lines = _title(title) + [f"Shape: {list(x.shape)}", f"Data type: {sequences.dtype}",
                                 f"Device: {sequences.device}", "", "Value Statistics:",
                                 f"  Mean: {x.mean():.4f}", f"  Std:  {x.std():.4f}",
                                 f"  Min:  {x.min():.4f}", f"  Max:  {x.max():.4f}", ""]
        if T > 1:
            d = x[:, 1:] - x[:, :-1]
            lines += ["Temporal Consistency:", f"  Frame difference mean: {d.mean():.4f}",
                      f"  Frame difference std:  {d.std():.4f}", ""]
        if C > 1:
            per_c = x.transpose(0, 2).reshape(C, -1)
            lines.append("Channel Statistics:")
            lines += [f"  Channel {c}: mean={m:.4f}, std={s:.4f}"
                      for c, (m, s) in enumerate(zip(per_c.mean(1).tolist(), per_c.std(1).tolist()))]
            lines.append("")
        sm, ss = x.mean(dim=(3, 4)), x.std(dim=(3, 4))
        lines += ["Spatial Statistics (per frame):",
                  f"  Spatial mean: {sm.mean():.4f} ± {sm.std():.4f}",
                  f"  Spatial std:  {ss.mean():.4f} ± {ss.std():.4f}"]
        return "\n".join(lines)

    def create_frame_difference_analysis(self, pred_sequence: torch.Tensor,
                                         target_sequence: torch.Tensor,
                                         title: str = "Frame Difference Analysis") -> str:
        diff = (pred_sequence.detach().float() - target_sequence.detach().float()).abs()
        lines = _title(title) + ["Overall Difference Statistics:",
                                 f"  Mean Absolute Error: {diff.mean():.4f}",
                                 f"  Max Absolute Error:  {diff.max():.4f}",
                                 f"  Std of Errors:       {diff.std():.4f}", ""]
        if diff.shape[1] > 1:
            per_t = diff.mean(dim=(0, 2, 3, 4)).tolist()
            lines += ["Per-Frame Error Analysis:"] + [f"  Frame {t:2d}: {e:.4f}" for t, e in enumerate(per_t)]
            lines.append(f"  trend: {sparkline(per_t)}")
            if len(per_t) > 2:
                lines.append("Error Trend (frame-to-frame change):")
                for t in range(len(per_t) - 1):
                    ch = per_t[t + 1] - per_t[t]
                    lines.append(f"  {t}->{t + 1}: {ch:+.4f} {'↑' if ch > 0 else '↓' if ch < 0 else '→'}")
            lines.append("")
        sp = diff.mean(dim=(0, 1, 2))
        lines.append("Spatial Error Distribution (normalized):")
        H, W = sp.shape
        if H <= 16 and W <= 32:
            top = float(sp.max())
            levels = (sp / top if top > 0 else sp).mul(5).clamp(max=4).long().tolist()
            lines += ["  " + "".join(".+xX#"[v] for v in row) for row in levels]
        else:
            lines.append(f"  Spatial error range: {sp.min():.4f} - {sp.max():.4f}")
        return "\n".join(lines)

    def create_temporal_consistency_report(self, sequence: torch.Tensor,
                                           title: str = "Temporal Consistency Report") -> str:
        x = sequence.detach().float()
        T = x.shape[1]
        if T < 2:
            return f"{title}\nSequence too short for temporal analysis"
        vel = (x[:, 1:] - x[:, :-1]).abs()                     # [B, T-1, C, H, W]
        step = vel.mean(dim=(0, 2, 3, 4))                        # [T-1]
        avg = float(step.mean())
        lines = _title(title) + ["Frame-to-Frame Differences:"]
        lines += [f"  Frame {t}->{t + 1}: {d:.4f}" for t, d in enumerate(step.tolist())]
        lines += ["", "Temporal Consistency Metrics:", f"  Average frame difference: {avg:.4f}",
                  f"  Std of frame differences: {float(step.std()) if step.numel() > 1 else 0.0:.4f}",
                  f"  Consistency score:        {1.0 / (1.0 + avg):.4f}"]
        if T >= 3:
            lines += ["", "Motion Analysis:", f"  Average velocity magnitude: {avg:.4f}",
                      f"  Average acceleration:       {float((step[1:] - step[:-1]).abs().mean()):.4f}"]
        return "\n".join(lines)


class ComparisonVisualizer(_Saver):
    def create_performance_comparison(self, performance_data: Dict[str, Dict[str, float]],
                                      title: str = "Performance Comparison", width: int = 30) -> str:
        if not performance_data:
            return "No performance data available"
        lines = _title(title)
        for m in sorted({k for r in performance_data.values() for k in r}):
            vals = {n: float(r[m]) for n, r in performance_data.items()
                    if isinstance(r.get(m), (int, float)) and not isinstance(r.get(m), bool)}
            if not vals:
                continue
            lo, hi = min(vals.values()), max(vals.values())
            low_good = lower_is_better(m)
            best = min(vals, key=vals.get) if low_good else max(vals, key=vals.get)
            worst = max(vals, key=vals.get) if low_good else min(vals, key=vals.get)
            lines += ["", f"{m}:", "-" * (len(m) + 1)]
            for name, v in sorted(vals.items(), key=lambda kv: kv[1]):
                n = int(round(width * ((v - lo) / (hi - lo) if hi > lo else 0.5)))
                tag = " ★ BEST" if name == best else (" ✗ WORST" if name == worst and len(vals) > 1 else "")
                lines.append(f"  {name:15} |{'█' * n}{'░' * (width - n)}| {v:.4f}{tag}")
        return "\n".join(lines)

    def create_ablation_summary(self, ablation_results: Dict[str, Any],
                                title: str = "Ablation Study Summary") -> str:
        lines = _title(title)
        analysis = ablation_results.get("analysis")
        if not analysis:
            return "\n".join(lines + ["No analysis data available"])
        for name, per_metric in analysis.items():
            lines += ["", f"{name}:", "-" * (len(name) + 1)]
            verdicts = [a for a in per_metric.values() if isinstance(a, dict) and "improved" in a]
            for metric, a in per_metric.items():
                if isinstance(a, dict) and "improved" in a:
                    ch = a["relative_change"]
                    lines.append(f"  {metric:20} {'↑' if ch > 0 else '↓'} {ch:+.2%} "
                                 f"{'✓' if a['improved'] else '✗'}")
            if verdicts:
                good = sum(1 for a in verdicts if a["improved"])
                lines.append(f"\n  Improvement rate: {good / len(verdicts):.1%} ({good}/{len(verdicts)})")
        return "\n".join(lines)


def create_evaluation_plots(evaluation_results: Dict[str, Any],
                            save_dir: Optional[str] = None) -> Dict[str, str]:
    v = MetricsVisualizer(save_dir)
    out = {}
    if "metrics" in evaluation_results:
        out["metrics_summary"] = v.create_metrics_table(evaluation_results["metrics"],
                                                        "Evaluation Metrics Summary", "metrics_summary")
    if "performance" in evaluation_results:
        out["performance_summary"] = v.create_metrics_table(evaluation_results["performance"],
                                                            "Performance Analysis", "performance_summary")
    if "training_history" in evaluation_results:
        out["training_progress"] = v.plot_metrics_over_time(evaluation_results["training_history"],
                                                            "Training Progress", "training_progress")
    return out


def create_comparison_plots(comparison_data: Dict[str, Dict[str, Any]],
                            save_dir: Optional[str] = None) -> Dict[str, str]:
    return {"model_comparison": MetricsVisualizer(save_dir).create_comparison_table(
                comparison_data, "Model Comparison", "model_comparison"),
            "performance_comparison": ComparisonVisualizer(save_dir).create_performance_comparison(
                comparison_data, "Performance Comparison")}
