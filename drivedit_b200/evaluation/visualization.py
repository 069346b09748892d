"""Text reports of evaluation results (the reference's ``evaluation/visualization.py``
builds tables and summaries without a plotting library; the same here, headless)."""
from __future__ import annotations

from typing import Any, Dict, List, Sequence


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
