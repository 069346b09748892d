"""Evaluation: metrics, closed-loop driving evaluation with the world model as simulator,
benchmarks, evaluators and text reports."""
