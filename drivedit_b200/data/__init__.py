"""Data layer: synthetic workloads, native ENFCAP / telemetry / frame loaders, the
Enfusion session dataset, memory-mapped video pipelines, transforms, collators and
samplers."""
from .synthetic import LatentBatch, make_batch

__all__ = ["LatentBatch", "make_batch"]
