from .synthetic import LatentBatch, make_batch

__all__ = ["LatentBatch", "make_batch"]
