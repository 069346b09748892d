"""Step schedules for loss weights and annealing factors.

One small piecewise-schedule object serves every weight that changes with the training
step: the VAE's KL weight (constant, linear warm-up, cyclical), the REPA weight under
HASTE (ramp in, hold, switch off) and anything else that needs a ramp. A schedule is a
list of segments, each ``steps`` long (``None``: open-ended), moving from ``start`` to
``end`` along a shape; an optional period repeats the segment list.

Shapes (``p`` is the progress through the segment, 0 at its first step):
``linear`` p; ``cosine`` (1 - cos(pi p)) / 2 (the half-cosine ramp of SGDR-style
schedules, Loshchilov & Hutter 2017); ``step`` 0 inside the segment, the end value once
it is over; ``constant`` the end value throughout.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

SHAPES = ("linear", "cosine", "step", "constant")


def ramp(progress: float, shape: str) -> float:
    """Fraction of the way from a segment's start value to its end value."""
    p = min(max(progress, 0.0), 1.0)
    if shape == "linear":
        return p
    if shape == "cosine":
        return 0.5 * (1.0 - math.cos(math.pi * p))
    if shape == "step":
        return 1.0 if p >= 1.0 else 0.0
    if shape == "constant":
        return 1.0
    raise ValueError(f"unknown schedule shape {shape!r}; choose from {SHAPES}")


@dataclass
class Segment:
    steps: Optional[int]           # None: lasts forever
    start: float
    end: float
    shape: str = "linear"
    name: str = ""


class PiecewiseSchedule:
    """value(step) over a list of segments; ``period`` repeats them (cyclical schedules)."""

    def __init__(self, segments: Sequence[Segment], period: Optional[int] = None):
        if not segments:
            raise ValueError("a schedule needs at least one segment")
        for s in segments[:-1]:
            if s.steps is None:
                raise ValueError("only the last segment may be open-ended")
        self.segments: List[Segment] = list(segments)
        self.period = period
        self.origin = 0          # step at which the schedule (re)starts

    def restart(self, step: int) -> None:
        """Start the schedule over at ``step`` (a warm restart)."""
        self.origin = step

    def locate(self, step: int) -> Tuple[int, float]:
        """(segment index, progress through it) at ``step``."""
        s = step - self.origin
        if self.period:
            s %= self.period
        s = max(s, 0)
        for i, seg in enumerate(self.segments):
            if seg.steps is None or s < seg.steps:
                return i, (s / seg.steps if seg.steps else 0.0)
            s -= seg.steps
        # past the last bounded segment: hold its end value
        return len(self.segments) - 1, 1.0

    def __call__(self, step: int) -> float:
        i, p = self.locate(step)
        seg = self.segments[i]
        if seg.steps is None and seg.shape != "constant":
            return seg.end
        return seg.start + (seg.end - seg.start) * ramp(p, seg.shape)

    def phase(self, step: int) -> str:
        i, _ = self.locate(step)
        return self.segments[i].name or str(i)
