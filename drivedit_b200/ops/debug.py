"""Debug switches of the sm_100a kernels (substitutes for a race detector and a memory
checker, which this framework does not rely on):

``deterministic``
    Reductions whose rounding would depend on thread timing run in a fixed order: the
    MoE dispatch places the routes to each expert in (token, route) order with a stable
    counting sort instead of by atomic arrival, the router's per-expert probability sums
    use a fixed-order reduction instead of float atomics, and fp32-accumulating GEMMs
    (weight gradients) run without split-K, so each output element has one writer. The
    MoE layer's forward and all its gradients then repeat bit for bit from run to run.
    Not covered: the attention backward's dQ, which CTAs of different key tiles add with
    TMA reductions (correct, but its last bits vary between runs).
``check_bounds``
    The MoE dispatch / combine / un-permute kernels check every table-derived index
    (expert ids, row slots) against the extent of the buffer it addresses; the first bad
    index is recorded in the device status word (code 6, the index in word 1) and the
    access is skipped, so a corrupt routing table shows up as an error instead of a
    memory fault. :func:`drivedit_b200.ops._ext.check_device_status` raises on it.

``sync_check``
    Every extension entry point is bracketed by a device synchronize and a read of the
    status word, so an asynchronous kernel fault (or an expired bounded wait) is raised
    as a :class:`~drivedit_b200.ops._ext.KernelFault` naming the entry point that launched
    it (or, when raised before it, the work in between), with the entry points called
    just before. ``DDB_SYNC_CHECK=1`` turns it on for a whole run (``bench.py``, the
    tests), ``DDB_SYNC_CHECK_LOG=<file>`` also appends every call to a file before it
    runs. For locating a fault, not for timing; not usable inside CUDA-graph capture.

All are process-wide and off by default.
"""
from __future__ import annotations

from contextlib import contextmanager

from ._ext import KernelFault, ext, set_sync_check, sync_check  # noqa: F401

BAD_INDEX_STATUS = 6


def set_deterministic(on: bool = True) -> None:
    ext().set_deterministic(bool(on))


def is_deterministic() -> bool:
    return bool(ext().deterministic())


def set_check_bounds(on: bool = True) -> None:
    ext().set_check_bounds(bool(on))


def is_checking_bounds() -> bool:
    return bool(ext().check_bounds())


def bad_index() -> int:
    """The index recorded with the last bad-index status."""
    return int(ext().read_status_index())


@contextmanager
def deterministic(on: bool = True):
    prev = is_deterministic()
    set_deterministic(on)
    try:
        yield
    finally:
        set_deterministic(prev)


@contextmanager
def check_bounds(on: bool = True):
    prev = is_checking_bounds()
    set_check_bounds(on)
    try:
        yield
    finally:
        set_check_bounds(prev)
