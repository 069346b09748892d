"""Loads the in-tree sm_100a extension (``drivedit_b200/_C*.so``).

The CUDA entry points fail loudly when the extension is missing on a machine that has a
GPU: there is no silent eager fallback on the device path. CPU tensors use the PyTorch
reference implementations in :mod:`drivedit_b200.ops.reference`.
"""
from __future__ import annotations

import collections
import importlib
import os

import torch

_mod = None
_err: Exception | None = None
_checked = None


class KernelFault(RuntimeError):
    """A CUDA error or a non-zero device status word, attributed by the sync-check mode
    to the extension entry point during which (or before which) it was raised."""


def _describe(args) -> str:
    out = []
    for a in args:
        if isinstance(a, torch.Tensor):
            out.append(f"{tuple(a.shape)}:{str(a.dtype).replace('torch.', '')}")
        elif isinstance(a, (int, float, bool, str)) or a is None:
            out.append(repr(a))
        else:
            out.append(type(a).__name__)
    return ", ".join(out)


class SyncChecked:
    """The extension module with every entry point bracketed by a device synchronize and
    a read of the status word (the sync-check debug mode).

    CUDA reports a kernel fault at some later host call, so in normal runs the call that
    raises is usually not the one that launched the faulting kernel. Here each entry
    point first synchronizes (an error then belongs to earlier work: a previous entry
    point or a PyTorch op in between), runs, and synchronizes again (an error then
    belongs to the kernels this entry point launched). Either way a :class:`KernelFault`
    names the entry point, the call number and the argument shapes, with the last
    entry points called before it. With a log path every call is also appended to that
    file before it runs, so the record survives a process that aborts. Far too slow for
    measurement: the device drains after every launch."""

    # queries of host or device state that launch nothing
    _passthrough = frozenset({"read_status", "reset_status", "read_status_index", "launch_count",
                              "deterministic", "check_bounds", "set_deterministic",
                              "set_check_bounds"})

    def __init__(self, mod, log_path: str | None = None, sync=None, history: int = 16):
        self._mod = mod
        self._log_path = log_path
        self._sync_fn = sync if sync is not None else torch.cuda.synchronize
        self.calls = 0
        self.recent = collections.deque(maxlen=history)

    def __getattr__(self, name):
        obj = getattr(self._mod, name)
        if name.startswith("_") or name in self._passthrough or not callable(obj):
            return obj

        def run(*args, **kwargs):
            return self._run(name, obj, args, kwargs)

        return run

    def _check(self, where: str) -> None:
        try:
            self._sync_fn()
        except Exception as e:
            raise KernelFault(f"CUDA error {where}: {e}; entry points before it: "
                              f"{list(self.recent)}") from e
        status = int(self._mod.read_status())
        if status != 0:
            self._mod.reset_status()
            raise KernelFault(f"device status {status} {where}; entry points before it: "
                              f"{list(self.recent)}")

    def _run(self, name, fn, args, kwargs):
        self.calls += 1
        desc = f"#{self.calls} {name}({_describe(args)})"
        if self._log_path:
            with open(self._log_path, "a") as f:
                f.write(desc + "\n")
        self._check(f"before {desc}")
        out = fn(*args, **kwargs)
        self._check(f"in {desc}")
        self.recent.append(desc)
        return out


def set_sync_check(on: bool = True, log_path: str | None = None) -> None:
    """Switch the sync-check debug mode (also on when the environment variable
    ``DDB_SYNC_CHECK`` is set to anything but 0; ``DDB_SYNC_CHECK_LOG`` names a log)."""
    global _checked
    _checked = SyncChecked(_load(), log_path) if on else None


def sync_check() -> bool:
    return _checked is not None


def _load():
    global _mod, _err
    if _mod is not None:
        return _mod
    try:
        _mod = importlib.import_module("drivedit_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _err = e
        raise RuntimeError(
            "drivedit_b200 CUDA extension is not built; run `python setup.py build_ext "
            f"--inplace` (import error: {e})"
        ) from e
    if os.environ.get("DDB_SYNC_CHECK", "0") not in ("", "0"):
        set_sync_check(True, os.environ.get("DDB_SYNC_CHECK_LOG") or None)
    return _mod


def ext():
    """Return the compiled extension module (wrapped by the sync-check mode when that is
    on), raising if it cannot be imported."""
    mod = _load()
    return _checked if _checked is not None else mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def device_status() -> int:
    """Status word written by kernels whose bounded waits expired (0 = ok)."""
    return int(ext().read_status())


def reset_device_status() -> None:
    ext().reset_status()


def check_device_status() -> None:
    """Raise if any kernel on the current device reported a timeout."""
    s = device_status()
    if s != 0:
        reset_device_status()
        raise RuntimeError(f"a drivedit_b200 kernel reported device status {s}")


def use_cuda_kernels(t: torch.Tensor) -> bool:
    """True when ``t`` lives on a CUDA device (the extension must then be present)."""
    return t.is_cuda
