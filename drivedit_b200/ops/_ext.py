"""Loads the in-tree sm_100a extension (``drivedit_b200/_C*.so``).

The CUDA entry points fail loudly when the extension is missing on a machine that has a
GPU: there is no silent eager fallback on the device path. CPU tensors use the PyTorch
reference implementations in :mod:`drivedit_b200.ops.reference`.
"""
from __future__ import annotations

import importlib

import torch

_mod = None
_err: Exception | None = None


def ext():
    """Return the compiled extension module, raising if it cannot be imported."""
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
    return _mod


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
