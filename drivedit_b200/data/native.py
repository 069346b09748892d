"""Loader of the native (C++) data runtime ``drivedit_b200._data``: ENFCAP capture files,
telemetry CSV parsing / control normalisation, PNG frame decoding. Built by
``python setup.py build_ext --inplace`` (no CUDA needed)."""
from __future__ import annotations

_mod = None


def native():
    global _mod
    if _mod is None:
        import torch  # noqa: F401  (loads libc10 / libtorch for the extension)

        from .. import _data

        _mod = _data
    return _mod


def available() -> bool:
    try:
        native()
        return True
    except ImportError:
        return False
