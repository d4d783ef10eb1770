"""Loader for the native extension ``ring_attention_benchmark_b200._C``.

The extension is built in place (``python setup.py build_ext --inplace``) and
holds every sm_100a kernel plus the native ring runtime.  On a machine with a
GPU a missing or stale extension is an error: no operation silently falls back
to an eager PyTorch path.
"""
from __future__ import annotations

import importlib
import os

_C = None
_ERR: Exception | None = None


def load():
    """Return the extension module, raising ImportError with the build hint."""
    global _C, _ERR
    if _C is not None:
        return _C
    try:
        import torch  # noqa: F401  (loads libtorch / libc10 the extension links against)

        _C = importlib.import_module("ring_attention_benchmark_b200._C")
    except Exception as exc:  # pragma: no cover - exercised when unbuilt
        _ERR = exc
        raise ImportError(
            "ring_attention_benchmark_b200._C is not built; run "
            "`python setup.py build_ext --inplace` in "
            f"{os.path.dirname(os.path.dirname(os.path.abspath(__file__)))} ({exc})"
        ) from exc
    return _C


def available() -> bool:
    try:
        load()
        return True
    except ImportError:
        return False
