"""Loader for the native extensions.

``_C`` holds the sm_100a kernels; ``_native`` the CPU runtime. On a machine
with a CUDA device, a missing or broken ``_C`` is an error (raised on first
use of a GPU op), never a silent fallback to eager PyTorch.
"""
from __future__ import annotations

import importlib

_C = None
_C_ERR: Exception | None = None
_native = None
_NATIVE_ERR: Exception | None = None

try:
    _C = importlib.import_module("flodl_b200._C")
except Exception as e:  # pragma: no cover - reported by cuda_ext()
    _C_ERR = e

try:
    _native = importlib.import_module("flodl_b200._native")
except Exception as e:  # pragma: no cover
    _NATIVE_ERR = e


def cuda_ext():
    """Return the compiled kernel module or raise with build instructions."""
    if _C is None:
        raise RuntimeError(
            "flodl_b200._C (sm_100a kernels) is not built or failed to load: "
            f"{_C_ERR!r}. Run `python setup.py build_ext --inplace`."
        )
    return _C


def native():
    """Return the native runtime module or raise."""
    if _native is None:
        raise RuntimeError(
            "flodl_b200._native failed to load: "
            f"{_NATIVE_ERR!r}. Run `python setup.py build_ext --inplace`."
        )
    return _native
