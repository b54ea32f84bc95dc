"""Hand-written sm_100a kernels and their autograd wrappers.

The compiled extension ``quantaweave_b200._C`` is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``). Each wrapper module exposes the CUDA path; the CPU path of every layer is plain
PyTorch and lives in ``quantaweave_b200.models``. On a CUDA tensor a missing extension is an error, never a
silent fallback.
"""

from __future__ import annotations

import importlib
import os

_ext = None
_error: Exception | None = None


def _load():
    global _ext, _error
    if _ext is not None or _error is not None:
        return _ext
    try:
        _ext = importlib.import_module("quantaweave_b200._C")
    except Exception as exc:  # noqa: BLE001 - reported by native_required()
        _error = exc
    return _ext


def native_available() -> bool:
    return _load() is not None


def native_required():
    """The compiled extension, or a RuntimeError saying how to build it."""
    ext = _load()
    if ext is None:
        raise RuntimeError(
            "quantaweave_b200._C is not built (run `python setup.py build_ext --inplace`); "
            f"CUDA tensors need the native kernels: {_error!r}"
        )
    return ext


def ext():
    return native_required()


def debug_bounds() -> bool:
    return os.environ.get("QW_DEBUG_BOUNDS", "0") == "1"
