"""NVTX ranges for timeline profilers (Nsight Systems and the like).

``nvtx_range(name)`` is a no-op unless ``QW_NVTX=1`` is set (or ``enable_nvtx()`` is called), so the instrumentation
in the trainer and the benchmark costs nothing in normal runs. The trainer marks ``forward``, ``backward``,
``grad_sync`` (gradient reduction and clipping) and ``optimizer`` for every step; ``bench.py --trace`` adds a chrome
trace of one step through the torch profiler.
"""

from __future__ import annotations

import contextlib
import os

import torch

_enabled = os.environ.get("QW_NVTX", "0") == "1"


def enable_nvtx(on: bool = True) -> None:
    global _enabled
    _enabled = on


def nvtx_enabled() -> bool:
    return _enabled and torch.cuda.is_available()


@contextlib.contextmanager
def nvtx_range(name: str):
    if not nvtx_enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
