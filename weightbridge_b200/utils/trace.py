"""NVTX ranges for the phases of a sync (visible in Nsight Systems / ncu range filters).

Ranges are pushed only when CUDA is available and ``WBRIDGE_NVTX`` is not ``0``; otherwise
``nvtx_range`` is a no-op context manager.
"""
from __future__ import annotations

import contextlib
import os

import torch

_ENABLED = None


def _enabled() -> bool:
    global _ENABLED
    if _ENABLED is None:
        _ENABLED = torch.cuda.is_available() and os.environ.get("WBRIDGE_NVTX", "1") != "0"
    return _ENABLED


@contextlib.contextmanager
def nvtx_range(name: str):
    if not _enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
