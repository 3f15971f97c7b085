"""NVTX ranges around the phases of a training step, for Nsight Systems / Nsight Compute timelines.

The reference has no NVTX markup (its tracing is the host-timed collective trace).  Here the phases
of a step (``step``, ``forward``, ``backward``, ``optimizer``, ZeRO-3 per-module gathers) can be
named on the profiler timeline.  Ranges are off unless ``ZB_NVTX=1`` or :func:`enable` is called
(``train_zero.py --nvtx``), so the hot path pays one boolean test per range when they are off.
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from typing import Iterator

import torch

_enabled = os.environ.get("ZB_NVTX", "0") not in ("", "0")


def enable(on: bool = True) -> None:
    global _enabled
    _enabled = bool(on)


def enabled() -> bool:
    return _enabled


@contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    """Push ``name`` on the NVTX range stack for the body; popped even if the body raises."""
    if not _enabled:
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def mark(name: str) -> None:
    """A single NVTX marker (an instant on the timeline)."""
    if _enabled:
        torch.cuda.nvtx.mark(name)


__all__ = ["enable", "enabled", "mark", "nvtx_range"]
