"""Named interval timers for the training step's phases.

Public surface as in the reference (``profiler/timer.py:11-99``): ``TimerRegistry(device).timer(name)``
hands out a ``NamedTimer`` with ``start()`` / ``stop() -> ms`` / ``summary() -> TimerSummary``, and
``TimerRegistry.summarize()`` maps every timer that has samples to its summary.

Design here: the *clock* is a separate object chosen once per timer.  ``_DeviceClock`` brackets the
interval with two CUDA events on the current stream and, at ``stop``, waits for the end event only,
so other streams (collective prefetch, copy engines) keep running; ``_HostClock`` uses
``time.perf_counter``.  Samples are kept as an ``array('d')`` and summarised with linearly
interpolated percentiles.
"""

from __future__ import annotations

import math
import time
from array import array
from dataclasses import dataclass
from typing import Dict, Iterable, Optional, Tuple

import torch


@dataclass
class TimerSummary:
    name: str
    count: int
    total_ms: float
    mean_ms: float
    p50_ms: float
    p95_ms: float
    min_ms: float
    max_ms: float


def _percentile(ordered: Tuple[float, ...], q: float) -> float:
    """Percentile of sorted samples by linear interpolation between the two nearest ranks."""
    pos = q * (len(ordered) - 1)
    lo = math.floor(pos)
    hi = min(lo + 1, len(ordered) - 1)
    frac = pos - lo
    return ordered[lo] + (ordered[hi] - ordered[lo]) * frac


def summarize_samples(name: str, samples_ms: Iterable[float]) -> TimerSummary:
    ordered = tuple(sorted(float(s) for s in samples_ms))
    if not ordered:
        raise RuntimeError(f"Timer '{name}' has no samples")
    total = math.fsum(ordered)
    return TimerSummary(name=name, count=len(ordered), total_ms=total, mean_ms=total / len(ordered),
                        p50_ms=_percentile(ordered, 0.50), p95_ms=_percentile(ordered, 0.95),
                        min_ms=ordered[0], max_ms=ordered[-1])


class _HostClock:
    def begin(self):
        return time.perf_counter()

    def end(self, token) -> float:
        return (time.perf_counter() - token) * 1e3


class _DeviceClock:
    def begin(self):
        pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        pair[0].record()
        return pair

    def end(self, token) -> float:
        first, last = token
        last.record()
        last.synchronize()
        return float(first.elapsed_time(last))


def _clock_for(device: Optional[torch.device]):
    if device is not None and device.type == "cuda" and torch.cuda.is_available():
        return _DeviceClock()
    return _HostClock()


class NamedTimer:
    """One named interval timer; every ``start()``/``stop()`` pair adds one sample in milliseconds."""

    def __init__(self, name: str, device: Optional[torch.device] = None) -> None:
        self.name = name
        self.device = device
        self._clock = _clock_for(device)
        self._open = None
        self._samples = array("d")

    @property
    def count(self) -> int:
        return len(self._samples)

    @property
    def samples_ms(self) -> Tuple[float, ...]:
        return tuple(self._samples)

    def start(self) -> None:
        self._open = self._clock.begin()

    def stop(self) -> float:
        if self._open is None:
            raise RuntimeError(f"timer '{self.name}': stop() without a matching start()")
        token, self._open = self._open, None
        ms = self._clock.end(token)
        self._samples.append(ms)
        return ms

    def add_sample(self, elapsed_ms: float) -> None:
        """Record an interval measured elsewhere (e.g. device-side stamps)."""
        self._samples.append(float(elapsed_ms))

    def summary(self) -> TimerSummary:
        return summarize_samples(self.name, self._samples)


class TimerRegistry:
    """The process's timers by name, created on first use."""

    def __init__(self, device: Optional[torch.device] = None) -> None:
        self.device = device
        self._by_name: Dict[str, NamedTimer] = {}

    def timer(self, name: str) -> NamedTimer:
        found = self._by_name.get(name)
        if found is None:
            found = self._by_name[name] = NamedTimer(name, self.device)
        return found

    def summarize(self) -> Dict[str, TimerSummary]:
        return {name: t.summary() for name, t in self._by_name.items() if t.count}
