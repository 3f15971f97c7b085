"""Named timers (reference ``profiler/timer.py:11-99``).

On CUDA a timer records a pair of events on the current stream; ``stop()``
synchronises on the *end event* only (not the whole device) and returns the
device-measured interval.  On CPU it falls back to ``time.perf_counter``.
"""

from __future__ import annotations

import statistics
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

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


@dataclass
class NamedTimer:
    name: str
    device: Optional[torch.device] = None
    _samples_ms: List[float] = field(default_factory=list)
    _start_wall: Optional[float] = None
    _start_event: Optional[torch.cuda.Event] = None
    _end_event: Optional[torch.cuda.Event] = None

    def _cuda(self) -> bool:
        return self.device is not None and self.device.type == "cuda" and torch.cuda.is_available()

    def start(self) -> None:
        if self._cuda():
            self._start_event = torch.cuda.Event(enable_timing=True)
            self._end_event = torch.cuda.Event(enable_timing=True)
            self._start_event.record()
        else:
            self._start_wall = time.perf_counter()

    def stop(self) -> float:
        if self._start_event is not None and self._end_event is not None:
            self._end_event.record()
            self._end_event.synchronize()
            elapsed = float(self._start_event.elapsed_time(self._end_event))
            self._start_event = self._end_event = None
        elif self._start_wall is not None:
            elapsed = (time.perf_counter() - self._start_wall) * 1000.0
            self._start_wall = None
        else:
            raise RuntimeError("Timer.stop() called before Timer.start()")
        self._samples_ms.append(elapsed)
        return elapsed

    def add_sample(self, elapsed_ms: float) -> None:
        self._samples_ms.append(float(elapsed_ms))

    def summary(self) -> TimerSummary:
        if not self._samples_ms:
            raise RuntimeError(f"Timer '{self.name}' has no samples")
        ordered = sorted(self._samples_ms)

        def pct(p: float) -> float:
            return float(ordered[int(round((len(ordered) - 1) * p))])

        return TimerSummary(
            name=self.name,
            count=len(ordered),
            total_ms=float(sum(ordered)),
            mean_ms=float(statistics.mean(ordered)),
            p50_ms=pct(0.50),
            p95_ms=pct(0.95),
            min_ms=float(ordered[0]),
            max_ms=float(ordered[-1]),
        )


@dataclass
class TimerRegistry:
    device: Optional[torch.device] = None
    _timers: Dict[str, NamedTimer] = field(default_factory=dict)

    def timer(self, name: str) -> NamedTimer:
        if name not in self._timers:
            self._timers[name] = NamedTimer(name=name, device=self.device)
        return self._timers[name]

    def summarize(self) -> Dict[str, TimerSummary]:
        return {name: t.summary() for name, t in self._timers.items() if t._samples_ms}
