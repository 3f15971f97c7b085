"""Labelled memory snapshots (reference ``profiler/memory.py:12-99``)."""

from __future__ import annotations

import resource
import sys
import time
from dataclasses import asdict, dataclass
from typing import Dict, List, Optional

import torch

_MB = 1024.0 * 1024.0


@dataclass
class MemorySnapshot:
    label: str
    timestamp_s: float
    host_maxrss_mb: float
    cuda_allocated_mb: float
    cuda_reserved_mb: float
    cuda_max_allocated_mb: float
    cuda_max_reserved_mb: float

    def to_dict(self) -> Dict[str, float | str]:
        return asdict(self)


def _host_maxrss_mb() -> float:
    raw = float(resource.getrusage(resource.RUSAGE_SELF).ru_maxrss)
    return raw / _MB if sys.platform == "darwin" else raw / 1024.0


def _cuda_device(device: Optional[torch.device]) -> bool:
    return device is not None and device.type == "cuda" and torch.cuda.is_available()


def take_memory_snapshot(label: str, device: Optional[torch.device] = None) -> MemorySnapshot:
    if _cuda_device(device):
        stats = (
            torch.cuda.memory_allocated(device) / _MB,
            torch.cuda.memory_reserved(device) / _MB,
            torch.cuda.max_memory_allocated(device) / _MB,
            torch.cuda.max_memory_reserved(device) / _MB,
        )
    else:
        stats = (0.0, 0.0, 0.0, 0.0)
    return MemorySnapshot(label, time.time(), _host_maxrss_mb(), *stats)


@dataclass
class MemoryTracker:
    device: Optional[torch.device] = None
    snapshots: List[MemorySnapshot] = None

    def __post_init__(self) -> None:
        if self.snapshots is None:
            self.snapshots = []

    def record(self, label: str) -> MemorySnapshot:
        self.synchronize()
        snap = take_memory_snapshot(label=label, device=self.device)
        self.snapshots.append(snap)
        return snap

    def synchronize(self) -> None:
        if _cuda_device(self.device):
            torch.cuda.synchronize(self.device)

    def reset_peak_stats(self) -> None:
        if _cuda_device(self.device):
            self.synchronize()
            torch.cuda.reset_peak_memory_stats(self.device)

    def peak_stats_mb(self) -> Dict[str, float]:
        if not _cuda_device(self.device):
            return {"peak_allocated_mb": 0.0, "peak_reserved_mb": 0.0}
        self.synchronize()
        return {
            "peak_allocated_mb": torch.cuda.max_memory_allocated(self.device) / _MB,
            "peak_reserved_mb": torch.cuda.max_memory_reserved(self.device) / _MB,
        }

    def as_dicts(self) -> List[Dict[str, float | str]]:
        return [s.to_dict() for s in self.snapshots]
