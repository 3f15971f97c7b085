"""Labelled memory snapshots of the host process and the CUDA caching allocator.

Record format as in the reference (``profiler/memory.py:12-99``): each snapshot carries ``label``,
``timestamp_s``, ``host_maxrss_mb`` and the allocator's current / peak allocated and reserved MiB, and
``MemoryTracker.as_dicts()`` lists them in recording order (the profile JSON's ``memory`` list).

Design here: one ``_probe`` function reads every counter at once into a ``MemorySnapshot``; on a
device without CUDA the allocator fields are zero.  The host peak RSS comes from ``getrusage``, whose
unit is kibibytes on Linux and bytes on macOS.
"""

from __future__ import annotations

import resource
import sys
import time
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

import torch

MIB = float(1 << 20)
# getrusage().ru_maxrss unit in bytes, by platform
_RSS_UNIT_BYTES = 1.0 if sys.platform == "darwin" else 1024.0


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


def _is_cuda(device: Optional[torch.device]) -> bool:
    return device is not None and device.type == "cuda" and torch.cuda.is_available()


def _allocator_mib(device: Optional[torch.device]) -> Dict[str, float]:
    if not _is_cuda(device):
        return dict(cuda_allocated_mb=0.0, cuda_reserved_mb=0.0, cuda_max_allocated_mb=0.0, cuda_max_reserved_mb=0.0)
    return dict(
        cuda_allocated_mb=torch.cuda.memory_allocated(device) / MIB,
        cuda_reserved_mb=torch.cuda.memory_reserved(device) / MIB,
        cuda_max_allocated_mb=torch.cuda.max_memory_allocated(device) / MIB,
        cuda_max_reserved_mb=torch.cuda.max_memory_reserved(device) / MIB,
    )


def take_memory_snapshot(label: str, device: Optional[torch.device] = None) -> MemorySnapshot:
    rss_mib = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss * _RSS_UNIT_BYTES / MIB
    return MemorySnapshot(label=label, timestamp_s=time.time(), host_maxrss_mb=rss_mib, **_allocator_mib(device))


@dataclass
class MemoryTracker:
    """Keeps the snapshots of one process; each ``record`` first waits for the device's queued work."""

    device: Optional[torch.device] = None
    snapshots: List[MemorySnapshot] = field(default_factory=list)

    def synchronize(self) -> None:
        if _is_cuda(self.device):
            torch.cuda.synchronize(self.device)

    def record(self, label: str) -> MemorySnapshot:
        self.synchronize()
        snap = take_memory_snapshot(label, self.device)
        self.snapshots.append(snap)
        return snap

    def reset_peak_stats(self) -> None:
        if _is_cuda(self.device):
            self.synchronize()
            torch.cuda.reset_peak_memory_stats(self.device)

    def peak_stats_mb(self) -> Dict[str, float]:
        self.synchronize()
        counters = _allocator_mib(self.device)
        return {"peak_allocated_mb": counters["cuda_max_allocated_mb"],
                "peak_reserved_mb": counters["cuda_max_reserved_mb"]}

    def as_dicts(self) -> List[Dict[str, float | str]]:
        return list(map(MemorySnapshot.to_dict, self.snapshots))
