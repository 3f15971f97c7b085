from .flops import (
    FlopSnapshot,
    FlopTracker,
    estimate_transformer_train_flops,
    executed_train_flops,
    flops_to_tflops_per_second,
    peak_bf16_tflops,
    roofline_fraction,
)
from . import nvtx
from .memory import MemorySnapshot, MemoryTracker, take_memory_snapshot
from .overlap import overlap_efficiency
from .timer import NamedTimer, TimerRegistry, TimerSummary

__all__ = [
    "FlopSnapshot",
    "FlopTracker",
    "estimate_transformer_train_flops",
    "executed_train_flops",
    "flops_to_tflops_per_second",
    "peak_bf16_tflops",
    "roofline_fraction",
    "MemorySnapshot",
    "MemoryTracker",
    "take_memory_snapshot",
    "overlap_efficiency",
    "NamedTimer",
    "TimerRegistry",
    "TimerSummary",
    "nvtx",
]
