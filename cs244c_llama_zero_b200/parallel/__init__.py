"""Data parallelism: collectives (ring / NCCL / NVLink kernels) and the ZeRO 0-3 engines."""

from .collectives import (
    CollectiveOps,
    LocalCollectives,
    SendRecvCollectives,
    TorchCollectives,
    TracingCollectives,
    aggregate_collective_trace,
    pick_collectives,
)
from .ring import ring_allgather, ring_allreduce, ring_reduce_scatter

__all__ = [
    "CollectiveOps",
    "LocalCollectives",
    "SendRecvCollectives",
    "TorchCollectives",
    "TracingCollectives",
    "aggregate_collective_trace",
    "pick_collectives",
    "ring_allgather",
    "ring_allreduce",
    "ring_reduce_scatter",
]
