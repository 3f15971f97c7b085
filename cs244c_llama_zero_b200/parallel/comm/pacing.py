"""Device-paced link emulation for the NVLink collectives (the harness's ``nvlink`` bandwidth mode).

The reference emulates slow interconnects three ways, all outside the GPU: a host ``sleep`` after
each collective (``ZERO_SIM_BW_GBPS``, ``collectives/interface.py:340-356``), an ``LD_PRELOAD``
token bucket on NCCL's sockets (``infra/socket_shaper.c``) and ``tc``.  None of them touches this
package's NVLink kernels, which move data by peer loads/stores and copy engines, not sockets.

Here the pacing runs on the device timeline instead.  Around every NVLink collective (and every
ZeRO-3 copy-engine gather) the runtime enqueues two one-thread kernels on the same stream: the
first stamps ``%globaltimer``; the second books this GPU's emulated link for the transfer's cost,
starting at the later of the stamp and the time the link frees up, and holds the stream until the
booking ends.  So a transfer takes ``max(its NVLink time, its cost on the emulated link)``, the host
is never blocked (enqueue stays asynchronous, unlike the ``sleep`` mode), and transfers issued on
several streams (the compute stream's reduce-scatter and the side stream's prefetching gathers)
queue on one link, as they would on a real NIC.

Cost model: the bytes that cross one GPU's link under a ring schedule of the collective (all-reduce
``2 (W-1)/W N``; reduce-scatter and all-gather ``(W-1)/W N`` of the full buffer ``N``), at
``ZERO_NVLINK_BW_GBPS`` Gbit/s (bits, like the ``socket`` and ``tc`` modes), plus
``ZERO_NVLINK_LATENCY_MS`` per transfer.  Collectives that still go through NCCL (scalar
all-reduces, the initial broadcast) are not paced.
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import torch

ENV_BW = "ZERO_NVLINK_BW_GBPS"
ENV_LATENCY = "ZERO_NVLINK_LATENCY_MS"

RING_FACTOR = {"allreduce": 2, "reduce_scatter": 1, "allgather": 1}


def pacing_from_env(env=None) -> Optional[Tuple[float, float]]:
    """(Gbit/s, latency ms) when either variable asks for pacing, else None."""
    env = os.environ if env is None else env
    bw = float(env.get(ENV_BW, "") or 0.0)
    lat = float(env.get(ENV_LATENCY, "") or 0.0)
    if bw <= 0 and lat <= 0:
        return None
    return bw, lat


def link_bytes(op: str, full_bytes: int, world: int) -> int:
    """Bytes one GPU sends over its link for ``op`` on a ``full_bytes`` buffer (ring schedule)."""
    if world <= 1:
        return 0
    return RING_FACTOR[op] * (world - 1) * int(full_bytes) // world


def pace_cost_ns(nbytes: int, gbps: float, latency_ms: float) -> int:
    """ns on a ``gbps`` Gbit/s link plus the latency (the formula the native pacer uses)."""
    ns = latency_ms * 1e6 if latency_ms > 0 else 0.0
    if gbps > 0:
        ns += 8.0 * nbytes / gbps
    return int(round(ns))


def make_pacer(device: torch.device, timeout_ns: int, env=None):
    """The native ``LinkPacer`` of ``device`` when the environment asks for pacing, else None."""
    cfg = pacing_from_env(env)
    if cfg is None:
        return None
    from ... import ops

    index = device.index if device.index is not None else torch.cuda.current_device()
    return ops.load_extension().LinkPacer(index, cfg[0], cfg[1], int(timeout_ns))


__all__ = ["ENV_BW", "ENV_LATENCY", "link_bytes", "make_pacer", "pace_cost_ns", "pacing_from_env"]
