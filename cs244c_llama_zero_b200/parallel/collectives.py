"""Collective-operations interface consumed by the ZeRO engines.

API parity with the reference's ``collectives/interface.py:30-356``:

* ``allreduce(t, average)`` returns a new tensor; ``allreduce_inplace`` reduces in place,
* ``reduce_scatter(t)`` returns this rank's flat shard of the sum (``ceil(n/W)`` chunks,
  the last one trimmed),
* ``allgather(shard)`` returns the flat concatenation of all ranks' shards,
* ``label_scope(label)`` and ``consume_trace()`` for tracing.

Implementations: ``LocalCollectives`` (world 1), ``SendRecvCollectives`` (the gloo ring,
``impl="ring"``), ``TorchCollectives`` (NCCL/Gloo built-ins, ``impl="torch"``) and
``TracingCollectives``.  The NVLink symmetric-memory implementation (``impl="nvls"``)
lives in :mod:`cs244c_llama_zero_b200.parallel.comm.nvlink`.

Differences from the reference, all additive: ``allgather`` accepts ``sizes=`` so the
engines (whose shard sizes are static) skip the per-call size exchange and its host
sync; ``reduce_scatter``/``allgather`` accept ``out=`` buffers; tracing records device
time when the inner implementation reports it.
"""

from __future__ import annotations

import os
import time
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Dict, Iterator, List, Optional, Sequence

import torch
import torch.distributed as dist

from .ring import ring_allgather, ring_allreduce, ring_reduce_scatter, simulated_link_delay_s


def simulated_collective_delay_s(num_bytes: int, world_size: int) -> float:
    """``(W-1) * bytes / (BW * 1e9) + latency`` from ``ZERO_SIM_BW_GBPS`` / ``ZERO_SIM_LATENCY_MS``."""
    bw = os.environ.get("ZERO_SIM_BW_GBPS", "").strip()
    lat = os.environ.get("ZERO_SIM_LATENCY_MS", "").strip()
    delay = 0.0
    if bw and float(bw) > 0:
        delay += ((world_size - 1) * num_bytes) / (float(bw) * 1e9)
    if lat and float(lat) > 0:
        delay += float(lat) / 1000.0
    return delay


def _maybe_simulate_collective_delay(num_bytes: int, world_size: int) -> None:
    delay = simulated_collective_delay_s(num_bytes, world_size)
    if delay > 0:
        time.sleep(delay)


def _world() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


@dataclass
class CollectiveOps:
    """Black-box communication interface consumed by the ZeRO engines."""

    name = "base"

    def allreduce(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        raise NotImplementedError

    def allreduce_inplace(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        reduced = self.allreduce(tensor, average=average)
        if reduced.data_ptr() != tensor.data_ptr():
            tensor.copy_(reduced)
        return tensor

    def reduce_scatter(self, tensor: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def allgather(self, local_shard: torch.Tensor, sizes: Optional[Sequence[int]] = None) -> torch.Tensor:
        raise NotImplementedError

    # ---- buffer-oriented entry points used by the ZeRO engines -----------------------
    # Implementations that own device kernels override these to fuse the arithmetic
    # into the collective; the defaults compose the basic operations above.
    supports_fused = False

    def allreduce_scaled_(self, flat: torch.Tensor, scale: float) -> torch.Tensor:
        """``flat = scale * sum_ranks(flat)`` in place."""
        self.allreduce_inplace(flat, average=False)
        if scale != 1.0:
            flat.mul_(scale)
        return flat

    def reduce_scatter_into(self, out: torch.Tensor, flat: torch.Tensor) -> torch.Tensor:
        """``out`` (length ``flat.numel() // W``) = this rank's chunk of the sum."""
        shard = self.reduce_scatter(flat)
        out[: shard.numel()].copy_(shard)
        return out

    def reduce_scatter_accumulate_(self, acc: torch.Tensor, flat: torch.Tensor, scale: float) -> torch.Tensor:
        """``acc += scale * chunk_rank(sum_ranks(flat))``; ``acc`` is fp32."""
        shard = self.reduce_scatter(flat)
        acc[: shard.numel()].add_(shard.to(acc.dtype), alpha=scale)
        return acc

    def allgather_into(self, out: torch.Tensor, shard: torch.Tensor) -> torch.Tensor:
        """``out`` = concatenation of every rank's equally sized ``shard``."""
        world = _world()
        out.copy_(self.allgather(shard, sizes=[shard.numel()] * world))
        return out

    @contextmanager
    def label_scope(self, label: str) -> Iterator[None]:
        del label
        yield

    def consume_trace(self) -> List[Dict[str, object]]:
        return []


@dataclass
class LocalCollectives(CollectiveOps):
    """Single-process fallback: identity (copies)."""

    name = "local"

    def allreduce(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        return tensor.clone()

    def allreduce_inplace(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        return tensor

    def reduce_scatter(self, tensor: torch.Tensor) -> torch.Tensor:
        return tensor.contiguous().view(-1).clone()

    def allgather(self, local_shard: torch.Tensor, sizes: Optional[Sequence[int]] = None) -> torch.Tensor:
        return local_shard.contiguous().view(-1).clone()


def _refuse_ring_on_nccl(tensor: torch.Tensor) -> None:
    if not (dist.is_available() and dist.is_initialized()) or tensor.device.type != "cuda":
        return
    if dist.get_backend() == "nccl":
        raise RuntimeError(
            "SendRecvCollectives uses point-to-point isend/irecv rings, which are a CPU/Gloo "
            "correctness oracle here. Use --collective-impl torch or nvls for CUDA tensors."
        )


@dataclass
class SendRecvCollectives(CollectiveOps):
    """Ring collectives from explicit send/recv (``--collective-impl ring``)."""

    name = "ring"

    def allreduce(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        _refuse_ring_on_nccl(tensor)
        return ring_allreduce(tensor=tensor, average=average)

    def reduce_scatter(self, tensor: torch.Tensor) -> torch.Tensor:
        _refuse_ring_on_nccl(tensor)
        return ring_reduce_scatter(tensor=tensor)

    def allgather(self, local_shard: torch.Tensor, sizes: Optional[Sequence[int]] = None) -> torch.Tensor:
        _refuse_ring_on_nccl(local_shard)
        return ring_allgather(local_shard=local_shard, sizes=sizes)


@dataclass
class TorchCollectives(CollectiveOps):
    """NCCL (GPU) or Gloo (CPU) built-in collectives (``--collective-impl torch``)."""

    name = "torch"

    @staticmethod
    def _fast(tensor: torch.Tensor) -> bool:
        return tensor.device.type == "cuda"

    @staticmethod
    def _maybe_synchronize(tensor: torch.Tensor) -> None:
        if tensor.device.type == "cuda" and os.environ.get("ZERO_COLLECTIVE_CUDA_SYNC", "0") == "1":
            torch.cuda.synchronize(tensor.device)

    def allreduce(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        return self.allreduce_inplace(tensor.clone(), average=average)

    def allreduce_inplace(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        dist.all_reduce(tensor)
        _maybe_simulate_collective_delay(tensor.numel() * tensor.element_size(), _world())
        self._maybe_synchronize(tensor)
        if average:
            tensor /= _world()
        return tensor

    def reduce_scatter(self, tensor: torch.Tensor) -> torch.Tensor:
        world, rank = _world(), _rank()
        flat = tensor.contiguous().view(-1)
        if flat.numel() == 0:
            return flat.clone()
        chunk = (flat.numel() + world - 1) // world
        start = rank * chunk
        keep = max(0, min(start + chunk, flat.numel()) - start)
        if self._fast(flat):
            padded = flat
            if chunk * world != flat.numel():
                padded = torch.zeros(chunk * world, dtype=flat.dtype, device=flat.device)
                padded[: flat.numel()] = flat
            out = torch.empty(chunk, dtype=flat.dtype, device=flat.device)
            dist.reduce_scatter_tensor(out, padded)
            _maybe_simulate_collective_delay(out.numel() * out.element_size(), world)
            self._maybe_synchronize(out)
            return out[:keep]
        # Gloo has no reduce-scatter: all-reduce and slice.
        reduced = flat.clone()
        dist.all_reduce(reduced)
        _maybe_simulate_collective_delay(reduced.numel() * reduced.element_size(), world)
        return reduced[start : start + keep].contiguous()

    def reduce_scatter_into(self, out: torch.Tensor, flat: torch.Tensor) -> torch.Tensor:
        if self._fast(flat) and flat.numel() == out.numel() * _world():
            dist.reduce_scatter_tensor(out, flat)
            _maybe_simulate_collective_delay(out.numel() * out.element_size(), _world())
            self._maybe_synchronize(out)
            return out
        return super().reduce_scatter_into(out, flat)

    def allgather_into(self, out: torch.Tensor, shard: torch.Tensor) -> torch.Tensor:
        if self._fast(shard) and out.numel() == shard.numel() * _world():
            dist.all_gather_into_tensor(out, shard)
            _maybe_simulate_collective_delay(shard.numel() * shard.element_size(), _world())
            self._maybe_synchronize(out)
            return out
        return super().allgather_into(out, shard)

    def allgather(self, local_shard: torch.Tensor, sizes: Optional[Sequence[int]] = None) -> torch.Tensor:
        world = _world()
        local = local_shard.contiguous().view(-1)
        if sizes is None:
            mine = torch.tensor([local.numel()], dtype=torch.long, device=local.device)
            if self._fast(local):
                all_sizes = torch.empty(world, dtype=torch.long, device=local.device)
                dist.all_gather_into_tensor(all_sizes, mine)
                sizes = all_sizes.tolist()
            else:
                parts = [torch.zeros_like(mine) for _ in range(world)]
                dist.all_gather(parts, mine)
                sizes = [int(p.item()) for p in parts]
        sizes = [int(s) for s in sizes]
        width = max(sizes)
        if width == 0:
            return torch.empty(0, dtype=local.dtype, device=local.device)
        padded = local
        if local.numel() < width:
            padded = torch.zeros(width, dtype=local.dtype, device=local.device)
            padded[: local.numel()] = local
        if self._fast(local):
            out = torch.empty(world * width, dtype=local.dtype, device=local.device)
            dist.all_gather_into_tensor(out, padded)
            parts = [out[i * width : (i + 1) * width] for i in range(world)]
        else:
            parts = [torch.empty_like(padded) for _ in range(world)]
            dist.all_gather(parts, padded)
            out = None
        _maybe_simulate_collective_delay(padded.numel() * padded.element_size(), world)
        self._maybe_synchronize(padded)
        if len(set(sizes)) == 1:
            return out if out is not None else torch.cat(parts)
        return torch.cat([parts[r][: sizes[r]] for r in range(world)])


@dataclass
class TracingCollectives(CollectiveOps):
    """Wraps another implementation and records one entry per call.

    Record fields match the reference (``collectives/interface.py:269-292``): op, label,
    input_bytes, output_bytes, elapsed_ms (host), world_size, device, dtype.
    """

    inner: CollectiveOps = None

    def __post_init__(self) -> None:
        self._labels: List[str] = []
        self._trace: List[Dict[str, object]] = []
        self.name = f"tracing({getattr(self.inner, 'name', '?')})"

    def __getattr__(self, item):
        # Forward fused-path capabilities (e.g. device buffers) to the wrapped implementation.
        if item.startswith("_") or item == "inner":
            raise AttributeError(item)
        return getattr(self.inner, item)

    def _record(self, op: str, inp: torch.Tensor, out: torch.Tensor, elapsed_ms: float) -> None:
        self._trace.append(
            {
                "op": op,
                "label": "/".join(self._labels),
                "input_bytes": int(inp.numel() * inp.element_size()),
                "output_bytes": int(out.numel() * out.element_size()),
                "elapsed_ms": float(elapsed_ms),
                "world_size": _world(),
                "device": str(inp.device),
                "dtype": str(inp.dtype).replace("torch.", ""),
            }
        )

    def record_external(self, op: str, label: str, input_bytes: int, output_bytes: int, elapsed_ms: float,
                        device: str, dtype: str) -> None:
        """Record a collective that a fused kernel issued outside this interface."""
        full = "/".join(self._labels + [label]) if label else "/".join(self._labels)
        self._trace.append(
            {"op": op, "label": full, "input_bytes": int(input_bytes), "output_bytes": int(output_bytes),
             "elapsed_ms": float(elapsed_ms), "world_size": _world(), "device": device, "dtype": dtype}
        )

    @contextmanager
    def label_scope(self, label: str) -> Iterator[None]:
        self._labels.append(label)
        try:
            yield
        finally:
            self._labels.pop()

    def consume_trace(self) -> List[Dict[str, object]]:
        trace, self._trace = self._trace, []
        return trace

    def _timed(self, op: str, fn, inp: torch.Tensor) -> torch.Tensor:
        t0 = time.perf_counter()
        out = fn()
        self._record(op, inp, out, (time.perf_counter() - t0) * 1000.0)
        return out

    def allreduce(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        return self._timed("allreduce", lambda: self.inner.allreduce(tensor, average=average), tensor)

    def allreduce_inplace(self, tensor: torch.Tensor, average: bool = False) -> torch.Tensor:
        return self._timed("allreduce_inplace", lambda: self.inner.allreduce_inplace(tensor, average=average), tensor)

    def reduce_scatter(self, tensor: torch.Tensor) -> torch.Tensor:
        return self._timed("reduce_scatter", lambda: self.inner.reduce_scatter(tensor), tensor)

    def allgather(self, local_shard: torch.Tensor, sizes: Optional[Sequence[int]] = None) -> torch.Tensor:
        return self._timed("allgather", lambda: self.inner.allgather(local_shard, sizes=sizes), local_shard)


    @property
    def supports_fused(self) -> bool:  # type: ignore[override]
        return bool(getattr(self.inner, "supports_fused", False))

    def _timed_buf(self, op: str, fn, inp: torch.Tensor, out_bytes: int) -> torch.Tensor:
        t0 = time.perf_counter()
        res = fn()
        self._trace.append(
            {"op": op, "label": "/".join(self._labels), "input_bytes": int(inp.numel() * inp.element_size()),
             "output_bytes": int(out_bytes), "elapsed_ms": (time.perf_counter() - t0) * 1000.0,
             "world_size": _world(), "device": str(inp.device), "dtype": str(inp.dtype).replace("torch.", "")}
        )
        return res

    def allreduce_scaled_(self, flat: torch.Tensor, scale: float) -> torch.Tensor:
        return self._timed_buf("allreduce_inplace", lambda: self.inner.allreduce_scaled_(flat, scale), flat,
                               flat.numel() * flat.element_size())

    def reduce_scatter_into(self, out: torch.Tensor, flat: torch.Tensor) -> torch.Tensor:
        return self._timed_buf("reduce_scatter", lambda: self.inner.reduce_scatter_into(out, flat), flat,
                               out.numel() * out.element_size())

    def reduce_scatter_accumulate_(self, acc: torch.Tensor, flat: torch.Tensor, scale: float) -> torch.Tensor:
        return self._timed_buf("reduce_scatter", lambda: self.inner.reduce_scatter_accumulate_(acc, flat, scale), flat,
                               acc.numel() * flat.element_size())

    def allgather_into(self, out: torch.Tensor, shard: torch.Tensor) -> torch.Tensor:
        return self._timed_buf("allgather", lambda: self.inner.allgather_into(out, shard), shard,
                               out.numel() * out.element_size())


def aggregate_collective_trace(records: List[Dict[str, object]]) -> List[Dict[str, object]]:
    """Sum calls/time/bytes per (op, label), sorted by descending time (``train_zero.py:182-201``)."""
    table: Dict[tuple, Dict[str, object]] = {}
    for rec in records:
        key = (str(rec.get("op", "")), str(rec.get("label", "")))
        entry = table.setdefault(
            key, {"op": key[0], "label": key[1], "calls": 0, "elapsed_ms": 0.0, "input_bytes": 0.0, "output_bytes": 0.0}
        )
        entry["calls"] = int(entry["calls"]) + 1
        entry["elapsed_ms"] = float(entry["elapsed_ms"]) + float(rec.get("elapsed_ms", 0.0))
        entry["input_bytes"] = float(entry["input_bytes"]) + float(rec.get("input_bytes", 0.0))
        entry["output_bytes"] = float(entry["output_bytes"]) + float(rec.get("output_bytes", 0.0))
    return sorted(table.values(), key=lambda e: (-float(e["elapsed_ms"]), str(e["label"]), str(e["op"])))


def pick_collectives(world_size: int, impl: str, device: Optional[torch.device] = None) -> CollectiveOps:
    """world 1 -> Local; ``ring`` -> SendRecv; ``torch`` -> Torch; ``nvls`` -> NVLink kernels."""
    if world_size == 1:
        return LocalCollectives()
    if impl == "ring":
        return SendRecvCollectives()
    if impl == "torch":
        return TorchCollectives()
    if impl in ("nvls", "p2p"):
        from .comm.nvlink import NvlinkCollectives

        return NvlinkCollectives(device=device, use_multicast=(impl == "nvls"))
    raise ValueError(f"unknown collective impl {impl!r}")


__all__ = [
    "CollectiveOps",
    "LocalCollectives",
    "SendRecvCollectives",
    "TorchCollectives",
    "TracingCollectives",
    "aggregate_collective_trace",
    "pick_collectives",
    "simulated_collective_delay_s",
    "simulated_link_delay_s",
    "ring_allreduce",
    "ring_reduce_scatter",
    "ring_allgather",
]
