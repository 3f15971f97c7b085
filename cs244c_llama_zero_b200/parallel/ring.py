"""Ring collectives built from point-to-point send/recv.

Behaviour follows the reference's ``collectives/_ring.py:1-252``: inputs are flattened
and zero-padded to ``W * ceil(n/W)``; the reduce-scatter leaves rank ``r`` with the
fully reduced chunk ``r``; the all-gather circulates chunks around the ring;
all-reduce is reduce-scatter followed by all-gather; variable-size all-gather
exchanges sizes first and trims.  Every hop is an ``irecv`` from the left
neighbour plus an ``isend`` to the right neighbour, followed by an optional
emulated link delay (``ZERO_SIM_BW_GBPS`` / ``ZERO_SIM_LATENCY_MS``).

These run on CPU/Gloo and serve as the correctness oracle for the GPU paths.
"""

from __future__ import annotations

import math
import os
import time
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

RS_TAG_BASE = 10_000
AR_TAG_BASE = 20_000
AG_TAG_BASE = 30_000


def _rank_world() -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("torch.distributed must be initialized before calling ring collectives")
    return dist.get_rank(), dist.get_world_size()


def _padded_copy(tensor: torch.Tensor, world_size: int) -> Tuple[torch.Tensor, int, int]:
    flat = tensor.contiguous().view(-1)
    numel = flat.numel()
    chunk = max(1, math.ceil(numel / world_size))
    out = torch.zeros(chunk * world_size, dtype=flat.dtype, device=flat.device)
    out[:numel] = flat
    return out, numel, chunk


def simulated_link_delay_s(num_bytes: int) -> float:
    bw = os.environ.get("ZERO_SIM_BW_GBPS", "").strip()
    lat = os.environ.get("ZERO_SIM_LATENCY_MS", "").strip()
    delay = 0.0
    if bw and float(bw) > 0:
        delay += num_bytes / (float(bw) * 1e9)
    if lat and float(lat) > 0:
        delay += float(lat) / 1000.0
    return delay


def _hop(send: torch.Tensor, recv: torch.Tensor, right: int, left: int, tag: int) -> None:
    rreq = dist.irecv(recv, src=left, tag=tag)
    sreq = dist.isend(send, dst=right, tag=tag)
    sreq.wait()
    rreq.wait()
    delay = simulated_link_delay_s(send.numel() * send.element_size())
    if delay > 0:
        time.sleep(delay)


def _reduce_scatter_chunks(chunks: Sequence[torch.Tensor], rank: int, world: int, tag_base: int) -> None:
    right, left = (rank + 1) % world, (rank - 1) % world
    for step in range(world - 1):
        send_idx = (rank - step - 1) % world
        recv_idx = (rank - step - 2) % world
        incoming = torch.empty_like(chunks[recv_idx])
        _hop(chunks[send_idx].clone(), incoming, right, left, tag_base + step)
        chunks[recv_idx].add_(incoming)


def _allgather_chunks(chunks: Sequence[torch.Tensor], rank: int, world: int, tag_base: int) -> None:
    right, left = (rank + 1) % world, (rank - 1) % world
    for step in range(world - 1):
        send_idx = (rank - step) % world
        recv_idx = (rank - step - 1) % world
        incoming = torch.empty_like(chunks[recv_idx])
        _hop(chunks[send_idx].clone(), incoming, right, left, tag_base + step)
        chunks[recv_idx].copy_(incoming)


def _split(flat: torch.Tensor, chunk: int, world: int) -> List[torch.Tensor]:
    return [flat[i * chunk : (i + 1) * chunk] for i in range(world)]


def ring_reduce_scatter(tensor: torch.Tensor, op: str = "sum", tag_base: int = RS_TAG_BASE) -> torch.Tensor:
    """Returns this rank's reduced (trimmed) flat shard."""
    if op != "sum":
        raise ValueError(f"Only op='sum' is supported, got '{op}'")
    rank, world = _rank_world()
    if world == 1:
        return tensor.contiguous().view(-1).clone()
    flat, numel, chunk = _padded_copy(tensor, world)
    chunks = _split(flat, chunk, world)
    _reduce_scatter_chunks(chunks, rank, world, tag_base)
    start = rank * chunk
    end = min(start + chunk, numel)
    return chunks[rank][: max(0, end - start)].clone()


def ring_allreduce(tensor: torch.Tensor, op: str = "sum", average: bool = False, tag_base: int = AR_TAG_BASE) -> torch.Tensor:
    """Same shape/dtype as the input; reduce-scatter then all-gather around the ring."""
    if op != "sum":
        raise ValueError(f"Only op='sum' is supported, got '{op}'")
    rank, world = _rank_world()
    if world == 1:
        out = tensor.clone()
        return out / 1.0 if average else out
    flat, numel, chunk = _padded_copy(tensor, world)
    chunks = _split(flat, chunk, world)
    _reduce_scatter_chunks(chunks, rank, world, tag_base)
    _allgather_chunks(chunks, rank, world, tag_base + 1_000)
    if average:
        flat /= world
    return flat[:numel].view_as(tensor).clone()


def ring_allgather(local_shard: torch.Tensor, tag_base: int = AG_TAG_BASE, sizes: Optional[Sequence[int]] = None) -> torch.Tensor:
    """Concatenation of every rank's flat shard; shards may differ in length.

    ``sizes`` (per-rank element counts) skips the size exchange when the caller
    already knows them.
    """
    rank, world = _rank_world()
    local = local_shard.contiguous().view(-1)
    if world == 1:
        return local.clone()
    if sizes is None:
        mine = torch.tensor([local.numel()], dtype=torch.long, device=local.device)
        gathered_sizes = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(gathered_sizes, mine)
        sizes = [int(s.item()) for s in gathered_sizes]
    sizes = list(sizes)
    width = max(sizes)
    if width == 0:
        return torch.empty(0, dtype=local.dtype, device=local.device)
    out = torch.zeros(width * world, dtype=local.dtype, device=local.device)
    chunks = _split(out, width, world)
    chunks[rank][: local.numel()].copy_(local)
    _allgather_chunks(chunks, rank, world, tag_base)
    if len(set(sizes)) == 1:
        return out
    return torch.cat([chunks[r][: sizes[r]] for r in range(world)])
