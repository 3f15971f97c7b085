"""Collective correctness on CPU gloo ranks (W = 2 and 3): ring and torch implementations vs dist.* references.

Sizes include ones that do not divide by W (the ring pads to W * ceil(n / W) and trims), variable
all-gather shard sizes, and the buffer-level entry points the ZeRO engines use
(allreduce_scaled_, reduce_scatter_accumulate_, reduce_scatter_into, allgather_into).
"""

from __future__ import annotations

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cs244c_llama_zero_b200.parallel.collectives import SendRecvCollectives, TorchCollectives
from cs244c_llama_zero_b200.parallel.ring import ring_allgather, ring_allreduce, ring_reduce_scatter

from .dist_utils import find_free_port, init_gloo


def _close(a, b, msg):
    torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5, msg=msg)


def _worker(rank: int, world: int, port: int) -> None:
    init_gloo(rank, world, port)
    try:
        for numel in (16, 257, 4096):
            x = torch.arange(numel, dtype=torch.float32) + rank * 0.25
            ref = x.clone()
            dist.all_reduce(ref)
            _close(ring_allreduce(x), ref, f"ring allreduce {numel}")
            _close(ring_allreduce(x, average=True), ref / world, f"ring allreduce avg {numel}")
            chunk = -(-numel // world)
            mine = ref[rank * chunk: min(numel, (rank + 1) * chunk)]
            _close(ring_reduce_scatter(x), mine, f"ring reduce_scatter {numel}")
            for impl in (SendRecvCollectives(), TorchCollectives()):
                _close(impl.allreduce(x), ref, f"{type(impl).__name__} allreduce {numel}")
                _close(impl.reduce_scatter(x), mine, f"{type(impl).__name__} reduce_scatter {numel}")
        for n in (8, 127):
            shard = torch.full((n,), float(rank))
            want = torch.cat([torch.full((n,), float(r)) for r in range(world)])
            _close(ring_allgather(shard), want, f"ring allgather {n}")
            _close(TorchCollectives().allgather(shard), want, f"torch allgather {n}")
        var = torch.full((5 + rank,), float(rank))
        want = torch.cat([torch.full((5 + r,), float(r)) for r in range(world)])
        sizes = [5 + r for r in range(world)]
        _close(ring_allgather(var, sizes=sizes), want, "ring allgather variable")
        _close(TorchCollectives().allgather(var, sizes=sizes), want, "torch allgather variable")
        _close(TorchCollectives().allgather(var), want, "torch allgather variable (sizes exchanged)")

        # buffer-level entry points used by the ZeRO engines
        coll = TorchCollectives()
        flat = torch.arange(12 * world, dtype=torch.float32) * (rank + 1)
        total = torch.arange(12 * world, dtype=torch.float32) * sum(r + 1 for r in range(world))
        buf = flat.clone()
        coll.allreduce_scaled_(buf, 0.5)
        _close(buf, total * 0.5, "allreduce_scaled_")
        acc = torch.ones(12)
        coll.reduce_scatter_accumulate_(acc, flat, 2.0)
        _close(acc, 1.0 + 2.0 * total[12 * rank: 12 * (rank + 1)], "reduce_scatter_accumulate_")
        out = torch.empty(12)
        coll.reduce_scatter_into(out, flat)
        _close(out, total[12 * rank: 12 * (rank + 1)], "reduce_scatter_into")
        gathered = torch.empty(12 * world)
        coll.allgather_into(gathered, torch.full((12,), float(rank)))
        _close(gathered, torch.cat([torch.full((12,), float(r)) for r in range(world)]), "allgather_into")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_collectives_match_dist(world):
    mp.spawn(_worker, args=(world, find_free_port()), nprocs=world, join=True)
