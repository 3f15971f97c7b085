"""Distributed sanity check: all-reduce of ``rank + 1`` must equal ``W(W+1)/2`` on every rank.

On CUDA with more than one rank it also checks this repository's NVLink all-reduce kernel (symmetric
memory, NVLS multicast when the switch offers it, else peer loads) against NCCL on a small buffer.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 scripts/distributed_sanity.py
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main() -> None:
    cuda = torch.cuda.is_available()
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local_rank) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    backend = "nccl" if cuda else "gloo"
    dist.init_process_group(backend=backend, timeout=timedelta(seconds=120),
                            **({"device_id": device} if cuda else {}))
    rank, world = dist.get_rank(), dist.get_world_size()
    x = torch.tensor([float(rank + 1)], device=device)
    dist.all_reduce(x)
    expected = world * (world + 1) / 2.0
    if abs(float(x.item()) - expected) > 1e-6:
        raise RuntimeError(f"all_reduce failed on rank {rank}: got {x.item()}, expected {expected}")
    line = f"[sanity] backend={backend} world_size={world} all_reduce_sum={x.item():.1f}"
    if cuda and world > 1:
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives

        coll = NvlinkCollectives(device, use_multicast=True)
        buf = coll.alloc(1 << 20, torch.float32)
        buf.copy_(torch.full_like(buf, float(rank + 1)))
        ref = buf.clone()
        dist.all_reduce(ref)
        coll.allreduce_scaled_(buf, 1.0)
        torch.cuda.synchronize()
        err = (buf - ref).abs().max().item()
        if err > 0.0:
            raise RuntimeError(f"NVLink all-reduce differs from NCCL on rank {rank}: max |err| = {err}")
        line += f" nvlink_allreduce=ok multicast={coll.buffers[-1].multicast}"
        del buf
    if rank == 0:
        print(line, flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
