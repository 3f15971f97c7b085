"""All-reduce throughput: NCCL (``torch.distributed.all_reduce``) or this repo's NVLink kernels.

Each iteration is timed on the device (CUDA events around the call, after a barrier); the reported
time is the mean over iterations of the max over ranks.  ``effective_allreduce_gbps`` keeps the
reference's definition (``2(W-1)/W * bytes * 8 / t`` in gigabits/s); ``bus_gbytes_per_s`` is the same
volume in GB/s, the figure to hold against NVLink's 900 GB/s per direction.  On CPU (gloo) it falls
back to wall-clock timing.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 scripts/benchmark_allreduce.py \
        --numel 268435456 --dtype bfloat16 --impl nvls
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Benchmark distributed all_reduce throughput")
    p.add_argument("--numel", type=int, default=64 * 1024 * 1024)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--dtype", type=str, default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--impl", type=str, default="torch", choices=["torch", "nvls", "p2p"])
    return p.parse_args(argv)


def main(argv=None) -> None:
    args = parse_args(argv)
    cuda = torch.cuda.is_available()
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local_rank) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(device)
    backend = "nccl" if cuda else "gloo"
    dist.init_process_group(backend=backend, timeout=timedelta(seconds=300),
                            **({"device_id": device} if cuda else {}))
    rank, world = dist.get_rank(), dist.get_world_size()
    dtype = torch.float32 if args.dtype == "float32" else torch.bfloat16
    if args.impl != "torch" and not (cuda and world > 1):
        raise SystemExit("--impl nvls/p2p needs CUDA and more than one rank")
    if args.impl == "torch":
        tensor = torch.ones(args.numel, dtype=dtype, device=device)
        run = lambda: dist.all_reduce(tensor)  # noqa: E731
    else:
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives

        coll = NvlinkCollectives(device, use_multicast=args.impl == "nvls")
        tensor = coll.alloc(args.numel, dtype)
        tensor.fill_(1.0)
        run = lambda: coll.allreduce_scaled_(tensor, 1.0 / world)  # noqa: E731
    for _ in range(args.warmup):
        run()
    times = []
    for _ in range(args.iters):
        dist.barrier()
        if cuda:
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            run()
            end.record()
            end.synchronize()
            ms = start.elapsed_time(end)
        else:
            t0 = time.perf_counter()
            run()
            ms = (time.perf_counter() - t0) * 1e3
        worst = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        times.append(float(worst.item()))
    mean_s = sum(times) / len(times) / 1e3
    payload = tensor.numel() * tensor.element_size()
    volume = 2.0 * (world - 1) / world * payload
    if rank == 0:
        print(json.dumps({"backend": backend, "impl": args.impl, "world_size": world, "numel": args.numel,
                          "dtype": args.dtype, "mean_ms": mean_s * 1e3, "min_ms": min(times),
                          "payload_mb": payload / 1e6, "effective_allreduce_gbps": volume * 8.0 / (mean_s * 1e9),
                          "bus_gbytes_per_s": volume / (mean_s * 1e9), "timing": "device max over ranks"
                          if cuda else "wall clock max over ranks"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
