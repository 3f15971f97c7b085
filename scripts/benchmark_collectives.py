"""Collective micro-benchmark: ring vs NCCL vs this repo's NVLink kernels.

CLI-compatible with the reference's ``scripts/benchmark_collectives.py`` (``--ops``, ``--sizes`` in
elements, ``--impl``, ``--dtype``, ``--iters``, ``--warmup``, ``--device``, ``--output-json``,
``--seed``; values ``randn`` seeded with ``1234 + rank``), extended with ``--impl nvls|p2p|all``,
``--sizes-bytes`` (e.g. the 1 KB .. 1 GB power-of-two sweep) and ``--check`` (compare every result
with NCCL).  On GPUs ``mean_ms`` is the device time per call of ``--iters`` calls enqueued back to
back (CUDA events, max over ranks), so small messages show the collective's latency rather than the
Python launch path; ``p50_ms`` / ``p95_ms`` / ``synced_mean_ms`` come from calls timed one at a time
after a barrier and a synchronize (host launch included).  On CPU every figure is the one-at-a-time
wall time, max over ranks;
bus bandwidth uses the usual conventions: all-reduce ``2(W-1)/W * bytes``, reduce-scatter and
all-gather ``(W-1)/W * bytes`` where bytes is the full (unsharded) buffer.  Each row also reports the
fraction of the 900 GB/s-per-direction NVLink 5 figure and of the measured 770 GB/s peer copy.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        scripts/benchmark_collectives.py --impl all --dtype bfloat16 --sizes-bytes 1024:1073741824
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Dict, List

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from cs244c_llama_zero_b200.parallel.collectives import SendRecvCollectives, TorchCollectives  # noqa: E402

NVLINK_GBPS = 900.0
MEASURED_PEER_GBPS = 770.0


@dataclass
class OpResult:
    op: str
    impl: str
    numel: int
    dtype: str
    bytes_sent_per_rank: int
    mean_ms: float
    p50_ms: float
    p95_ms: float
    bus_gbps: float = 0.0
    frac_of_nvlink: float = 0.0
    frac_of_measured_peer: float = 0.0
    max_abs_err_vs_nccl: float = float("nan")
    synced_mean_ms: float = float("nan")  # mean of the individually synchronised calls (host launch included)


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--ops", nargs="+", default=["allreduce", "reduce_scatter", "allgather"])
    p.add_argument("--sizes", nargs="+", type=int, default=[1 << 12, 1 << 16, 1 << 20])
    p.add_argument("--sizes-bytes", type=str, default="", help="lo:hi power-of-two byte sweep, overrides --sizes")
    p.add_argument("--impl", choices=["ring", "torch", "nvls", "p2p", "both", "all"], default="both")
    p.add_argument("--dtype", choices=["float32", "float16", "bfloat16"], default="float32")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--device", choices=["auto", "cpu", "cuda"], default="auto")
    p.add_argument("--output-json", type=str, default="")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--check", action="store_true")
    return p.parse_args(argv)


def bytes_per_rank(op: str, numel: int, world: int, element_size: int) -> int:
    chunk = max(1, (numel + world - 1) // world)
    if op == "allreduce":
        return int(2 * (world - 1) * chunk * element_size)
    if op == "reduce_scatter":
        return int((world - 1) * chunk * element_size)
    if op == "allgather":
        return int((world - 1) * numel * element_size)
    raise ValueError(op)


def bus_factor(op: str, world: int) -> float:
    return 2.0 * (world - 1) / world if op == "allreduce" else (world - 1) / world


def init(device_choice: str) -> torch.device:
    use_cuda = torch.cuda.is_available() and device_choice != "cpu"
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if use_cuda:
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        if use_cuda:
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    return torch.device("cuda", local) if use_cuda else torch.device("cpu")


def _back_to_back_ms(fn, iters: int, device: torch.device) -> float:
    """Device time per call of ``iters`` calls enqueued back to back (max over ranks): the host stays
    ahead of the device, so the figure is the collective's own latency, not the launch path's."""
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(fn, iters: int, warmup: int, device: torch.device) -> List[float]:
    """Per-call samples, each bracketed by a barrier and a synchronize (includes the host launch)."""
    for _ in range(warmup):
        fn()
    samples = []
    for _ in range(iters):
        dist.barrier()
        if device.type == "cuda":
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            samples.append(s.elapsed_time(e))
        else:
            t0 = time.perf_counter()
            fn()
            samples.append((time.perf_counter() - t0) * 1000.0)
    t = torch.tensor(samples, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run(op: str, impl: str, numel: int, dtype: torch.dtype, args, device, nvl: Dict) -> OpResult:
    world, rank = dist.get_world_size(), dist.get_rank()
    torch.manual_seed(1234 + rank)
    numel = max(world * 8, (numel // (world * 8)) * world * 8)
    x = torch.randn(numel, dtype=dtype, device=device)
    chunk = numel // world
    err = float("nan")
    if impl in ("nvls", "p2p"):
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives

        coll = nvl.setdefault(impl, NvlinkCollectives(device=device, use_multicast=(impl == "nvls")))
        buf = coll.alloc(numel, dtype)
        acc = torch.zeros(chunk, dtype=torch.float32, device=device)
        shard = x[rank * chunk : (rank + 1) * chunk].contiguous()
        if op == "allreduce":
            fn = lambda: coll.allreduce_scaled_(buf, 1.0)  # noqa: E731
        elif op == "reduce_scatter":
            fn = lambda: coll.reduce_scatter_accumulate_(acc, buf, 1.0)  # noqa: E731
        else:
            fn = lambda: coll.allgather_into(buf, shard)  # noqa: E731
        if args.check:
            ref = x.float().clone()
            buf.copy_(x)
            if op == "allreduce":
                dist.all_reduce(ref)
                coll.allreduce_scaled_(buf, 1.0)
                err = (buf.float() - ref).abs().max().item()
            elif op == "reduce_scatter":
                dist.all_reduce(ref)
                acc.zero_()
                coll.reduce_scatter_accumulate_(acc, buf, 1.0)
                err = (acc - ref[rank * chunk : (rank + 1) * chunk]).abs().max().item()
            else:
                parts = [torch.empty(chunk, dtype=dtype, device=device) for _ in range(world)]
                dist.all_gather(parts, shard)
                coll.allgather_into(buf, shard)
                err = (buf.float() - torch.cat(parts).float()).abs().max().item()
        buf.copy_(x)
    else:
        coll = SendRecvCollectives() if impl == "ring" else TorchCollectives()
        shard = x[rank * chunk : (rank + 1) * chunk].contiguous()
        if op == "allreduce":
            fn = lambda: coll.allreduce(x)  # noqa: E731
        elif op == "reduce_scatter":
            fn = lambda: coll.reduce_scatter(x)  # noqa: E731
        else:
            fn = lambda: coll.allgather(shard, sizes=[chunk] * world)  # noqa: E731
    samples = sorted(_timed(fn, args.iters, args.warmup, device))
    synced = sum(samples) / len(samples)
    mean = _back_to_back_ms(fn, args.iters, device) if device.type == "cuda" else synced
    nbytes = numel * x.element_size()
    bus = bus_factor(op, world) * nbytes / (mean / 1000.0) / 1e9
    return OpResult(op=op, impl=impl, numel=numel, dtype=str(dtype).replace("torch.", ""),
                    bytes_sent_per_rank=bytes_per_rank(op, numel, world, x.element_size()), mean_ms=mean,
                    p50_ms=samples[len(samples) // 2], p95_ms=samples[min(len(samples) - 1, int(0.95 * len(samples)))],
                    bus_gbps=bus, frac_of_nvlink=bus / NVLINK_GBPS, frac_of_measured_peer=bus / MEASURED_PEER_GBPS,
                    max_abs_err_vs_nccl=err, synced_mean_ms=synced)


def main(argv=None) -> None:
    args = parse_args(argv)
    device = init(args.device)
    rank, world = dist.get_rank(), dist.get_world_size()
    dtype = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[args.dtype]
    elem = torch.tensor([], dtype=dtype).element_size()
    sizes = args.sizes
    if args.sizes_bytes:
        lo, hi = (int(v) for v in args.sizes_bytes.split(":"))
        sizes, b = [], lo
        while b <= hi:
            sizes.append(max(1, b // elem))
            b *= 2
    impls = {"both": ["ring", "torch"], "all": ["torch", "nvls", "p2p"]}.get(args.impl, [args.impl])
    if device.type == "cuda":
        impls = [i for i in impls if i != "ring"]  # the send/recv ring is a CPU/gloo oracle
    else:
        impls = [i for i in impls if i in ("ring", "torch")]
    results: List[OpResult] = []
    cache: Dict = {}
    t0 = time.perf_counter()
    for op in args.ops:
        for numel in sizes:
            for impl in impls:
                results.append(run(op, impl, numel, dtype, args, device, cache))
                if rank == 0:
                    r = results[-1]
                    print(f"{r.op:15s} {r.impl:6s} {r.numel * elem:>12d} B  {r.mean_ms:9.4f} ms  "
                          f"bus {r.bus_gbps:8.1f} GB/s ({100 * r.frac_of_nvlink:5.1f}% of 900)", flush=True)
    report = {"world_size": world, "backend": dist.get_backend(), "elapsed_s": time.perf_counter() - t0,
              "args": vars(args), "results": [asdict(r) for r in results]}
    if rank == 0 and args.output_json:
        Path(args.output_json).parent.mkdir(parents=True, exist_ok=True)
        Path(args.output_json).write_text(json.dumps(report, indent=2))
        print(f"[benchmark] wrote {args.output_json}")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
