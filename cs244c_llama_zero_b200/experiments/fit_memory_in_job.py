"""Fit-to-memory on B200 inside one job: the largest per-GPU micro-batch of each ZeRO stage, its
throughput and its peak memory, from a memory model measured in the same processes.

The reference's fit-to-memory workflow (``experiments/run_fit_memory_bandwidth.py:238-326``, reproduced
here by ``run_fit_memory_bandwidth.py`` + ``tuning.search_max_batch_size``) launches one training job
per probed batch size and bisects on out-of-memory failures.  At 7B scale each launch spends most of
its time building the model, and a probe that runs out of memory on one rank can leave the others
waiting inside a collective.  This runner keeps one process group per GPU count and, per stage:

1. builds the engine once (parameters created on the GPUs),
2. runs two training steps at each probe batch size (``--probe-batches``, default 1 and 2), with the
   allocator's cache emptied first, and reads the allocated peak (max over ranks),
3. fits ``peak(b) = slope * b + base`` (the reference's ``memory_model`` predictor kind) and takes
   ``b_max = floor((capacity_fraction * total_memory - base - outside) / slope)``, min over ranks,
   where ``outside`` is the memory held outside PyTorch's allocator (the symmetric NVLink buffers),
4. times ``--steps`` steps at ``b_max`` (device events, max over ranks) and records tokens/s and the
   measured peak.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m cs244c_llama_zero_b200.experiments.fit_memory_in_job --model-size baseline-7b --seq-len 2048 \\
        --stages 0,1,2,3 --output-json results/fit_7b_w8.json

Inputs are uniform random token ids; weights normal(0, 0.02); bf16 with fp32 master weights.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import time
from typing import Dict, List

import torch
import torch.distributed as dist


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--model-size", default="baseline-7b")
    p.add_argument("--seq-len", type=int, default=2048)
    p.add_argument("--stages", default="0,1,2,3")
    p.add_argument("--probe-batches", default="1,2")
    p.add_argument("--capacity-fraction", type=float, default=0.85,
                   help="share of the GPU's memory the predicted batch's allocated peak may use (the rest is "
                        "headroom for the allocator's fragmentation)")
    p.add_argument("--max-batch", type=int, default=256)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--collective-impl", default="auto")
    p.add_argument("--output-json", default="")
    p.add_argument("--pg-timeout", type=float, default=300.0,
                   help="seconds a collective may wait before the process group reports an error")
    return p.parse_args(argv)


def _max_over_ranks(x: float) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def _batch(b: int, seq: int, vocab: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (b, seq), generator=g, dtype=torch.long).pin_memory()


def fit_line(points: List[tuple]) -> tuple:
    """(slope, base) of the least-squares line through (batch, peak MB) points."""
    n = len(points)
    mx = sum(x for x, _ in points) / n
    my = sum(y for _, y in points) / n
    sxx = sum((x - mx) ** 2 for x, _ in points)
    if sxx == 0:
        raise ValueError("probe batches must differ")
    slope = sum((x - mx) * (y - my) for x, y in points) / sxx
    return slope, my - slope * mx


def predict_max_batch(slope: float, base: float, capacity_mb: float, fraction: float, cap: int) -> int:
    if slope <= 0:
        return cap
    return max(0, min(cap, int(math.floor((fraction * capacity_mb - base) / slope))))


def measure_stage(args, stage: int, rank: int, world: int, impl: str) -> Dict[str, object]:
    from ..models import BASELINE_VOCAB_SIZE
    from ..train import SessionConfig, TrainSession

    t_build = time.perf_counter()
    sess = TrainSession(SessionConfig(model_size=args.model_size, vocab_size=BASELINE_VOCAB_SIZE,
                                      seq_len=args.seq_len, batch_size=1, zero_stage=stage,
                                      collective_impl=impl, backend="b200"))
    build_s = time.perf_counter() - t_build
    dev = sess.device
    total_mb = torch.cuda.get_device_properties(dev).total_memory / 2**20
    points = []
    for b in [int(x) for x in args.probe_batches.split(",")]:
        ids = _batch(b, args.seq_len, BASELINE_VOCAB_SIZE, 7 + rank).to(dev)
        # The allocator's cache from the build (or the previous probe) would absorb this probe's
        # activations and flatten the fitted slope: release it, and fit the allocated peak.
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        for _ in range(2):
            sess.train_step(ids)
        torch.cuda.synchronize(dev)
        points.append((b, _max_over_ranks(torch.cuda.max_memory_allocated(dev) / 2**20)))
        del ids
    # Memory outside PyTorch's caching allocator (symmetric NVLink buffers of the parameters and
    # gradients, NCCL, the CUDA context) does not show in the allocator's statistics but fills the
    # same HBM: measured after the probes (lazy allocations included) and subtracted from the budget.
    torch.cuda.synchronize(dev)
    free_b, total_b = torch.cuda.mem_get_info(dev)
    other_mb = _max_over_ranks((total_b - free_b - torch.cuda.memory_reserved(dev)) / 2**20)
    slope, base = fit_line(points)
    b_max = predict_max_batch(slope, base + other_mb, total_mb, args.capacity_fraction, args.max_batch)
    if dist.is_initialized() and world > 1:  # every rank runs the same batch
        t = torch.tensor([b_max], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        b_max = int(t.item())
    rec: Dict[str, object] = {"stage": stage, "world_size": world, "build_s": build_s,
                              "probe_peak_allocated_mb": points, "slope_mb_per_sample": slope,
                              "base_mb": base, "outside_allocator_mb": other_mb, "gpu_total_mb": total_mb,
                              "capacity_fraction": args.capacity_fraction, "selected_batch_size": b_max}
    if b_max >= 1:
        ids = _batch(b_max, args.seq_len, BASELINE_VOCAB_SIZE, 11 + rank).to(dev)
        torch.cuda.synchronize(dev)
        torch.cuda.reset_peak_memory_stats(dev)
        for _ in range(args.warmup):
            sess.train_step(ids)
        if dist.is_initialized() and world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            loss = sess.train_step(ids)
        end.record()
        torch.cuda.synchronize(dev)
        ms = _max_over_ranks(start.elapsed_time(end) / args.steps)
        rec.update({"ms_per_step": ms, "tokens_per_s": b_max * args.seq_len * world / (ms / 1000.0),
                    "peak_reserved_mb": _max_over_ranks(torch.cuda.max_memory_reserved(dev) / 2**20),
                    "peak_allocated_mb": _max_over_ranks(torch.cuda.max_memory_allocated(dev) / 2**20),
                    "loss": float(loss)})
    del sess
    torch.cuda.empty_cache()
    return rec


def main(argv=None) -> None:
    args = parse_args(argv)
    from ..train.session import init_distributed

    rank, world, _ = init_distributed(args.pg_timeout)
    impl = args.collective_impl
    if impl == "auto":
        impl = "nvls" if world > 1 else "torch"
    results = []
    for stage in [int(s) for s in args.stages.split(",") if s.strip()]:
        rec = measure_stage(args, stage, rank, world, impl)
        rec["model"] = args.model_size
        rec["seq_len"] = args.seq_len
        rec["collective_impl"] = impl
        results.append(rec)
        if rank == 0:
            print(json.dumps(rec), flush=True)
    if rank == 0 and args.output_json:
        os.makedirs(os.path.dirname(os.path.abspath(args.output_json)), exist_ok=True)
        with open(args.output_json, "w") as fh:
            json.dump({"results": results}, fh, indent=2)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
