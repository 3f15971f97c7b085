"""Headline benchmark: ZeRO training throughput of the 'small' LLaMA on N B200 GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference] [--stages 0,1,2,3]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

For every ZeRO stage in ``--stages`` the script builds the model and engine, runs W untimed
warm-up steps, then times exactly K optimizer steps with CUDA events between a barrier +
``torch.cuda.synchronize()`` on both sides; the step time is the maximum over ranks.  The
end-to-end number repeats K steps through the public training API with a pinned-host -> device
copy of each step's tokens and a device -> host read of each step's loss.  Rank 0 prints one JSON
line.  ``value`` is the whole-job tokens/s of the headline stage; every measured stage is listed
under ``per_stage``.

``--impl reference`` drives the unmodified reference implementation installed in
``baseline/_ref`` through its own model / engine / collectives classes (see
``baseline/run_reference.py``); it never imports this repository's package.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/s (device-timed, max over ranks) per ZeRO stage 0–3 at 1/2/4/8 B200; comm_ms"
MODEL_DESC = "small LLaMA d768/L12/H12/KV4/ffn2048/V32000 (tied embeddings)"


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["mine", "reference"], default="mine")
    p.add_argument("--stages", type=str, default="0,1,2,3")
    p.add_argument("--headline-stage", type=int, default=2)
    p.add_argument("--batch-size", type=int, default=8, help="micro-batch per GPU")
    p.add_argument("--seq-len", type=int, default=1024)
    p.add_argument("--collective-impl", type=str, default="auto", help="auto | torch | nvls | p2p")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--clocks-csv", type=str, default=None, help="keep the raw nvidia-smi clock samples here")
    p.add_argument("--fused-step", action="store_true",
                   help="ZeRO-1/2 unclipped step as one NVLink kernel (reduce-scatter + norm + AdamW + all-gather)")
    p.add_argument("--routed-grads", action="store_true",
                   help="ZeRO-2 without a full gradient buffer: gradients added into their owners' shards over NVLink")
    p.add_argument("--cuda-graph", action="store_true",
                   help="run stages 0-2 as one captured CUDA graph per step (TrainSession cuda_graph mode)")
    p.add_argument("--model-size", type=str, default="baseline-small",
                   help="model preset: baseline-small (the headline config), baseline-1.3b, baseline-7b, ...")
    args = p.parse_args(argv)
    args.warmup = max(3, args.warmup)
    args.stage_list = [int(s) for s in args.stages.split(",") if s.strip()]
    if args.headline_stage not in args.stage_list:
        args.headline_stage = args.stage_list[0]
    return args


# ----------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices, path=None):
        self.gpu_indices = set(gpu_indices)
        self.proc = None
        # The raw samples go to --clocks-csv when given (kept), else to a temporary file; the JSON
        # line carries the summary either way.
        self.path = path or os.path.join(tempfile.gettempdir(), f"zb_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        mhz, max_mhz, reasons = [], [], set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    idx = int(parts[0])
                except ValueError:
                    continue
                if self.gpu_indices and idx not in self.gpu_indices:
                    continue
                try:
                    mhz.append(float(parts[1]))
                    max_mhz.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names[1:], parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [m for m in mhz if m > 0.5 * max(mhz)] or mhz
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(max_mhz), "reasons": sorted(reasons),
                "samples": len(mhz)}


# ----------------------------------------------------------------------------------- helpers
def model_desc(size: str) -> str:
    if size == "baseline-small":
        return MODEL_DESC
    from cs244c_llama_zero_b200.models import BASELINE_VOCAB_SIZE
    from cs244c_llama_zero_b200.models.config import build_config

    c = build_config(size, vocab_size=BASELINE_VOCAB_SIZE)
    return (f"{size} LLaMA d{c.dim}/L{c.n_layers}/H{c.n_heads}/KV{c.n_kv_heads}/ffn{c.ffn_dim}/V{c.vocab_size}"
            f" ({'tied' if c.tie_word_embeddings else 'untied'} embeddings)")


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def max_over_ranks(value: float) -> float:
    import torch
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return value


def barrier_sync():
    import torch
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
    torch.cuda.synchronize()


def time_device(step_fn, steps: int) -> float:
    """Device time of ``steps`` calls (ms per step), max over ranks."""
    import torch

    barrier_sync()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step_fn()
    end.record()
    barrier_sync()
    return max_over_ranks(start.elapsed_time(end) / steps)


def time_wall(step_fn, steps: int, finish=None) -> float:
    barrier_sync()
    t0 = time.perf_counter()
    for _ in range(steps):
        step_fn()
    if finish is not None:
        finish()
    barrier_sync()
    return max_over_ranks((time.perf_counter() - t0) * 1000.0 / steps)


def random_batches(n: int, batch: int, seq: int, vocab: int, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (batch, seq), generator=g, dtype=torch.long).pin_memory() for _ in range(n)]


def emit(record: dict, rank: int) -> None:
    if rank == 0:
        print(json.dumps(record), flush=True)


def base_record(args, world: int, impl: str) -> dict:
    return {
        "metric": METRIC,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic uniform-random token ids (seeded), random-init weights normal(0, 0.02)",
        "impl": impl,
    }


# ----------------------------------------------------------------------------------- our arm
def roofline_entry(sess, args, stage: int, ms: float, peak_tflops: float) -> dict:
    """Executed tensor-core TFLOP/s of one GPU's step (causal attention halved, no recompute unless the
    stage-3 engine recomputes) and its fraction of the peak."""
    from cs244c_llama_zero_b200.profiler import executed_train_flops, roofline_fraction

    recompute = stage == 3 and bool(getattr(sess.engine, "recompute", False))
    executed = executed_train_flops(sess.model_cfg, args.batch_size, args.seq_len, recompute_forward=recompute)
    return {"executed_tflops_per_gpu": executed / (ms / 1000.0) / 1e12,
            "roofline_fraction": roofline_fraction(executed, ms / 1000.0, peak_tflops)}


def run_mine(args) -> None:
    import torch
    import torch.distributed as dist

    from cs244c_llama_zero_b200 import ops
    from cs244c_llama_zero_b200.models import BASELINE_VOCAB_SIZE
    from cs244c_llama_zero_b200.profiler import peak_bf16_tflops
    from cs244c_llama_zero_b200.train import SessionConfig, TrainSession

    peak_tflops, peak_source = peak_bf16_tflops()
    rank, world, local = dist_env()
    if world != args.gpus and rank == 0:
        print(f"[bench] note: --gpus {args.gpus} but WORLD_SIZE={world}; using {world}", file=sys.stderr)
    if args.fused_step:
        os.environ["ZB_FUSED_STEP"] = "1"
    if args.routed_grads:
        os.environ["ZB_ROUTED_GRADS"] = "1"
    impl = args.collective_impl
    if impl == "auto":
        impl = "nvls" if world > 1 else "torch"
    per_stage = {}
    e2e = None
    launches = None
    clocks = None
    headline_ms = None
    tokens_per_step = args.batch_size * args.seq_len * world
    for stage in args.stage_list:
        sess = TrainSession(SessionConfig(model_size=args.model_size, vocab_size=BASELINE_VOCAB_SIZE,
                                          seq_len=args.seq_len, batch_size=args.batch_size, zero_stage=stage,
                                          collective_impl=impl, backend="b200",
                                          cuda_graph=args.cuda_graph and stage != 3))
        host = random_batches(4, args.batch_size, args.seq_len, BASELINE_VOCAB_SIZE, seed=1234 + rank * 100 + stage)
        dev = [h.to(sess.device) for h in host]
        it = {"i": 0}

        def device_step():
            sess.train_step(dev[it["i"] % len(dev)])
            it["i"] += 1

        # The sampler starts before the warm-up so that short timed regions still get samples taken
        # under steady load; it stops right after the timed steps.
        sampler = ClockSampler([local], args.clocks_csv) if stage == args.headline_stage and rank == 0 else None
        if sampler:
            sampler.__enter__()
        for _ in range(args.warmup):
            device_step()
        torch.cuda.synchronize()
        launches_before = ops.launch_count()
        ms = time_device(device_step, args.steps)
        if sampler:
            sampler.__exit__(None, None, None)
            clocks = sampler.summary()
        stage_launches = (ops.launch_count() - launches_before) // args.steps
        entry = {"tokens_per_s": tokens_per_step / (ms / 1000.0), "ms_per_step": ms,
                 "gpu_launches_per_step": stage_launches}
        entry.update(roofline_entry(sess, args, stage, ms, peak_tflops))
        # comm time of one extra instrumented step (device events around each collective); the
        # barrier keeps host-side skew between ranks out of the measured intervals
        barrier_sync()
        sess.engine.clock.timing = True  # an eager instrumented step, also in graph mode
        sess.engine.zero_grad()
        sess.engine.prepare_forward()
        sess.forward_backward([dev[0]])
        st = sess.engine.step_with_stats(max_grad_norm=0.0)
        entry["comm_ms"] = max_over_ranks(float(st["comm_ms"]))
        if stage == args.headline_stage:
            headline_ms = ms
            launches = stage_launches * args.steps
            if not args.no_e2e:
                h2d = host[0].numel() * host[0].element_size()

                pending = []
                d2h = 0

                def e2e_step():
                    # pinned host batch -> device inside train_step; the step's loss is copied to
                    # pinned host memory and read (.item()) after the next step has been queued
                    nonlocal d2h
                    pending.append(sess.train_step_async(host[it["i"] % len(host)]))
                    d2h = pending[-1].nbytes  # loss + the kernels' error record
                    it["i"] += 1
                    if len(pending) > 1:
                        losses.append(pending.pop(0).item())

                def e2e_finish():  # the last step's loss is read inside the timed region too
                    while pending:
                        losses.append(pending.pop(0).item())

                losses = []
                for _ in range(2):
                    e2e_step()
                e2e_finish()
                losses.clear()
                e2e_ms = time_wall(e2e_step, args.steps, finish=e2e_finish)
                if len(losses) != args.steps or not all(math.isfinite(x) for x in losses):
                    raise RuntimeError(f"e2e: expected {args.steps} finite losses, got {losses}")
                e2e = {"value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s",
                       "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "api": "cs244c_llama_zero_b200.train.TrainSession.train_step_async(pinned host int64 [B,S])"
                              " + AsyncLoss.item() one step later (every step's loss and error record read on the host)"}
        per_stage[str(stage)] = entry
        del sess
        torch.cuda.empty_cache()
    errors = ops.load_extension().read_device_errors()
    rec = base_record(args, world, "mine")
    head = per_stage[str(args.headline_stage)]
    rec.update({
        "value": head["tokens_per_s"],
        "ms_per_step": headline_ms,
        "config": {"model": model_desc(args.model_size), "global_batch": args.batch_size * world, "micro_batch_per_gpu": args.batch_size,
                   "seq_len": args.seq_len, "grad_accum": 1, "parallelism": f"dp{world}",
                   "zero_stage": args.headline_stage, "collective_impl": impl,
                   "cuda_graph": bool(args.cuda_graph and args.headline_stage != 3),
                   "fused_step": bool(args.fused_step),
                   "routed_grads": bool(args.routed_grads),
                   "l2": "no flush: each step touches >2 GB (activations, 1.2 GB fp32 optimizer state) vs 126 MB L2"},
        "per_stage": per_stage,
        "roofline": {"executed_tflops_per_gpu": head["executed_tflops_per_gpu"],
                     "fraction": head["roofline_fraction"], "peak_bf16_tflops": peak_tflops,
                     "peak_source": peak_source, "note": "of measured sustained cuBLAS bf16 GEMM peak"
                     if peak_source == "measured" else "of fallback peak"},
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks,
        "device_errors": list(errors),
    })
    emit(rec, rank)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(HERE, "baseline"))
        import run_reference

        run_reference.main(args, ClockSampler, base_record, emit, time_device, time_wall, random_batches,
                           max_over_ranks, METRIC, MODEL_DESC)
        return
    run_mine(args)


if __name__ == "__main__":
    main()
