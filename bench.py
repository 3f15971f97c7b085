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
# BASELINE.json shapes: model dimensions and the per-GPU micro-batch / sequence length they are run at.
CONFIG_SHAPES = {
    "baseline-small": dict(dim=768, n_layers=12, n_heads=12, n_kv_heads=4, ffn_dim=2048, batch=8, seq=1024),
    "baseline-1.3b": dict(dim=2048, n_layers=24, n_heads=16, n_kv_heads=8, ffn_dim=5504, batch=4, seq=2048),
}
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
    p.add_argument("--cuda-graph", nargs="?", const="on", default="auto", choices=["auto", "on", "off"],
                   help="run stages 0-2 as one captured CUDA graph per step (TrainSession cuda_graph mode); "
                        "auto (default): on for one GPU, where it measured 8.04-8.08 vs 8.41-8.44 ms per step")
    p.add_argument("--model-size", type=str, default="baseline-small",
                   help="model preset of the headline: baseline-small (the headline config), baseline-1.3b, ...")
    p.add_argument("--extra-configs", type=str, default="baseline-1.3b",
                   help="comma-separated presets measured after the headline at their BASELINE shapes (every "
                        "stage, same steps and warm-up), reported under per_config; '' for none")
    args = p.parse_args(argv)
    args.warmup = max(3, args.warmup)
    args.stage_list = [int(s) for s in args.stages.split(",") if s.strip()]
    args.extra_list = [c.strip() for c in args.extra_configs.split(",") if c.strip() and c.strip() != args.model_size]
    if args.headline_stage not in args.stage_list:
        args.headline_stage = args.stage_list[0]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    args.cuda_graph = args.cuda_graph == "on" or (args.cuda_graph == "auto" and world == 1)
    return args


# ----------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons while the timed region runs.

    Through ``nvidia-smi -lms 50`` (default), or with ``ZB_CLOCK_SAMPLER=nvml`` through NVML every
    5 ms on a background thread (a 20-step region of ~9 ms steps then gets dozens of samples).
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}
    PERIOD_S = 0.005

    def __init__(self, gpu_indices, path=None):
        self.gpu_indices = set(gpu_indices)
        self.proc = None
        self.thread = None
        self.samples = []  # (index, sm_mhz, max_mhz, reason names)
        # nvidia-smi fallback: the raw samples go to --clocks-csv when given (kept), else to a temp file
        self.path = path or os.path.join(tempfile.gettempdir(), f"zb_clocks_{os.getpid()}.csv")
        self.keep_csv = path is not None

    def _nvml_loop(self, nvml, handles):
        import threading  # noqa: F401

        while not self._stop.is_set():
            for idx, h in handles:
                try:
                    mhz = nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM)
                    max_mhz = nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM)
                    bits = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:  # noqa: BLE001 - a failed read is a missing sample
                    continue
                names = [n for n, b in self.REASON_BITS.items() if bits & b]
                self.samples.append((idx, float(mhz), float(max_mhz), names))
            self._stop.wait(self.PERIOD_S)

    def __enter__(self):
        import threading

        try:
            if os.environ.get("ZB_CLOCK_SAMPLER", "smi") != "nvml":
                raise RuntimeError("nvidia-smi sampler selected")
            import pynvml as nvml

            nvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            order = [int(x) for x in visible.split(",")] if visible and all(
                x.strip().isdigit() for x in visible.split(",")) else None
            handles = []
            for idx in sorted(self.gpu_indices):
                phys = order[idx] if order and idx < len(order) else idx
                handles.append((idx, nvml.nvmlDeviceGetHandleByIndex(phys)))
            self._nvml = nvml
            self._stop = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nvml, handles), daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001 - no NVML bindings / driver: use the CLI
            self.thread = None
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            try:
                self._nvml.nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass
            if self.keep_csv:
                with open(self.path, "w") as fh:
                    for idx, mhz, mx, names in self.samples:
                        fh.write(f"{idx}, {mhz:.0f}, {mx:.0f}, {'|'.join(names) or 'none'}\n")
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()
            self._read_csv()

    def _read_csv(self):
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        if not os.path.exists(self.path):
            return
        with open(self.path) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    idx, mhz, mx = int(parts[0]), float(parts[1]), float(parts[2])
                except ValueError:
                    continue
                if self.gpu_indices and idx not in self.gpu_indices:
                    continue
                active = [n for n, v in zip(names[1:], parts[5:9]) if v.lower().startswith("active")]
                self.samples.append((idx, mhz, mx, active))

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        mhz = [x[1] for x in self.samples]
        loaded = [m for m in mhz if m > 0.5 * max(mhz)] or mhz
        reasons = sorted({n for x in self.samples for n in x[3]})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(x[2] for x in self.samples),
                "reasons": reasons, "samples": len(mhz),
                "source": "nvml" if self.thread is not None else "nvidia-smi"}


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


def progress(rank: int, msg: str) -> None:
    """One timestamped line on stderr per phase (the JSON result goes to stdout at the end)."""
    if rank == 0:
        print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


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
def roofline_entry(sess, batch: int, seq: int, stage: int, ms: float, peak_tflops: float) -> dict:
    """Executed tensor-core TFLOP/s of one GPU's step (causal attention halved, no recompute unless the
    stage-3 engine recomputes) and its fraction of the peak."""
    from cs244c_llama_zero_b200.profiler import executed_train_flops, roofline_fraction

    recompute = stage == 3 and bool(getattr(sess.engine, "recompute", False))
    executed = executed_train_flops(sess.model_cfg, batch, seq, recompute_forward=recompute)
    return {"executed_tflops_per_gpu": executed / (ms / 1000.0) / 1e12,
            "roofline_fraction": roofline_fraction(executed, ms / 1000.0, peak_tflops)}


def _measure_stages(args, size: str, batch: int, seq: int, world: int, rank: int, local: int, impl: str,
                    peak_tflops: float, headline: bool) -> dict:
    """Every stage of ``args.stage_list`` on one model config: W warm-up steps, then K device-timed
    steps (max over ranks), then one instrumented step for comm_ms.  With ``headline`` the headline
    stage also gets the clock samples, the launch count and the end-to-end run."""
    import torch

    from cs244c_llama_zero_b200 import ops
    from cs244c_llama_zero_b200.models import BASELINE_VOCAB_SIZE
    from cs244c_llama_zero_b200.train import SessionConfig, TrainSession

    out = {"per_stage": {}, "e2e": None, "launches": None, "clocks": None, "headline_ms": None}
    tokens_per_step = batch * seq * world
    for stage in args.stage_list:
        progress(rank, f"{size} stage {stage}: building (B{batch} S{seq})")
        sess = TrainSession(SessionConfig(model_size=size, vocab_size=BASELINE_VOCAB_SIZE,
                                          seq_len=seq, batch_size=batch, zero_stage=stage,
                                          collective_impl=impl, backend="b200",
                                          cuda_graph=args.cuda_graph and stage != 3))
        host = random_batches(4, batch, seq, BASELINE_VOCAB_SIZE, seed=1234 + rank * 100 + stage)
        dev = [h.to(sess.device) for h in host]
        it = {"i": 0}

        debug = os.environ.get("ZB_BENCH_DEBUG", "0") == "1"

        def device_step():
            sess.train_step(dev[it["i"] % len(dev)])
            it["i"] += 1
            if debug:  # diagnosis only: per-step synchronisation (timings are not valid then)
                torch.cuda.synchronize()
                progress(rank, f"{size} stage {stage}: step {it['i']} done, device errors "
                               f"{list(ops.load_extension().read_device_errors())}")

        is_head = headline and stage == args.headline_stage
        # The sampler starts before the warm-up so that short timed regions still get samples taken
        # under steady load; it stops right after the timed steps.
        sampler = ClockSampler([local], args.clocks_csv) if is_head and rank == 0 else None
        if sampler:
            sampler.__enter__()
        for _ in range(args.warmup):
            device_step()
        torch.cuda.synchronize()
        progress(rank, f"{size} stage {stage}: warm-up done")
        launches_before = ops.launch_count()
        ms = time_device(device_step, args.steps)
        progress(rank, f"{size} stage {stage}: {ms:.3f} ms/step")
        if sampler:
            sampler.__exit__(None, None, None)
            out["clocks"] = sampler.summary()
        stage_launches = (ops.launch_count() - launches_before) // args.steps
        entry = {"tokens_per_s": tokens_per_step / (ms / 1000.0), "ms_per_step": ms,
                 "gpu_launches_per_step": stage_launches}
        if stage == 2:
            entry["gradient_mode"] = getattr(sess.engine, "gradient_mode", "full")
        entry.update(roofline_entry(sess, batch, seq, stage, ms, peak_tflops))
        # comm time of one extra instrumented step (device events around each collective); the
        # barrier keeps host-side skew between ranks out of the measured intervals
        barrier_sync()
        sess.engine.clock.timing = True  # an eager instrumented step, also in graph mode
        sess.engine.zero_grad()
        sess.engine.prepare_forward()
        sess.forward_backward([dev[0]])
        st = sess.engine.step_with_stats(max_grad_norm=0.0)
        entry["comm_ms"] = max_over_ranks(float(st["comm_ms"]))
        if is_head:
            out["headline_ms"] = ms
            out["launches"] = stage_launches * args.steps
            if not args.no_e2e:
                out["e2e"] = _e2e(sess, host, it, args.steps, tokens_per_step)
        out["per_stage"][str(stage)] = entry
        del sess
        torch.cuda.empty_cache()
    return out


def _e2e(sess, host, it, steps: int, tokens_per_step: int) -> dict:
    """K steps through the public API: each step's pinned host batch is copied in by train_step and its
    loss (+ the kernels' error record) comes back to the host, read one step later."""
    h2d = host[0].numel() * host[0].element_size()
    pending = []
    losses = []
    d2h = {"n": 0}

    def e2e_step():
        pending.append(sess.train_step_async(host[it["i"] % len(host)]))
        d2h["n"] = pending[-1].nbytes  # loss + the kernels' error record
        it["i"] += 1
        if len(pending) > 1:
            losses.append(pending.pop(0).item())

    def e2e_finish():  # the last step's loss is read inside the timed region too
        while pending:
            losses.append(pending.pop(0).item())

    for _ in range(2):
        e2e_step()
    e2e_finish()
    losses.clear()
    e2e_ms = time_wall(e2e_step, steps, finish=e2e_finish)
    if len(losses) != steps or not all(math.isfinite(x) for x in losses):
        raise RuntimeError(f"e2e: expected {steps} finite losses, got {losses}")
    return {"value": tokens_per_step / (e2e_ms / 1000.0), "unit": "tokens/s",
            "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h["n"],
            "api": "cs244c_llama_zero_b200.train.TrainSession.train_step_async(pinned host int64 [B,S])"
                   " + AsyncLoss.item() one step later (every step's loss and error record read on the host)"}


def run_mine(args) -> None:
    import torch.distributed as dist

    from cs244c_llama_zero_b200 import ops
    from cs244c_llama_zero_b200.profiler import peak_bf16_tflops

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
    head = _measure_stages(args, args.model_size, args.batch_size, args.seq_len, world, rank, local, impl,
                           peak_tflops, headline=True)
    per_config = {}
    for size in args.extra_list:
        shape = CONFIG_SHAPES[size]
        extra = _measure_stages(args, size, shape["batch"], shape["seq"], world, rank, local, impl, peak_tflops,
                                headline=False)
        per_config[size] = {"model": model_desc(size), "global_batch": shape["batch"] * world,
                            "micro_batch_per_gpu": shape["batch"], "seq_len": shape["seq"],
                            "per_stage": extra["per_stage"]}
    errors = ops.load_extension().read_device_errors()
    rec = base_record(args, world, "mine")
    hs = head["per_stage"][str(args.headline_stage)]
    rec.update({
        "value": hs["tokens_per_s"],
        "ms_per_step": head["headline_ms"],
        "config": {"model": model_desc(args.model_size), "global_batch": args.batch_size * world,
                   "micro_batch_per_gpu": args.batch_size,
                   "seq_len": args.seq_len, "grad_accum": 1, "parallelism": f"dp{world}",
                   "zero_stage": args.headline_stage, "collective_impl": impl,
                   "cuda_graph": bool(args.cuda_graph and args.headline_stage != 3),
                   "fused_step": bool(args.fused_step),
                   "routed_grads": bool(args.routed_grads),
                   "l2": "no flush: each step touches >2 GB (activations, 1.2 GB fp32 optimizer state) vs 126 MB L2"},
        "per_stage": head["per_stage"],
        "per_config": per_config,
        "roofline": {"executed_tflops_per_gpu": hs["executed_tflops_per_gpu"],
                     "fraction": hs["roofline_fraction"], "peak_bf16_tflops": peak_tflops,
                     "peak_source": peak_source, "note": "of measured sustained cuBLAS bf16 GEMM peak"
                     if peak_source == "measured" else "of fallback peak"},
        "e2e": head["e2e"],
        "gpu_launches": head["launches"],
        "clocks": head["clocks"],
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
                           max_over_ranks, METRIC, MODEL_DESC, CONFIG_SHAPES)
        return
    run_mine(args)


if __name__ == "__main__":
    main()
