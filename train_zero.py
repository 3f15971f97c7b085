"""ZeRO stage 0-3 training driver.

Flag surface, stdout step line, per-step profile records, profile JSON and per-rank checkpoint
files follow the reference's ``train_zero.py`` (``train_zero.py:49-117, 416-771``) so the
experiment harness and the analysis tools read either program's output.  Extensions (all
additive): ``--collective-impl nvls|p2p`` (this repo's NVLink kernels), ``--backend``, explicit
model-shape overrides and the benchmark presets, ``--data-mode random``, ``--resume PATH``, and
extra profile keys (``iteration_ms_max_over_ranks``, ``exposed_comm_ms``).  ``tokens/s`` uses the
device-timed iteration time maximised over ranks.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import time
from contextlib import nullcontext
from dataclasses import asdict
from pathlib import Path
from typing import Dict, Iterator, List, Optional

import torch
import torch.distributed as dist

from cs244c_llama_zero_b200 import ops
from cs244c_llama_zero_b200.models import LlamaForCausalLM, estimate_num_parameters, human_readable_count
from cs244c_llama_zero_b200.parallel.collectives import TracingCollectives, aggregate_collective_trace, pick_collectives
from cs244c_llama_zero_b200.parallel.zero import (
    ZeROStage0DDP,
    ZeROStage1Optimizer,
    ZeROStage2Optimizer,
    ZeROStage3Optimizer,
)
from cs244c_llama_zero_b200.profiler import (
    FlopTracker,
    MemoryTracker,
    TimerRegistry,
    estimate_transformer_train_flops,
    executed_train_flops,
    flops_to_tflops_per_second,
    overlap_efficiency,
    peak_bf16_tflops,
    roofline_fraction,
)
from cs244c_llama_zero_b200.profiler import nvtx
from cs244c_llama_zero_b200.profiler.nvtx import nvtx_range
from cs244c_llama_zero_b200.train.faults import FaultInjector
from cs244c_llama_zero_b200.train.session import init_distributed
from train import (
    add_data_args,
    add_model_args,
    autocast_context,
    batch_from_chunk,
    make_data_loader,
    model_config_from_args,
    model_param_dtype,
    resolve_backend,
    set_seed,
)

STEP_COMM_KEYS = [
    f"communication_{phase}_{field}"
    for phase in ("backward_reduce_scatter", "post_allgather", "forward_allgather", "backward_allgather")
    for field in ("ms", "calls", "bytes")
]


def log_event(rank: int, message: str, *, force: bool = True) -> None:
    if force:
        print(f"[{time.strftime('%H:%M:%S')}][rank {rank}] {message}", flush=True)


def format_device_memory(device: torch.device) -> str:
    if device.type != "cuda" or not torch.cuda.is_available():
        return "host-only"
    mb = 1024.0 * 1024.0
    return (f"cuda_allocated_mb={torch.cuda.memory_allocated(device) / mb:.1f} "
            f"cuda_reserved_mb={torch.cuda.memory_reserved(device) / mb:.1f} "
            f"cuda_max_allocated_mb={torch.cuda.max_memory_allocated(device) / mb:.1f}")


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="ZeRO stages 0-3 training")
    p.add_argument("--zero-stage", type=int, default=0, choices=[0, 1, 2, 3])
    p.add_argument("--collective-impl", type=str, default="torch", choices=["ring", "torch", "nvls", "p2p"])
    add_model_args(p)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--batch-size", type=int, default=2)
    p.add_argument("--grad-accum-steps", type=int, default=1)
    p.add_argument("--max-steps", type=int, default=200)
    p.add_argument("--learning-rate", type=float, default=3e-4)
    p.add_argument("--weight-decay", type=float, default=0.1)
    p.add_argument("--beta1", type=float, default=0.9)
    p.add_argument("--beta2", type=float, default=0.95)
    p.add_argument("--eps", type=float, default=1e-8)
    p.add_argument("--max-grad-norm", type=float, default=0.0)
    p.add_argument("--stage2-grad-bucket-mb", type=float, default=64.0,
                   help="Compatibility knob; stage 2 reduce-scatters one contiguous gradient buffer per backward.")
    p.add_argument("--dtype", type=str, default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--seed", type=int, default=1337)
    p.add_argument("--loss-chunk-size", type=int, default=128)
    p.add_argument("--activation-checkpointing", dest="activation_checkpointing", action="store_true")
    p.add_argument("--no-activation-checkpointing", dest="activation_checkpointing", action="store_false")
    add_data_args(p, default_mode="synthetic")
    p.add_argument("--log-interval", type=int, default=10)
    p.add_argument("--checkpoint-interval", type=int, default=100)
    p.add_argument("--save-dir", type=str, default="checkpoints")
    p.add_argument("--resume", type=str, default="", help="per-rank checkpoint path; {rank} is substituted")
    p.add_argument("--profile-json", type=str, default="")
    p.add_argument("--profile-memory-interval", type=int, default=0)
    p.add_argument("--profile-rank0-only", action="store_true")
    p.add_argument("--profile-collectives", action="store_true")
    p.add_argument("--measure-memory-step", action="store_true")
    p.add_argument("--memory-warmup-steps", type=int, default=0)
    p.add_argument("--tflops-mode", type=str, default="estimate", choices=["estimate", "profile", "off"])
    p.add_argument("--nvtx", action="store_true", help="name the step phases with NVTX ranges (Nsight timelines)")
    p.add_argument("--routed-grads", action="store_true",
                   help="stage 2 with --collective-impl nvls|p2p: no full gradient buffer; gradients are added into "
                        "their owners' shards over NVLink during backward")
    p.add_argument("--fused-step", action="store_true",
                   help="stages 1/2 with --collective-impl nvls|p2p and no clipping: the step as one NVLink kernel "
                        "(reduce-scatter + norm + AdamW + all-gather)")
    p.add_argument("--verbose", action="store_true")
    p.add_argument("--verbose-memory", action="store_true")
    p.add_argument("--stage3-recompute", action="store_true",
                   help="ZeRO-3: re-run every module in backward (the reference's behaviour) instead of keeping "
                        "the activations of modules on the B200 kernels")
    p.add_argument("--pg-timeout-s", type=float, default=600.0,
                   help="Process-group timeout: a collective waiting longer than this on a missing rank fails")
    p.set_defaults(activation_checkpointing=False)
    return p.parse_args(argv)


def configure_runtime(device: torch.device) -> None:
    if device.type == "cuda":
        torch.backends.cuda.matmul.allow_tf32 = True
        torch.backends.cudnn.allow_tf32 = True
        torch.backends.cudnn.benchmark = True
        torch.set_float32_matmul_precision("high")


def broadcast_model(model: torch.nn.Module) -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        for p in model.parameters():
            dist.broadcast(p.data, src=0)


def build_engine(args: argparse.Namespace, model, collectives):
    kwargs = dict(model=model, lr=args.learning_rate, betas=(args.beta1, args.beta2), eps=args.eps,
                  weight_decay=args.weight_decay, collectives=collectives)
    if args.zero_stage == 0:
        return ZeROStage0DDP(**kwargs)
    if args.zero_stage == 1:
        return ZeROStage1Optimizer(**kwargs)
    if args.zero_stage == 2:
        return ZeROStage2Optimizer(**kwargs, grad_bucket_numel=max(1, int(args.stage2_grad_bucket_mb * 1024 * 1024 / 4)))
    return ZeROStage3Optimizer(**kwargs, recompute=args.stage3_recompute)


def global_mean_scalar(value: float, device: torch.device, world_size: int) -> float:
    t = torch.tensor([value], dtype=torch.float32, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(t)
    return float(t.item() / world_size)


def global_max_scalar(value: float, device: torch.device) -> float:
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def checkpoint_path(save_dir: str, stage: int, step: int, rank: int) -> str:
    return os.path.join(save_dir, f"zero_stage{stage}_step{step:06d}_rank{rank:03d}.pt")


def save_checkpoint(save_dir: str, step: int, rank: int, model, engine, args, extra: Dict[str, object]) -> str:
    os.makedirs(save_dir, exist_ok=True)
    path = checkpoint_path(save_dir, args.zero_stage, step, rank)
    ctx = engine.summon_full_params() if hasattr(engine, "summon_full_params") else nullcontext()
    with ctx:
        model_state = {k: v.detach().cpu() for k, v in model.state_dict().items()}
    torch.save({"step": step, "rank": rank, "model_state_dict": model_state, "engine_state_dict": engine.state_dict(),
                "train_args": vars(args), "extra": extra}, path)
    return path


def load_checkpoint(path: str, rank: int, model, engine) -> int:
    payload = torch.load(path.format(rank=rank), map_location="cpu", weights_only=False)
    ctx = engine.summon_full_params() if hasattr(engine, "summon_full_params") else nullcontext()
    with ctx:
        model.load_state_dict(payload["model_state_dict"])
    engine.load_state_dict(payload["engine_state_dict"])
    return int(payload["step"])


class MemoryRecorder:
    """Labelled memory snapshots with peak observation (reference ``train_zero.py:376-401``)."""

    def __init__(self, memory: MemoryTracker, engine, enabled: bool, rank: int, log: bool) -> None:
        self.memory = memory
        self.enabled = enabled
        self.rank = rank
        self.log = log
        self.live = getattr(engine, "live_model_state_breakdown_mb", None) or getattr(engine, "memory_state_breakdown_mb", None)
        self.debug = getattr(engine, "debug_memory_components_mb", None)
        self.peak_observation: Optional[Dict[str, object]] = None
        self.peak_max = -1.0
        self.timeline: List[Dict[str, object]] = []

    def record(self, label: str, capture_peak: bool, timeline: bool = False) -> None:
        if not self.enabled:
            return
        snap = self.memory.record(label)
        if timeline and self.live is not None:
            self.timeline.append({"label": label, **self.live()})
        if self.log:
            log_event(self.rank, f"recorded memory snapshot {label} {format_device_memory(self.memory.device)}")
        if not capture_peak or snap.cuda_max_allocated_mb <= self.peak_max + 1e-6:
            return
        self.peak_max = snap.cuda_max_allocated_mb
        obs = {"label": label, "timestamp_s": snap.timestamp_s, "allocated_mb": snap.cuda_allocated_mb,
               "reserved_mb": snap.cuda_reserved_mb, "max_allocated_mb": snap.cuda_max_allocated_mb,
               "max_reserved_mb": snap.cuda_max_reserved_mb}
        if self.live is not None:
            obs["live_state_breakdown_mb"] = self.live()
        if callable(self.debug):
            obs["debug_memory_components_mb"] = self.debug()
        self.peak_observation = obs


def train(args: argparse.Namespace) -> None:
    rank, world_size, device = init_distributed(args.pg_timeout_s)
    faults = FaultInjector(rank)
    verbose = bool(args.verbose)
    if getattr(args, "nvtx", False):
        nvtx.enable(True)
    if getattr(args, "fused_step", False):
        os.environ["ZB_FUSED_STEP"] = "1"  # read by the stage 1/2 engines when they are built
    if getattr(args, "routed_grads", False):
        os.environ["ZB_ROUTED_GRADS"] = "1"
    configure_runtime(device)
    set_seed(args.seed)
    log_event(rank, f"initialized distributed world_size={world_size} device={device} pid={os.getpid()}", force=verbose)
    base_vocab = args.synthetic_vocab_size
    try:
        loader, vocab, metadata = make_data_loader(args, vocab_size_for_model=base_vocab, rank=rank, world_size=world_size)
    except Exception as exc:
        if not args.allow_synthetic_fallback:
            raise
        if rank == 0:
            print(f"[warn] data init failed ({exc}); falling back to synthetic")
        args.data_mode = "synthetic"
        loader, vocab, metadata = make_data_loader(args, vocab_size_for_model=base_vocab, rank=rank, world_size=world_size)
    cfg = model_config_from_args(args, vocab)
    dtype = model_param_dtype(device, args.dtype)
    model = LlamaForCausalLM(cfg).to(device=device, dtype=dtype)
    model.set_loss_chunk_size(args.loss_chunk_size)
    model.set_activation_checkpointing(args.activation_checkpointing)
    backend = resolve_backend(args, device, dtype)
    model.set_backend(backend)
    check_device_waits = device.type == "cuda" and (backend == "b200" or args.collective_impl in ("nvls", "p2p"))
    broadcast_model(model)
    collectives = pick_collectives(world_size, args.collective_impl, device)
    if args.profile_collectives:
        collectives = TracingCollectives(collectives)
    engine = build_engine(args, model, collectives)
    start_step = 1
    if args.resume:
        start_step = load_checkpoint(args.resume, rank, model, engine) + 1
        if rank == 0:
            print(f"[resume] continuing from step {start_step - 1} ({args.resume})", flush=True)
    n_params = estimate_num_parameters(cfg)
    if rank == 0:
        print(f"[init] stage={args.zero_stage} impl={args.collective_impl} world_size={world_size} model={cfg.name} "
              f"params={human_readable_count(n_params)} ({n_params:,}) vocab={cfg.vocab_size:,} "
              f"seq_len={cfg.max_seq_len} device={device} dtype={args.dtype} backend={backend}", flush=True)
        print(f"[init] data_mode={args.data_mode} metadata={json.dumps(metadata)}", flush=True)

    global_tokens = args.batch_size * args.grad_accum_steps * args.seq_len * world_size
    data_iter: Iterator[torch.Tensor] = iter(loader)
    timers = TimerRegistry(device=device)
    flop_tracker = FlopTracker(device=device) if rank == 0 and args.tflops_mode == "profile" else None
    memory = MemoryTracker(device=device)
    profile_enabled = bool(args.profile_json) and (rank == 0 or not args.profile_rank0_only)
    record_memory = args.profile_memory_interval > 0 or args.measure_memory_step
    measured_step = args.memory_warmup_steps + 1 if args.measure_memory_step else None
    if args.measure_memory_step and args.max_steps < measured_step:
        raise ValueError(f"max_steps={args.max_steps} is too small for memory warmup + measured step; need at least "
                         f"{measured_step}")
    recorder = MemoryRecorder(memory, engine, record_memory and profile_enabled, rank, args.verbose_memory)
    engine.memory_tracker = memory
    engine.memory_trace_active = False
    engine.memory_state_timeline = recorder.timeline
    if recorder.enabled and not args.measure_memory_step:
        memory.record("start")
    step_flops = None
    if args.tflops_mode == "estimate":
        step_flops = estimate_transformer_train_flops(cfg, args.batch_size, args.seq_len, args.grad_accum_steps,
                                                      world_size, stage=args.zero_stage)
    # roofline: the FLOPs this GPU really executes per step (no 4x stage-3 convention) over the peak
    executed_flops = executed_train_flops(cfg, args.batch_size, args.seq_len,
                                          recompute_forward=args.zero_stage == 3 and (
                                              backend != "b200" or bool(getattr(args, "stage3_recompute", False)))
                                          ) * args.grad_accum_steps
    peak_tflops, peak_source = peak_bf16_tflops()
    step_profiles: List[Dict[str, object]] = []
    measured_step_memory = None
    recent: List[float] = []
    t_start = time.perf_counter()

    for step in range(start_step, args.max_steps + 1):
        if faults:
            faults.at_step(step, collectives)
        sample = args.profile_memory_interval > 0 and (step == 1 or step == args.max_steps
                                                       or step % args.profile_memory_interval == 0)
        is_measured = measured_step is not None and step == measured_step
        prefix = f"measured_step_{step}" if is_measured else f"step_{step}"
        snap = (lambda label, timeline=is_measured: recorder.record(f"{prefix}_{label}", capture_peak=is_measured,
                                                                    timeline=timeline)) \
            if (is_measured or sample) else (lambda label, timeline=False: None)
        if args.profile_collectives:
            collectives.consume_trace()
        iter_timer = timers.timer("iteration")
        iter_timer.start()
        model.train()
        engine.zero_grad()
        if is_measured:
            memory.reset_peak_stats()
            engine.memory_trace_active = recorder.enabled
        snap("start")
        nvtx.mark(f"step {step}")
        with nvtx_range("prepare_forward"):
            prepare_comm_ms = float(engine.prepare_forward().get("prepare_comm_ms", 0.0))
        snap("post_prepare")
        fb_timer = timers.timer("forward_backward")
        fb_timer.start()

        loss_scales: Dict[int, torch.Tensor] = {}

        def loss_scale_context(n: int):
            """B200 backend: each micro-batch loss is back-propagated as loss / n, so the LM head may
            compute its gradients during the forward pass (no [tokens, vocab] logits tensor)."""
            if backend != "b200" or device.type != "cuda":
                return contextlib.nullcontext()
            from cs244c_llama_zero_b200.ops import functional as B

            if n not in loss_scales:
                loss_scales[n] = torch.full((), 1.0 / n, dtype=torch.float32, device=device)
            return B.loss_gradient_scale(loss_scales[n])

        def run_microbatches() -> List[torch.Tensor]:
            nonlocal data_iter
            losses = []
            for micro in range(args.grad_accum_steps):
                try:
                    chunk = next(data_iter)
                except StopIteration:
                    data_iter = iter(loader)
                    chunk = next(data_iter)
                batch = batch_from_chunk(chunk)
                ids = batch.input_ids.to(device, non_blocking=True)
                labels = batch.labels.to(device, non_blocking=True)
                with nvtx_range(f"forward.micro{micro + 1}"), autocast_context(device, args.dtype), \
                        loss_scale_context(args.grad_accum_steps):
                    loss = model(input_ids=ids, labels=labels, return_logits=False).loss
                snap(f"micro_{micro + 1}_after_forward")
                losses.append(loss.detach().float())
                with nvtx_range(f"backward.micro{micro + 1}"):
                    engine.backward(loss / args.grad_accum_steps)
                snap(f"micro_{micro + 1}_after_backward")
            return losses

        if flop_tracker is not None and step_flops is None:
            micro_losses, profiled = flop_tracker.measure(label=f"step_{step}", fn=run_microbatches)
            if profiled is not None:
                step_flops = profiled * world_size
        else:
            micro_losses = run_microbatches()
        fb_ms = fb_timer.stop()
        snap("post_backward")
        opt_timer = timers.timer("optimizer_step")
        opt_timer.start()
        with nvtx_range("optimizer"):
            stats = engine.step_with_stats(max_grad_norm=args.max_grad_norm)
        opt_timer.stop()
        grad_norm = float(stats["grad_norm"])
        comm_ms = float(stats["comm_ms"]) + prepare_comm_ms
        snap("post_optimizer")
        local_loss = float(torch.stack(micro_losses).mean())
        if check_device_waits:  # a kernel whose bounded wait expired (e.g. a peer never signalled) ends the run
            ops.check_device_errors()
        step_loss = global_mean_scalar(local_loss, device, world_size)
        recent = (recent + [step_loss])[-100:]
        iter_ms = iter_timer.stop()
        iter_ms_max = global_max_scalar(iter_ms, device)
        step_time = iter_ms_max / 1000.0
        tokens_per_second = global_tokens / max(step_time, 1e-8)
        tflops = flops_to_tflops_per_second(step_flops, step_time) if step_flops is not None else None
        compute_ms = max(iter_ms - comm_ms, 0.0)
        overlap = overlap_efficiency(iter_ms, compute_ms, comm_ms)
        if rank == 0 and (step % args.log_interval == 0 or step == 1 or step == args.max_steps):
            print(f"[step {step:05d}] loss={step_loss:.4f} avg100={sum(recent) / len(recent):.4f} "
                  f"tokens/s={tokens_per_second:,.0f} grad_norm={grad_norm:.3f} fb_ms={fb_ms:.2f} "
                  f"comm_ms={comm_ms:.2f} opt_ms={float(stats['optim_ms']):.2f}"
                  + (f" tflops={tflops:.3f}" if tflops is not None else ""), flush=True)
        trace, trace_summary = [], []
        if args.profile_collectives:
            trace = collectives.consume_trace()
            trace_summary = aggregate_collective_trace(trace)
        if profile_enabled:
            record = {"step": step, "loss": step_loss, "tokens_per_second": tokens_per_second,
                      "tflops_per_second": tflops, "grad_norm": grad_norm, "forward_backward_ms": fb_ms,
                      "communication_ms": comm_ms, "optimizer_ms": float(stats["optim_ms"]), "iteration_ms": iter_ms,
                      "iteration_ms_max_over_ranks": iter_ms_max,
                      "executed_tflops_per_gpu": executed_flops / max(iter_ms_max, 1e-6) / 1e9,
                      "roofline_fraction": roofline_fraction(executed_flops, iter_ms_max / 1000.0, peak_tflops)}
            for key in STEP_COMM_KEYS:
                record[key] = float(stats.get(key, 0.0))
            record.update({"collective_trace": trace, "collective_trace_summary": trace_summary,
                           "overlap_ratio": overlap, "exposed_comm_ms": max(0.0, iter_ms - fb_ms - float(stats["optim_ms"]))})
            step_profiles.append(record)
        if is_measured and recorder.enabled:
            snap("end")
            peaks = memory.peak_stats_mb()
            measured_step_memory = {"step": step, "warmup_steps": args.memory_warmup_steps,
                                    "peak_allocated_mb": peaks["peak_allocated_mb"],
                                    "peak_reserved_mb": peaks["peak_reserved_mb"]}
            if recorder.peak_observation is not None:
                measured_step_memory["peak_observation"] = recorder.peak_observation
            engine.memory_trace_active = False
        elif sample:
            snap("end")
        if args.checkpoint_interval > 0 and (step % args.checkpoint_interval == 0 or step == args.max_steps):
            path = save_checkpoint(args.save_dir, step, rank, model, engine, args,
                                   {"model_config": cfg.to_dict(), "step_loss": step_loss})
            if rank == 0:
                print(f"[checkpoint] wrote {path}", flush=True)

    if rank == 0:
        print(f"[done] trained {args.max_steps} steps in {time.perf_counter() - t_start:.1f}s", flush=True)
    if profile_enabled:
        overlap_summary = None
        if step_profiles:
            vals = [float(s["overlap_ratio"]) for s in step_profiles]
            overlap_summary = {"mean": sum(vals) / len(vals), "min": min(vals), "max": max(vals)}
        trace_summary = None
        if step_profiles and args.profile_collectives:
            combined = [r for s in step_profiles for r in s.get("collective_trace", [])]
            trace_summary = aggregate_collective_trace(combined)
        payload = {
            "rank": rank, "world_size": world_size, "stage": args.zero_stage, "collective_impl": args.collective_impl,
            "args": vars(args), "model_config": cfg.to_dict(),
            "optimizer_config": {"lr": args.learning_rate, "betas": [args.beta1, args.beta2], "eps": args.eps,
                                 "weight_decay": args.weight_decay, "max_grad_norm": args.max_grad_norm},
            "global_batch_size": args.batch_size * args.grad_accum_steps * world_size,
            "microbatch_size_per_gpu": args.batch_size, "overlap_enabled": False,
            "timers": {name: asdict(s) for name, s in timers.summarize().items()},
            "memory": memory.as_dicts() if record_memory else [],
            "flops": {"measurements": flop_tracker.as_dicts() if flop_tracker is not None else [],
                      "profiled_step_flops": step_flops, "tflops_mode": args.tflops_mode},
            "steps": step_profiles, "collective_trace_summary": trace_summary,
            "state_memory_breakdown_mb": engine.memory_state_breakdown_mb(), "overlap_summary": overlap_summary,
            "measured_step_memory": measured_step_memory, "measured_step_state_timeline": recorder.timeline,
            "backend": backend,
            "roofline": {"executed_flops_per_gpu_step": executed_flops, "peak_bf16_tflops": peak_tflops,
                         "peak_source": peak_source},
        }
        path = Path(args.profile_json)
        if world_size > 1 and not args.profile_rank0_only:
            path = path.with_suffix(f".rank{rank:03d}.json")
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(payload, indent=2))
        print(f"[profile] wrote {path}", flush=True)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def main(argv=None) -> None:
    train(parse_args(argv))


if __name__ == "__main__":
    main()
