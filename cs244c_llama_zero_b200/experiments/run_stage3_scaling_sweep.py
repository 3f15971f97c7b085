"""ZeRO stage-3 GPU-count scaling sweep (the ZeRO paper's Figure-3 idea on one node).

For each GPU count (ascending) the per-GPU micro-batch is tuned to the OOM boundary - the first probe
predicted from earlier GPU counts (``tuning.predict_initial_batch_size``) - then benchmarked without
bandwidth shaping.  ``--fixed-batch-size`` skips tuning and benchmarks one micro-batch everywhere.
``summary.json`` carries per-GPU-count tuning records and ``scaling_points`` with speedup and scaling
efficiency against the smallest GPU count.  Same flags and outputs as the reference's
``experiments/run_stage3_scaling_sweep.py``.

    python -m cs244c_llama_zero_b200.experiments.run_stage3_scaling_sweep --gpu-counts 1 2 4 8 \
        --model-size baseline-1.3b --seq-len 1024 --tflops-mode estimate
"""

from __future__ import annotations

import argparse
import itertools
from dataclasses import asdict
from pathlib import Path
from typing import Dict, List, Optional

from . import harness
from .common import add_launch_args, add_run_args, add_training_args, add_tuning_args, make_case, \
    parse_with_config, write_json
from .tuning import (TuningTrial, detect_gpu_total_memory_mb, memory_probe_extra_args, predict_initial_batch_size,
                     search_max_batch_size, trial_from_result)

_predict_initial_batch_size = predict_initial_batch_size  # name used by the reference's tests


def _build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Sweep ZeRO Stage 3 across GPU counts with OOM-boundary microbatch tuning")
    add_run_args(p, "stage3_gpu_scaling")
    p.add_argument("--gpu-counts", nargs="+", type=int, default=[1, 2, 4, 8])
    add_launch_args(p, nproc=None, timeout_s=3600.0)
    add_training_args(p, model_size="medium", steps=10, seq_len=256)
    p.add_argument("--tflops-mode", type=str, default="estimate", choices=["estimate", "profile", "off"])
    p.add_argument("--profile-collectives", action="store_true")
    add_tuning_args(p, max_batch=64, multiple=1, fit_modes=["oom_boundary"])
    p.add_argument("--tuning-strategy", type=str, default="predictive", choices=["predictive", "exponential"],
                   help="'predictive' seeds each GPU count's search from the earlier fits.")
    p.add_argument("--fixed-batch-size", type=int, default=0,
                   help="If >0, skip tuning and benchmark this per-GPU microbatch for every GPU count.")
    return p


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    return parse_with_config(_build_parser(), argv, matrix_keys=("gpu_counts",))


def _gpu_counts(values) -> List[int]:
    counts = sorted({int(v) for v in values if int(v) > 0})
    if not counts:
        raise ValueError("gpu_counts must contain at least one positive integer")
    return counts


def _benchmark_extra_args(args: argparse.Namespace) -> str:
    parts = [args.extra_args.strip()] if args.extra_args.strip() else []
    parts.append(f"--tflops-mode {args.tflops_mode}")
    if args.profile_collectives:
        parts.append("--profile-collectives")
    return " ".join(parts)


def scaling_row(gpu_count: int, batch: int, peak_mb: Optional[float], result: harness.CaseResult) -> Dict[str, object]:
    if result.mean_tflops_per_s is None:
        raise RuntimeError(f"missing TFLOPs for gpu_count={gpu_count}; rerun with --tflops-mode estimate or profile")
    cfg = result.config
    return {
        "gpu_count": int(gpu_count), "selected_batch_size": int(batch),
        "selected_peak_memory_mb": None if peak_mb is None else float(peak_mb),
        "global_tokens_per_step": int(cfg["batch_size"] * cfg["grad_accum_steps"] * cfg["seq_len"]
                                      * cfg["nproc_per_node"]),
        "mean_tokens_per_s": result.mean_tokens_per_s, "mean_tflops_per_s": float(result.mean_tflops_per_s),
        "per_gpu_tflops_per_s": float(result.mean_tflops_per_s) / gpu_count,
        "peak_cuda_max_allocated_mb": result.peak_cuda_max_allocated_mb, "mean_comm_ms": result.mean_comm_ms,
        "mean_fb_ms": result.mean_fb_ms, "mean_opt_ms": result.mean_opt_ms, "return_code": int(result.return_code),
        "case_id": result.case_id, "log_path": result.log_path, "profile_path": result.profile_path,
    }


def add_scaling_efficiency(points: List[Dict[str, object]]) -> None:
    """Speedup / efficiency of each point against the smallest GPU count (points sorted in place)."""
    points.sort(key=lambda r: int(r["gpu_count"]))
    if not points:
        return
    n0, t0 = int(points[0]["gpu_count"]), float(points[0]["mean_tflops_per_s"])
    for r in points:
        ideal = int(r["gpu_count"]) / n0
        speedup = float(r["mean_tflops_per_s"]) / t0
        r["perfect_linear_tflops_per_s"] = t0 * ideal
        r["speedup_vs_base"] = speedup
        r["scaling_efficiency_vs_base"] = speedup / ideal
        r["superlinear_gain_vs_perfect_linear"] = float(r["mean_tflops_per_s"]) / (t0 * ideal)


def run(args: argparse.Namespace, per_gpu_total_memory_mb: Optional[float] = None) -> Dict[str, object]:
    counts = _gpu_counts(args.gpu_counts)
    launch = harness._launch_config_from_args(args)
    run_dir = Path(args.results_dir) / args.name
    run_dir.mkdir(parents=True, exist_ok=True)
    if per_gpu_total_memory_mb is None:
        per_gpu_total_memory_mb = detect_gpu_total_memory_mb(max(counts))
    bench_extra = _benchmark_extra_args(args)
    counter = itertools.count()
    fixed = int(args.fixed_batch_size)
    per_count: Dict[str, object] = {}
    results: List[harness.CaseResult] = []
    points: List[Dict[str, object]] = []
    prev_batch: Optional[int] = None
    prev_count: Optional[int] = None
    selected: Dict[int, TuningTrial] = {}
    history: Dict[int, List[TuningTrial]] = {}

    def bench(n: int, batch: int) -> harness.CaseResult:
        case = make_case(args, stage=3, batch_size=batch, bandwidth_gbps=0.0, steps=int(args.steps),
                         metrics_warmup_steps=int(args.metrics_warmup_steps), bandwidth_mode="none",
                         extra_args=bench_extra, nproc_per_node=n)
        print(f"[stage3-scaling] benchmark gpu_count={n} batch_size={batch}", flush=True)
        res = harness._run_case(case, run_dir, args.skip_existing, args.dry_run, launch, next(counter))
        results.append(res)
        return res

    for n in counts:
        if fixed > 0:
            res = bench(n, fixed)
            per_count[str(n)] = {"gpu_count": n, "fit_status": "fit" if res.return_code == 0 else "benchmark_failed",
                                 "reason": "fixed_batch", "selected_batch_size": fixed, "selected_peak_memory_mb": None,
                                 "selected_case_id": None, "selected_log_path": None, "selected_profile_path": None,
                                 "tuning_trials": [], "benchmark_result": asdict(res)}
            if res.return_code == 0 and not args.dry_run:
                points.append(scaling_row(n, fixed, None, res))
            continue

        first, prediction = predict_initial_batch_size(
            args, gpu_count=n, previous_selected_batch_size=prev_batch, previous_gpu_count=prev_count,
            selected_trials_by_gpu_count=selected, trial_history_by_gpu_count=history)

        def probe(batch: int, n=n) -> TuningTrial:
            case = make_case(args, stage=3, batch_size=batch, bandwidth_gbps=0.0,
                             steps=int(args.tuning_memory_warmup_steps) + 1, metrics_warmup_steps=0,
                             bandwidth_mode="none", nproc_per_node=n,
                             extra_args=memory_probe_extra_args(bench_extra, args.tuning_memory_warmup_steps))
            res = harness._run_case(case, run_dir / "tuning", args.skip_existing, args.dry_run, launch, next(counter))
            return trial_from_result(res, fit_mode=args.fit_mode, memory_metric=args.memory_metric,
                                     memory_budget_mb=None)

        print(f"[stage3-scaling] tuning gpu_count={n} initial_batch_size={first} "
              f"predictor={prediction.get('kind', 'unknown')}", flush=True)
        record = {"gpu_count": n, "tuning_strategy": str(args.tuning_strategy), "initial_batch_size": int(first),
                  "tuning_prediction": prediction}
        try:
            best, trials = search_max_batch_size(int(args.min_batch_size), int(args.max_batch_size),
                                                 int(args.batch_size_multiple), float(args.growth_factor),
                                                 int(first), probe)
        except RuntimeError as exc:
            record.update(fit_status="no_fit", reason=str(exc), selected_batch_size=None, benchmark_result=None,
                          tuning_trials=[])
            per_count[str(n)] = record
            print(f"[stage3-scaling] gpu_count={n} no fit: {exc}", flush=True)
            continue
        prev_batch, prev_count = int(best.batch_size), n
        selected[n] = best
        history[n] = list(trials)
        record.update(fit_status="fit", reason=str(best.reason), selected_batch_size=int(best.batch_size),
                      selected_peak_memory_mb=best.peak_memory_mb, selected_case_id=best.case_id,
                      selected_log_path=best.log_path, selected_profile_path=best.profile_path,
                      tuning_trials=[asdict(t) for t in trials])
        res = bench(n, int(best.batch_size))
        record["benchmark_result"] = asdict(res)
        per_count[str(n)] = record
        if res.return_code != 0:
            print(f"[stage3-scaling] benchmark failed gpu_count={n} (see {res.log_path})", flush=True)
        elif not args.dry_run:
            points.append(scaling_row(n, int(best.batch_size), best.peak_memory_mb, res))

    add_scaling_efficiency(points)
    summary = harness._build_summary(results, args)
    mode = "fixed_batch" if fixed > 0 else "fit_to_oom"
    summary.update(
        experiment_type="stage3_gpu_scaling", scaling_mode=mode, fixed_batch_size=fixed if fixed > 0 else None,
        tuning_strategy=str(args.tuning_strategy), gpu_counts=counts,
        per_gpu_total_memory_mb=float(per_gpu_total_memory_mb), per_gpu_count=per_count, scaling_points=points,
        num_successful_scaling_points=len(points),
        base_gpu_count=int(points[0]["gpu_count"]) if points else None,
        base_total_tflops_per_s=float(points[0]["mean_tflops_per_s"]) if points else None,
        methodology_note=("Single-node GPU-count sweep of ZeRO stage 3 with one fixed per-GPU microbatch."
                          if mode == "fixed_batch" else
                          "Single-node GPU-count sweep of ZeRO stage 3; each GPU count is tuned to the largest "
                          f"per-GPU microbatch at the OOM boundary ('{args.tuning_strategy}' seeding), then "
                          "benchmarked without bandwidth shaping."),
        figure3_reference_note=("The ZeRO paper's Figure 3 scales a fixed 60B model from 64 to 400 GPUs; this sweep "
                                "applies the same idea to the GPUs of one node."),
    )
    write_json(run_dir / "summary.json", summary)
    print(f"[stage3-scaling] wrote {run_dir / 'summary.json'}", flush=True)
    if not points and not args.dry_run:
        raise RuntimeError("stage3 scaling sweep produced no successful benchmark points")
    return summary


def main(argv: Optional[List[str]] = None) -> None:
    run(parse_args(argv))


if __name__ == "__main__":
    main()
