"""Fit-to-memory bandwidth sweep: tune each ZeRO stage's micro-batch to a memory limit, then sweep bandwidth.

Phase 1 runs short tuning launches (``--measure-memory-step``) per stage and picks the largest
micro-batch that fits (``oom_boundary``: the launch exits cleanly; ``memory_budget``: its peak stays
within ``--memory-budget-mb`` or ``--memory-budget-fraction`` of the smallest GPU).  Phase 2 runs every
(stage, bandwidth) pair at that stage's micro-batch, so each stage converts the memory ZeRO saves
into batch.  Outputs ``tuning_summary.json`` and ``summary.json`` (harness record format).
Same flags and outputs as the reference's ``experiments/run_fit_memory_bandwidth.py``.

    python -m cs244c_llama_zero_b200.experiments.run_fit_memory_bandwidth --nproc-per-node 8 \
        --model-size baseline-1.3b --seq-len 1024 --bandwidth-mode none --bandwidth-gbps 0
"""

from __future__ import annotations

import argparse
import itertools
from dataclasses import asdict
from pathlib import Path
from typing import Dict, List, Optional, Tuple

from . import harness
from .common import (add_bandwidth_args, add_launch_args, add_run_args, add_training_args, add_tuning_args,
                     make_case, parse_with_config, write_json)
from .tuning import (TuningTrial, detect_gpu_total_memory_mb, memory_probe_extra_args, search_max_batch_size,
                     trial_from_result)

_select_max_batch_size = search_max_batch_size  # name used by the reference's tests and sibling runners


def _build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Tune per-stage microbatch to a fixed memory budget, then sweep bandwidth")
    add_run_args(p, "fit_memory_bandwidth")
    p.add_argument("--stages", nargs="+", type=int, default=[0, 1, 2, 3])
    p.add_argument("--bandwidth-gbps", nargs="+", type=float, default=[0.0, 1.0, 2.0, 5.0, 10.0])
    add_launch_args(p, nproc=4, timeout_s=1800.0)
    add_training_args(p, model_size="small", steps=10, seq_len=128)
    add_bandwidth_args(p)
    add_tuning_args(p, max_batch=0, multiple=1, fit_modes=["oom_boundary", "memory_budget"])
    p.add_argument("--memory-budget-mb", type=float, default=0.0)
    p.add_argument("--memory-budget-fraction", type=float, default=0.90,
                   help="If --memory-budget-mb is 0, use this fraction of the smallest visible GPU memory.")
    return p


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    return parse_with_config(_build_parser(), argv)


def memory_budget_mb(args: argparse.Namespace) -> Tuple[float, float]:
    """(budget MB, smallest GPU total MB); an explicit budget works without CUDA (then total = budget)."""
    if args.memory_budget_mb > 0:
        try:
            total = detect_gpu_total_memory_mb(args.nproc_per_node)
        except RuntimeError:
            total = float(args.memory_budget_mb)
        return float(args.memory_budget_mb), total
    total = detect_gpu_total_memory_mb(args.nproc_per_node)
    return float(total * args.memory_budget_fraction), total


def stage_tuning_payload(best: TuningTrial, trials: List[TuningTrial], args: argparse.Namespace,
                         nproc: int) -> Dict[str, object]:
    return {
        "selected_batch_size": int(best.batch_size),
        "selected_peak_memory_mb": None if best.peak_memory_mb is None else float(best.peak_memory_mb),
        "selected_case_id": best.case_id,
        "selected_log_path": best.log_path,
        "selected_profile_path": best.profile_path,
        "selected_mean_tokens_per_s": None if best.mean_tokens_per_s is None else float(best.mean_tokens_per_s),
        "selected_global_tokens_per_step": int(best.batch_size * args.grad_accum_steps * args.seq_len * nproc),
        "trials": [asdict(t) for t in trials],
    }


def run(args: argparse.Namespace, gpu_total_memory_mb: Optional[float] = None) -> Dict[str, object]:
    launch = harness._launch_config_from_args(args)
    run_dir = Path(args.results_dir) / args.name
    run_dir.mkdir(parents=True, exist_ok=True)
    if args.fit_mode == "memory_budget":
        budget, total = memory_budget_mb(args)
    else:
        budget, total = None, gpu_total_memory_mb
        if total is None:
            total = detect_gpu_total_memory_mb(args.nproc_per_node)
    max_batch = int(args.max_batch_size) if int(args.max_batch_size) > 0 else 1024
    counter = itertools.count()
    tuning: Dict[str, object] = {
        "experiment_type": "fit_to_memory_bandwidth", "name": args.name, "model_size": args.model_size,
        "seq_len": int(args.seq_len), "grad_accum_steps": int(args.grad_accum_steps),
        "nproc_per_node": int(args.nproc_per_node), "gpu_total_memory_mb": float(total),
        "fit_mode": str(args.fit_mode), "memory_budget_mb": budget,
        "memory_budget_fraction": float(args.memory_budget_fraction) if args.fit_mode == "memory_budget" else None,
        "memory_metric": str(args.memory_metric), "tuning_memory_warmup_steps": int(args.tuning_memory_warmup_steps),
        "stages": [int(s) for s in args.stages], "per_stage": {},
    }
    chosen: Dict[int, int] = {}
    for stage in (int(s) for s in args.stages):
        def probe(batch: int, stage=stage) -> TuningTrial:
            case = make_case(args, stage=stage, batch_size=batch, bandwidth_gbps=0.0,
                             steps=int(args.tuning_memory_warmup_steps) + 1, metrics_warmup_steps=0,
                             bandwidth_mode="none",
                             extra_args=memory_probe_extra_args(args.extra_args, args.tuning_memory_warmup_steps))
            result = harness._run_case(case, run_dir / "tuning", args.skip_existing, args.dry_run, launch,
                                       next(counter))
            return trial_from_result(result, fit_mode=args.fit_mode, memory_metric=args.memory_metric,
                                     memory_budget_mb=budget)

        best, trials = search_max_batch_size(int(args.min_batch_size), max_batch, max(1, int(args.batch_size_multiple)),
                                             max(1.1, float(args.growth_factor)), int(args.initial_batch_size), probe)
        chosen[stage] = best.batch_size
        tuning["per_stage"][str(stage)] = stage_tuning_payload(best, trials, args, int(args.nproc_per_node))
        print(f"[fit-memory] stage {stage}: selected microbatch {best.batch_size} "
              f"peak={best.peak_memory_mb if best.peak_memory_mb is not None else 'NA'} MB", flush=True)
    write_json(run_dir / "tuning_summary.json", tuning)
    print(f"[fit-memory] wrote {run_dir / 'tuning_summary.json'}", flush=True)
    if args.dry_run:
        print("[fit-memory] dry run complete; skipping final bandwidth sweep", flush=True)
        return tuning

    cases = [make_case(args, stage=s, batch_size=chosen[s], bandwidth_gbps=float(bw), steps=int(args.steps),
                       metrics_warmup_steps=int(args.metrics_warmup_steps), bandwidth_mode=str(args.bandwidth_mode),
                       extra_args=str(args.extra_args))
             for s in (int(x) for x in args.stages) for bw in args.bandwidth_gbps]
    print(f"[fit-memory] prepared {len(cases)} final sweep case(s)", flush=True)
    results = []
    for i, case in enumerate(cases, start=1):
        print(f"[fit-memory] ({i}/{len(cases)}) {harness._case_id(case)}", flush=True)
        res = harness._run_case(case, run_dir, args.skip_existing, False, launch, next(counter))
        results.append(res)
        if res.return_code != 0:
            print(f"[fit-memory] case failed: {res.case_id} (see {res.log_path})", flush=True)
    summary = harness._build_summary(results, args)
    summary.update(experiment_type="fit_to_memory_bandwidth", fit_mode=str(args.fit_mode), memory_budget_mb=budget,
                   gpu_total_memory_mb=float(total), memory_metric=str(args.memory_metric))
    summary["fit_memory_tuning"] = {
        stage: {k: payload[k] for k in ("selected_batch_size", "selected_peak_memory_mb",
                                        "selected_global_tokens_per_step")}
        for stage, payload in tuning["per_stage"].items()}
    write_json(run_dir / "summary.json", summary)
    print(f"[fit-memory] wrote {run_dir / 'summary.json'}", flush=True)
    return summary


def main(argv: Optional[List[str]] = None) -> None:
    run(parse_args(argv))


if __name__ == "__main__":
    main()
