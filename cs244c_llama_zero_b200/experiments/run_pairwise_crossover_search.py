"""Adaptive search for the bandwidth at which two ZeRO stages trade places.

Each stage's micro-batch is tuned to the OOM boundary (or fixed with ``--stage-{a,b}-batch-size``).
Bandwidth is then sampled in log space: the range ends and their geometric midpoint (plus any
``--seed-bandwidth-gbps``), then geometric midpoints of the most promising neighbouring pair -
first an interval where the throughput ratio B/A changes sign (the crossover is inside), else the
interval closest to parity.  It stops at ``--max-pairwise-bandwidth-points``, when the bracketing
interval is within ``--bandwidth-tolerance-ratio``, or when a sample is within
``--near-parity-log-ratio`` of parity.  Writes ``tuning_summary.json``, ``summary.json`` and
``pairwise_report.md``.  Same flags, selection rule and outputs as the reference's
``experiments/run_pairwise_crossover_search.py``.
"""

from __future__ import annotations

import argparse
import itertools
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Dict, List, Optional, Tuple

from . import harness
from .common import (add_bandwidth_args, add_launch_args, add_run_args, add_training_args, add_tuning_args,
                     make_case, parse_with_config, write_json)
from .tuning import (TuningTrial, detect_gpu_total_memory_mb, memory_probe_extra_args, search_max_batch_size,
                     trial_from_result)


@dataclass(frozen=True)
class PairwisePoint:
    bandwidth_gbps: float
    stage_a_tokens_per_s: float
    stage_b_tokens_per_s: float
    stage_a_comm_ms: float
    stage_b_comm_ms: float
    stage_a_fb_ms: float
    stage_b_fb_ms: float
    ratio_stage_b_over_stage_a: float
    winner_stage: int

    @property
    def log_ratio(self) -> float:
        return math.log(self.ratio_stage_b_over_stage_a)

    def payload(self) -> Dict[str, object]:
        return {k: (int(v) if k == "winner_stage" else float(v)) for k, v in asdict(self).items()}


def _build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Tune two ZeRO stages to the OOM boundary, then search bandwidth for a "
                                            "throughput crossover")
    add_run_args(p, "pairwise_crossover_search")
    p.add_argument("--stage-a", type=int, default=2)
    p.add_argument("--stage-b", type=int, default=3)
    p.add_argument("--stage-a-batch-size", type=int, default=0, help="If >0, fixed stage-a microbatch (no tuning).")
    p.add_argument("--stage-b-batch-size", type=int, default=0, help="If >0, fixed stage-b microbatch (no tuning).")
    add_launch_args(p, nproc=4, timeout_s=1800.0)
    add_training_args(p, model_size="small", steps=6, seq_len=256)
    add_bandwidth_args(p)
    add_tuning_args(p, max_batch=1024, multiple=4, fit_modes=["oom_boundary"])
    p.add_argument("--include-unlimited", action="store_true")
    p.add_argument("--bandwidth-min-gbps", type=float, default=0.01)
    p.add_argument("--bandwidth-max-gbps", type=float, default=0.5)
    p.add_argument("--seed-bandwidth-gbps", nargs="*", type=float, default=[],
                   help="Extra finite seed points; the range ends and their geometric midpoint are always sampled.")
    p.add_argument("--max-pairwise-bandwidth-points", type=int, default=6)
    p.add_argument("--bandwidth-tolerance-ratio", type=float, default=1.25,
                   help="Stop refining a bracketing interval once high/low bandwidth is within this ratio.")
    p.add_argument("--near-parity-log-ratio", type=float, default=0.05,
                   help="Treat a sample with |log(B/A throughput)| below this as parity.")
    return p


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    return parse_with_config(_build_parser(), argv)


# ------------------------------------------------------------------------------ search rule
def _sign(x: float) -> int:
    return (x > 0) - (x < 0)


def _neighbours(sampled: Dict[float, PairwisePoint]) -> List[Tuple[PairwisePoint, PairwisePoint]]:
    pts = sorted(sampled.values(), key=lambda p: p.bandwidth_gbps)
    return list(zip(pts, pts[1:]))


def choose_next_finite_bandwidth(sampled: Dict[float, PairwisePoint], *, tolerance_ratio: float) -> Optional[float]:
    """Geometric midpoint of the best unresolved neighbouring pair, or None.

    Pairs already within ``tolerance_ratio`` (or whose midpoint was sampled) are resolved.  Ranking:
    a sign flip of log(B/A) first, the narrowest (log-span) flip winning; otherwise the pair whose
    worse endpoint is closest to parity, wider pairs first on ties.
    """
    best: Optional[Tuple[Tuple[int, float, float], float]] = None
    for lo, hi in _neighbours(sampled):
        if hi.bandwidth_gbps / lo.bandwidth_gbps <= tolerance_ratio:
            continue
        mid = math.sqrt(lo.bandwidth_gbps * hi.bandwidth_gbps)
        if any(math.isclose(mid, bw, rel_tol=1e-9, abs_tol=1e-12) for bw in sampled):
            continue
        span = math.log(hi.bandwidth_gbps / lo.bandwidth_gbps)
        if _sign(lo.log_ratio) != _sign(hi.log_ratio):
            key = (0, span, 0.0)
        else:
            key = (1, max(abs(lo.log_ratio), abs(hi.log_ratio)), -span)
        if best is None or key < best[0]:
            best = (key, mid)
    return None if best is None else best[1]


def best_flip_bracket(sampled: Dict[float, PairwisePoint]) -> Optional[Tuple[PairwisePoint, PairwisePoint]]:
    """The narrowest neighbouring pair whose throughput ratio changes sign."""
    flips = [(hi.bandwidth_gbps / lo.bandwidth_gbps, lo, hi) for lo, hi in _neighbours(sampled)
             if _sign(lo.log_ratio) != _sign(hi.log_ratio)]
    if not flips:
        return None
    _, lo, hi = min(flips, key=lambda f: f[0])
    return lo, hi


def nearest_parity_point(sampled: Dict[float, PairwisePoint]) -> Optional[PairwisePoint]:
    return min(sampled.values(), key=lambda p: abs(p.log_ratio)) if sampled else None


def seed_bandwidths(lo: float, hi: float, extras: List[float]) -> List[float]:
    """Initial finite samples, highest bandwidth first."""
    seeds = {float(lo), float(hi), math.sqrt(lo * hi)} | {float(x) for x in extras if x > 0}
    return sorted(seeds, reverse=True)


def make_point(bw: float, stage_a: int, stage_b: int, a: harness.CaseResult, b: harness.CaseResult) -> PairwisePoint:
    ta, tb = float(a.mean_tokens_per_s), float(b.mean_tokens_per_s)
    return PairwisePoint(bandwidth_gbps=float(bw), stage_a_tokens_per_s=ta, stage_b_tokens_per_s=tb,
                         stage_a_comm_ms=float(a.mean_comm_ms or 0.0), stage_b_comm_ms=float(b.mean_comm_ms or 0.0),
                         stage_a_fb_ms=float(a.mean_fb_ms or 0.0), stage_b_fb_ms=float(b.mean_fb_ms or 0.0),
                         ratio_stage_b_over_stage_a=tb / ta, winner_stage=stage_b if tb >= ta else stage_a)


# ------------------------------------------------------------------------------ report
def render_report(args: argparse.Namespace, selected: Dict[int, TuningTrial], unlimited: Optional[PairwisePoint],
                  finite: Dict[float, PairwisePoint],
                  bracket: Optional[Tuple[PairwisePoint, PairwisePoint]]) -> str:
    a, b = int(args.stage_a), int(args.stage_b)
    out = ["# Pairwise Crossover Search", "", "## Setup", "",
           f"- stage A: `{a}`", f"- stage B: `{b}`", f"- model: `{args.model_size}`",
           f"- seq len: `{int(args.seq_len)}`", f"- steps: `{int(args.steps)}`",
           f"- bandwidth range searched: `{float(args.bandwidth_min_gbps):g}` to `{float(args.bandwidth_max_gbps):g} Gbps`",
           f"- max finite bandwidth points: `{int(args.max_pairwise_bandwidth_points)}`", "",
           "## Tuned Microbatches", "",
           "| stage | selected microbatch / GPU | peak allocated MB | tuned unlimited tokens/s |",
           "| --- | --- | --- | --- |"]
    for s in (a, b):
        t = selected[s]
        peak = "NA" if t.peak_memory_mb is None else f"{t.peak_memory_mb:.1f}"
        tps = "NA" if t.mean_tokens_per_s is None else f"{t.mean_tokens_per_s:.1f}"
        out.append(f"| {s} | {t.batch_size} | {peak} | {tps} |")
    if unlimited is not None:
        out += ["", "## Unlimited Context", "",
                f"- stage {b} / stage {a} throughput ratio at unlimited bandwidth: "
                f"`{unlimited.ratio_stage_b_over_stage_a:.3f}x`"]
    out += ["", "## Finite Bandwidth Samples", "", "| bandwidth (Gbps) | stage A tok/s | stage B tok/s | B / A | winner |",
            "| --- | --- | --- | --- | --- |"]
    for bw in sorted(finite, reverse=True):
        p = finite[bw]
        out.append(f"| {bw:g} | {p.stage_a_tokens_per_s:.1f} | {p.stage_b_tokens_per_s:.1f} | "
                   f"{p.ratio_stage_b_over_stage_a:.3f}x | stage {p.winner_stage} |")
    out += ["", "## Conclusion", ""]
    near = nearest_parity_point(finite)
    if bracket is not None:
        out.append(f"- sampled points bracket a crossover between `{bracket[0].bandwidth_gbps:g}` and "
                   f"`{bracket[1].bandwidth_gbps:g} Gbps`")
    elif near is not None:
        out.append(f"- no sampled crossover was found in the searched bandwidth range; the closest sampled point to "
                   f"parity was `{near.bandwidth_gbps:g} Gbps`, where stage {near.winner_stage} still led by "
                   f"`{abs(near.log_ratio):.3f}` log-ratio (`{near.ratio_stage_b_over_stage_a:.3f}x` B/A)")
    else:
        out.append("- no finite bandwidth samples were completed")
    out += ["", "Method note:", "- this is an adaptive pairwise search, not an exhaustive grid",
            "- if no bracketing sign change appears, the result is 'no crossover found in the searched range', "
            "not a proof of impossibility"]
    return "\n".join(out) + "\n"


# ------------------------------------------------------------------------------ driver
def run(args: argparse.Namespace, gpu_total_memory_mb: Optional[float] = None) -> Dict[str, object]:
    a, b = int(args.stage_a), int(args.stage_b)
    if a == b:
        raise ValueError("stage-a and stage-b must be different")
    lo_bw, hi_bw = float(args.bandwidth_min_gbps), float(args.bandwidth_max_gbps)
    if lo_bw <= 0 or hi_bw <= 0:
        raise ValueError("bandwidth-min-gbps and bandwidth-max-gbps must be > 0")
    if lo_bw >= hi_bw:
        raise ValueError("bandwidth-min-gbps must be smaller than bandwidth-max-gbps")
    launch = harness._launch_config_from_args(args)
    run_dir = Path(args.results_dir) / args.name
    run_dir.mkdir(parents=True, exist_ok=True)
    if gpu_total_memory_mb is None:
        gpu_total_memory_mb = detect_gpu_total_memory_mb(args.nproc_per_node)
    counter = itertools.count()
    fixed = {a: int(args.stage_a_batch_size), b: int(args.stage_b_batch_size)}
    selected: Dict[int, TuningTrial] = {}
    tuning: Dict[str, object] = {
        "experiment_type": "pairwise_crossover_search", "name": args.name, "model_size": args.model_size,
        "seq_len": int(args.seq_len), "grad_accum_steps": int(args.grad_accum_steps),
        "nproc_per_node": int(args.nproc_per_node), "gpu_total_memory_mb": float(gpu_total_memory_mb),
        "memory_metric": str(args.memory_metric), "stages": [a, b], "per_stage": {}}
    for stage in (a, b):
        if fixed[stage] > 0:
            selected[stage] = TuningTrial(fixed[stage], True, None, 0, "fixed_batch_size", "", "", "", None)
            tuning["per_stage"][str(stage)] = {"selected_batch_size": fixed[stage], "selected_peak_memory_mb": None,
                                               "selected_case_id": "", "selected_mean_tokens_per_s": None,
                                               "trials": [], "selection_mode": "fixed_batch_size"}
            print(f"[pairwise] stage {stage}: using fixed microbatch {fixed[stage]}", flush=True)
            continue

        def probe(batch: int, stage=stage) -> TuningTrial:
            case = make_case(args, stage=stage, batch_size=batch, bandwidth_gbps=0.0,
                             steps=int(args.tuning_memory_warmup_steps) + 1, metrics_warmup_steps=0,
                             bandwidth_mode="none",
                             extra_args=memory_probe_extra_args(args.extra_args, args.tuning_memory_warmup_steps))
            res = harness._run_case(case, run_dir / "tuning", args.skip_existing, args.dry_run, launch, next(counter))
            return trial_from_result(res, fit_mode="oom_boundary", memory_metric=args.memory_metric,
                                     memory_budget_mb=None)

        best, trials = search_max_batch_size(int(args.min_batch_size), int(args.max_batch_size),
                                             max(1, int(args.batch_size_multiple)), max(1.1, float(args.growth_factor)),
                                             int(args.initial_batch_size), probe)
        selected[stage] = best
        tuning["per_stage"][str(stage)] = {
            "selected_batch_size": int(best.batch_size), "selected_peak_memory_mb": best.peak_memory_mb,
            "selected_case_id": best.case_id, "selected_mean_tokens_per_s": best.mean_tokens_per_s,
            "trials": [asdict(t) for t in trials], "selection_mode": "tuned"}
        print(f"[pairwise] stage {stage}: selected microbatch {best.batch_size} "
              f"peak={best.peak_memory_mb if best.peak_memory_mb is not None else 'NA'} MB", flush=True)
    write_json(run_dir / "tuning_summary.json", tuning)
    print(f"[pairwise] wrote {run_dir / 'tuning_summary.json'}", flush=True)
    if args.dry_run:
        print("[pairwise] dry run complete; skipping pairwise search", flush=True)
        return tuning

    history: List[Dict[str, object]] = []

    def measure(bw: float) -> PairwisePoint:
        res = {}
        for stage in (a, b):
            case = make_case(args, stage=stage, batch_size=selected[stage].batch_size, bandwidth_gbps=bw,
                             steps=int(args.steps), metrics_warmup_steps=int(args.metrics_warmup_steps),
                             bandwidth_mode=str(args.bandwidth_mode), extra_args=str(args.extra_args))
            r = harness._run_case(case, run_dir, args.skip_existing, False, launch, next(counter))
            if r.return_code != 0 or r.mean_tokens_per_s is None:
                raise RuntimeError(f"pairwise case failed: {r.case_id} (see {r.log_path})")
            res[stage] = r
        point = make_point(bw, a, b, res[a], res[b])
        history.append({**point.payload(), "stage_a": a, "stage_b": b})
        print(f"[pairwise] bw={bw:g} Gbps: stage {a}={point.stage_a_tokens_per_s:.1f} tok/s, "
              f"stage {b}={point.stage_b_tokens_per_s:.1f} tok/s, ratio={point.ratio_stage_b_over_stage_a:.3f}x",
              flush=True)
        return point

    unlimited = measure(0.0) if args.include_unlimited else None
    budget = int(args.max_pairwise_bandwidth_points)
    finite: Dict[float, PairwisePoint] = {}
    for bw in seed_bandwidths(lo_bw, hi_bw, [float(x) for x in args.seed_bandwidth_gbps]):
        if len(finite) >= budget:
            break
        finite[bw] = measure(bw)
    while len(finite) < budget:
        bracket = best_flip_bracket(finite)
        if bracket is not None and bracket[1].bandwidth_gbps / bracket[0].bandwidth_gbps <= args.bandwidth_tolerance_ratio:
            break
        near = nearest_parity_point(finite)
        if near is not None and abs(near.log_ratio) <= float(args.near_parity_log_ratio):
            break
        nxt = choose_next_finite_bandwidth(finite, tolerance_ratio=float(args.bandwidth_tolerance_ratio))
        if nxt is None:
            break
        finite[nxt] = measure(nxt)

    bracket = best_flip_bracket(finite)
    near = nearest_parity_point(finite)
    summary = {
        "experiment_type": "pairwise_crossover_search", "name": args.name, "stage_a": a, "stage_b": b,
        "model_size": str(args.model_size), "seq_len": int(args.seq_len), "steps": int(args.steps),
        "nproc_per_node": int(args.nproc_per_node),
        "tuning": {str(s): {"selected_batch_size": int(t.batch_size), "selected_peak_memory_mb": t.peak_memory_mb,
                            "selected_mean_tokens_per_s": t.mean_tokens_per_s} for s, t in selected.items()},
        "include_unlimited": bool(args.include_unlimited),
        "unlimited_point": None if unlimited is None else unlimited.payload(),
        "finite_points": [finite[bw].payload() for bw in sorted(finite)],
        "nearest_parity_point": None if near is None else near.payload(),
        "crossover_bracket": None if bracket is None else {
            "low_bandwidth_gbps": bracket[0].bandwidth_gbps, "high_bandwidth_gbps": bracket[1].bandwidth_gbps,
            "low_ratio_stage_b_over_stage_a": bracket[0].ratio_stage_b_over_stage_a,
            "high_ratio_stage_b_over_stage_a": bracket[1].ratio_stage_b_over_stage_a},
        "search_history": history,
    }
    write_json(run_dir / "summary.json", summary)
    (run_dir / "pairwise_report.md").write_text(render_report(args, selected, unlimited, finite, bracket))
    print(f"[pairwise] wrote {run_dir / 'summary.json'}", flush=True)
    print(f"[pairwise] wrote {run_dir / 'pairwise_report.md'}", flush=True)
    return summary


def main(argv: Optional[List[str]] = None) -> None:
    run(parse_args(argv))


if __name__ == "__main__":
    main()
