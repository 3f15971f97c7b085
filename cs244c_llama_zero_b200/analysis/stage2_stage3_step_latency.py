"""Stage 2 vs stage 3 step latency as a function of link bandwidth.

Per stage, step time is modelled as ``t(BW) = a + b / BW``: ``a`` is the unlimited-bandwidth step
time (measured), ``b`` the bytes-over-the-link term, fitted by least squares through the origin on
the finite-bandwidth points (``t - a`` against ``1 / BW``).  Step time comes from each case's
tokens/s and its global tokens per step.  Outputs the fitted coefficients, the latency ratio
stage3 / stage2 and the throughput ratio (which also counts the different per-step token counts of
fit-to-memory runs) at unlimited and at vanishing bandwidth, and an SVG chart.  Same model as the
reference's ``analysis/stage2_stage3_step_latency.py``.

    python -m cs244c_llama_zero_b200.analysis.stage2_stage3_step_latency --stage2-run runA --stage3-run runB
"""

from __future__ import annotations

import argparse
import json
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Tuple

from . import svg


@dataclass
class Point:
    bandwidth_gbps: float
    step_time_s: float
    tokens_per_s: float
    stage: int
    tokens_per_step: int


def load_run_points(run_dir: Path) -> List[Point]:
    summary = json.loads((Path(run_dir) / "summary.json").read_text())
    world = int(summary["args"]["nproc_per_node"])
    out = []
    for r in summary["results"]:
        if int(r.get("return_code", 1)) != 0 or not r.get("mean_tokens_per_s"):
            continue
        cfg = r["config"]
        tps = float(r["mean_tokens_per_s"])
        tokens = int(cfg["batch_size"]) * int(cfg["seq_len"]) * int(cfg["grad_accum_steps"]) * world
        out.append(Point(float(cfg["bandwidth_gbps"]), tokens / tps, tps, int(cfg["stage"]), tokens))
    return out


def load_points(run_dirs: List[str], stage: int) -> List[Point]:
    """Points of ``stage`` from several run dirs; a later run replaces an earlier one at the same bandwidth."""
    by_bw: Dict[float, Point] = {}
    for d in run_dirs:
        for p in load_run_points(Path(d)):
            if p.stage == stage:
                by_bw[p.bandwidth_gbps] = p
    return sorted(by_bw.values(), key=lambda p: (p.bandwidth_gbps <= 0, -p.bandwidth_gbps))


def fit_bandwidth_model(points: List[Point]) -> Tuple[float, float]:
    """(a, b) of t = a + b / BW; needs exactly one unlimited point and at least one finite one."""
    unlimited = [p for p in points if p.bandwidth_gbps <= 0]
    finite = [p for p in points if p.bandwidth_gbps > 0]
    if len(unlimited) != 1:
        raise ValueError("expected exactly one unlimited-bandwidth point")
    if not finite:
        raise ValueError("expected at least one finite-bandwidth point")
    a = unlimited[0].step_time_s
    xs = [1.0 / p.bandwidth_gbps for p in finite]
    ys = [p.step_time_s - a for p in finite]
    sxx = sum(x * x for x in xs)
    if sxx <= 0:
        raise ValueError("degenerate finite-bandwidth points")
    return a, sum(x * y for x, y in zip(xs, ys)) / sxx


def ratios(a2: float, b2: float, a3: float, b3: float, token_ratio: float) -> Dict[str, float]:
    return {"latency_ratio_unlimited": a3 / a2, "latency_ratio_low_bw": b3 / b2,
            "throughput_ratio_unlimited": token_ratio * a2 / a3, "throughput_ratio_low_bw": token_ratio * b2 / b3}


def analyse(stage2_runs: List[str], stage3_runs: List[str]) -> Dict[str, object]:
    p2, p3 = load_points(stage2_runs, 2), load_points(stage3_runs, 3)
    if not p2 or not p3:
        raise RuntimeError("missing successful points")
    a2, b2 = fit_bandwidth_model(p2)
    a3, b3 = fit_bandwidth_model(p3)
    token_ratio = p3[0].tokens_per_step / p2[0].tokens_per_step
    return {"stage2": {"a_s": a2, "b_s_gbps": b2, "points": [p.__dict__ for p in p2]},
            "stage3": {"a_s": a3, "b_s_gbps": b3, "points": [p.__dict__ for p in p3]},
            "token_ratio_stage3_over_stage2": token_ratio, **ratios(a2, b2, a3, b3, token_ratio)}


def plot(result: Dict[str, object], output: Path) -> Path:
    bws = sorted({p["bandwidth_gbps"] for s in ("stage2", "stage3") for p in result[s]["points"]
                  if p["bandwidth_gbps"] > 0})
    lo, hi = min(bws), max(bws)
    grid = [lo * (hi / lo) ** (k / 40) for k in range(41)] if hi > lo else [lo]
    series = {}
    for s in ("stage2", "stage3"):
        a, b = result[s]["a_s"], result[s]["b_s_gbps"]
        series[f"{s} fit"] = [(x, a + b / x) for x in grid]
        series[f"{s} observed"] = [(p["bandwidth_gbps"], p["step_time_s"]) for p in result[s]["points"]
                                   if p["bandwidth_gbps"] > 0]
    return svg.line_chart(series, output, title="Stage 2 vs Stage 3 step latency", xlabel="Bandwidth (Gbps, log)",
                          ylabel="Step latency (s)", log_x=True)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Fit and plot stage-2 vs stage-3 step latency over bandwidth")
    p.add_argument("--stage2-run", action="append", required=True)
    p.add_argument("--stage3-run", action="append", required=True)
    p.add_argument("--output", default="analysis/figures/stage2_stage3_step_latency.svg")
    a = p.parse_args(argv)
    result = analyse(a.stage2_run, a.stage3_run)
    out = plot(result, Path(a.output))
    print(json.dumps({k: v for k, v in result.items() if not isinstance(v, dict)}, indent=2))
    print(f"[step-latency] wrote {out}")


if __name__ == "__main__":
    main()
