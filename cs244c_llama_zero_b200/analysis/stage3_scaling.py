"""Figure-3-style outputs of a stage-3 GPU-count sweep: a scaling chart and a markdown report.

Reads ``summary.json`` of ``experiments.run_stage3_scaling_sweep``, re-bases the perfect-linear
projection on a chosen GPU count (default: the smallest multi-GPU point), and reports total and
per-GPU TFLOP/s, speedup, efficiency and any super-linear gain (ZeRO-3 frees memory as the GPU count
grows, so the per-GPU micro-batch - and with it per-GPU efficiency - can grow).  Record keys follow
the reference's ``analysis/stage3_scaling.py``.

    python -m cs244c_llama_zero_b200.analysis.stage3_scaling --run-dir experiments/results/<name> \
        --figure-output scaling.svg --report-output scaling.md
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Dict, List, Optional

from . import svg

_FLOAT_KEYS = ("selected_peak_memory_mb", "mean_tokens_per_s", "perfect_linear_tflops_per_s", "speedup_vs_base",
               "scaling_efficiency_vs_base", "superlinear_gain_vs_perfect_linear", "peak_cuda_max_allocated_mb")


def load_summary(run_dir: Path) -> Dict[str, object]:
    path = Path(run_dir) / "summary.json"
    if not path.exists():
        raise FileNotFoundError(f"missing summary.json under {run_dir}")
    data = json.loads(path.read_text())
    if not isinstance(data, dict):
        raise ValueError(f"summary.json under {run_dir} must contain a JSON object")
    return data


def _opt(v, cast):
    return None if v is None else cast(v)


def scaling_points(summary: Dict[str, object]) -> List[Dict[str, object]]:
    """Typed, GPU-count-sorted points that have TFLOP/s; ``peak_memory_mb`` prefers the tuned peak."""
    raw = summary.get("scaling_points", [])
    if not isinstance(raw, list):
        raise ValueError("summary scaling_points must be a list")
    out = []
    for r in raw:
        if not isinstance(r, dict) or r.get("mean_tflops_per_s") is None or r.get("per_gpu_tflops_per_s") is None:
            continue
        p = {"gpu_count": int(r["gpu_count"]),
             "selected_batch_size": _opt(r.get("selected_batch_size"), int),
             "global_tokens_per_step": _opt(r.get("global_tokens_per_step"), int),
             "mean_tflops_per_s": float(r["mean_tflops_per_s"]),
             "per_gpu_tflops_per_s": float(r["per_gpu_tflops_per_s"])}
        p.update({k: _opt(r.get(k), float) for k in _FLOAT_KEYS})
        peak = r.get("selected_peak_memory_mb")
        peak = r.get("peak_cuda_max_allocated_mb") if peak is None else peak
        p["peak_memory_mb"] = _opt(peak, float)
        out.append(p)
    if not out:
        raise RuntimeError("no successful scaling points were found in summary.json")
    return sorted(out, key=lambda p: p["gpu_count"])


def choose_baseline_gpu_count(points: List[Dict[str, object]], requested: int) -> int:
    counts = {int(p["gpu_count"]) for p in points}
    if requested > 0:
        if requested not in counts:
            raise ValueError(f"requested baseline GPU count {requested} is not present in the scaling points")
        return requested
    multi = sorted(c for c in counts if c > 1)
    return multi[0] if multi else min(counts)


def annotate_points(points: List[Dict[str, object]], baseline: int) -> List[Dict[str, object]]:
    """Points at or above ``baseline`` GPUs with speedup/efficiency against it."""
    by = {int(p["gpu_count"]): dict(p) for p in points}
    if baseline not in by:
        raise ValueError(f"baseline GPU count {baseline} is not present in the scaling points")
    t0 = float(by[baseline]["mean_tflops_per_s"])
    out = []
    for n in sorted(c for c in by if c >= baseline):
        p = by[n]
        ideal = n / baseline
        p["perfect_linear_tflops_per_s"] = t0 * ideal
        p["speedup_vs_base"] = float(p["mean_tflops_per_s"]) / t0
        p["scaling_efficiency_vs_base"] = p["speedup_vs_base"] / ideal
        p["superlinear_gain_vs_perfect_linear"] = float(p["mean_tflops_per_s"]) / (t0 * ideal) if t0 > 0 else None
        out.append(p)
    return out


def plot_figure(points: List[Dict[str, object]], output: Path, baseline: int) -> Path:
    """Total TFLOP/s (observed vs perfect linear) over the GPU counts; per-GPU TFLOP/s as a second chart."""
    observed = [(float(p["gpu_count"]), float(p["mean_tflops_per_s"])) for p in points]
    linear = [(float(p["gpu_count"]), float(p["perfect_linear_tflops_per_s"] or p["mean_tflops_per_s"]))
              for p in points]
    labels = {float(p["gpu_count"]): str(p["gpu_count"]) for p in points}
    out = svg.line_chart({"Observed Performance (TFLOPs)": observed, "Perfect Linear Scalability (TFLOPs)": linear},
                         output, title=f"ZeRO Scaling (baseline {baseline} GPU)", xlabel="Number of GPUs",
                         ylabel="Total Performance (TFLOPs)", log_x=True, x_tick_labels=labels)
    svg.bar_chart([str(p["gpu_count"]) for p in points],
                  {"Performance/GPU (TFLOPs)": [float(p["per_gpu_tflops_per_s"]) for p in points]},
                  out.with_name(out.stem + "_per_gpu.svg"), title="Per-GPU Performance", xlabel="Number of GPUs",
                  ylabel="Performance/GPU (TFLOPs)", annotate=True)
    return out


def _f(v: Optional[float], digits: int = 2) -> str:
    return "NA" if v is None else f"{v:.{digits}f}"


def render_report(summary: Dict[str, object], points: List[Dict[str, object]], baseline_gpu_count: int) -> str:
    args = summary.get("args", {}) or {}
    fixed = str(summary.get("scaling_mode", "fit_to_oom")) == "fixed_batch"
    lines = ["# Stage 3 GPU Scaling", "", "Methodology:",
             "- Adapted from Figure 3 of the ZeRO paper: fixed model, sweep GPU count, and measure total TFLOPs plus "
             "TFLOPs/GPU.",
             (f"- This run uses one fixed per-GPU microbatch across all GPU counts: "
              f"`{summary.get('fixed_batch_size', 'unknown')}`.") if fixed else
             "- For each GPU count, this run tunes the largest ZeRO Stage 3 microbatch that fits, then benchmarks that "
             "tuned workload.",
             "- This differs from the original paper in scale: the paper reports a 60B model from 64 to 400 GPUs, while "
             "this run sweeps the GPUs of one node with this repository's preset model sizes.", "",
             "Configuration:"]
    for key in ("model_size", "seq_len", "dtype", "tflops_mode", "steps"):
        lines.append(f"- {key}: `{args.get(key, 'unknown')}`")
    lines += [f"- baseline_gpu_count_for_linear_reference: `{baseline_gpu_count}`", "",
              "| GPUs | batch/GPU | global tokens/step | total TFLOPs | TFLOPs/GPU | perfect linear TFLOPs | speedup vs "
              "base | efficiency | peak alloc MB |",
              "| --- | --- | --- | --- | --- | --- | --- | --- | --- |"]
    for p in points:
        lines.append("| " + " | ".join([
            str(p["gpu_count"]), str(p["selected_batch_size"]), str(p["global_tokens_per_step"]),
            _f(p["mean_tflops_per_s"]), _f(p["per_gpu_tflops_per_s"]), _f(p["perfect_linear_tflops_per_s"]),
            _f(p["speedup_vs_base"]), _f(p["scaling_efficiency_vs_base"], 3), _f(p["peak_memory_mb"])]) + " |")
    base = next(p for p in points if int(p["gpu_count"]) == baseline_gpu_count)
    best = max(points, key=lambda p: float(p["mean_tflops_per_s"]))
    lines += ["", "Observations:",
              f"- Base point: `{base['gpu_count']}` GPU at `{_f(base['mean_tflops_per_s'])}` TFLOPs total and "
              f"`{_f(base['per_gpu_tflops_per_s'])}` TFLOPs/GPU.",
              f"- Best total throughput: `{best['gpu_count']}` GPUs at `{_f(best['mean_tflops_per_s'])}` TFLOPs."]
    superlinear = [p for p in points if (p["superlinear_gain_vs_perfect_linear"] or 0.0) > 1.01]
    if superlinear:
        top = max(superlinear, key=lambda p: float(p["superlinear_gain_vs_perfect_linear"]))
        lines.append(f"- Strongest superlinear gain vs the base-point linear projection: `{top['gpu_count']}` GPUs at "
                     f"`{_f(top['superlinear_gain_vs_perfect_linear'], 3)}x` of perfect-linear.")
    else:
        lines.append("- No superlinear gain above the base-point linear projection was observed in this run.")
    per_count = summary.get("per_gpu_count", {})
    skipped = sorted((str(k) for k, v in (per_count.items() if isinstance(per_count, dict) else [])
                      if isinstance(v, dict) and v.get("fit_status") == "no_fit"), key=int)
    if skipped:
        lines.append(f"- GPU counts skipped for lack of fit at microbatch 1: `{', '.join(skipped)}`.")
    lines += ["", "Reference:",
              "- ZeRO paper, Figure 3: [ZeRO: Memory Optimizations Toward Training Trillion Parameter Models]"
              "(https://arxiv.org/pdf/1910.02054.pdf)"]
    return "\n".join(lines) + "\n"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Render Figure-3-style Stage 3 GPU-scaling outputs")
    p.add_argument("--run-dir", type=str, required=True, help="experiments/results/<name>")
    p.add_argument("--figure-output", type=str, default="", help="Optional output path for the figure (SVG)")
    p.add_argument("--report-output", type=str, default="", help="Optional output path for the markdown report")
    p.add_argument("--baseline-gpu-count", type=int, default=0,
                   help="GPU count of the perfect-linear reference; 0 = smallest point with >1 GPU, else smallest.")
    args = p.parse_args(argv)
    summary = load_summary(Path(args.run_dir))
    raw = scaling_points(summary)
    base = choose_baseline_gpu_count(raw, int(args.baseline_gpu_count))
    points = annotate_points(raw, base)
    if args.figure_output:
        print(f"[stage3-scaling] wrote {plot_figure(points, Path(args.figure_output), base)}")
    if args.report_output:
        out = Path(args.report_output)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(render_report(summary, points, base))
        print(f"[stage3-scaling] wrote {out}")


if __name__ == "__main__":
    main()
