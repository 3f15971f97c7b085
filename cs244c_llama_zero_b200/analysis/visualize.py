"""Read harness run directories and plot them (SVG).

``parse_summary`` turns ``summary.json`` into ``CaseView`` rows (also accepting the older flat
``{"stage": ...}`` result schema and rebasing repo-relative log/profile paths into the run directory).
The memory helpers split a case's GPU memory into logical ZeRO model state (params, grads, optimizer
state, from the profile's ``measured_step_state_timeline`` or ``measured_state_memory_mb``) and the rest
(activations, buffers, allocator slack), at the peak or averaged over the sampled snapshots (time
weighted when snapshots carry ``timestamp_s``).  Field names, plot kinds and split rules follow the
reference's ``analysis/visualize.py`` so its result directories read the same here.

    python -m cs244c_llama_zero_b200.analysis.visualize --run-dir experiments/results/<name> --plot peak-memory
"""

from __future__ import annotations

import argparse
import json
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Tuple

from . import svg

STEP_RE = re.compile(r"\[step\s+(\d+)\]\s+loss=([0-9.]+)")
PLOTS = ["loss", "throughput", "tflops", "comm", "stage-throughput", "grouped-stage-throughput", "stage-comm",
         "memory", "peak-memory", "avg-memory"]
STATE_KEYS = ("params_mb", "grads_mb", "optimizer_mb", "total_mb")


@dataclass
class CaseView:
    stage: int
    model_size: str
    bandwidth_gbps: float
    batch_size: int
    grad_accum_steps: int
    seq_len: int
    log_path: Path
    profile_path: Optional[Path]
    mean_tokens_per_s: Optional[float]
    mean_tflops_per_s: Optional[float]
    mean_comm_ms: Optional[float]
    mean_fb_ms: Optional[float]
    mean_opt_ms: Optional[float]
    peak_host_rss_mb: Optional[float]
    peak_cuda_allocated_mb: Optional[float]
    peak_cuda_reserved_mb: Optional[float]
    peak_cuda_max_allocated_mb: Optional[float]
    peak_cuda_max_reserved_mb: Optional[float]
    final_loss: Optional[float]
    return_code: int
    measured_state_memory_mb: Optional[Dict[str, float]]
    theoretical_memory_mb: Optional[Dict[str, float]]


# ------------------------------------------------------------------------------ parsing
def _opt_float(v) -> Optional[float]:
    return None if v is None else float(v)


def _opt_mem(v) -> Optional[Dict[str, float]]:
    return {str(k): float(x) for k, x in v.items()} if isinstance(v, dict) else None


def _resolve_run_path(run_dir: Path, raw: Path) -> Path:
    """Absolute or existing paths as-is; else try the part after the run dir's name, then run_dir/raw."""
    if raw.is_absolute() or raw.exists():
        return raw
    if run_dir.name in raw.parts:
        rebased = run_dir.joinpath(*raw.parts[raw.parts.index(run_dir.name) + 1:])
        if rebased.exists():
            return rebased
    direct = run_dir / raw
    return direct if direct.exists() else raw


def parse_summary(summary_path: Path) -> List[CaseView]:
    summary = json.loads(Path(summary_path).read_text())
    run_dir = Path(summary_path).parent
    out = []
    for r in summary.get("results", []):
        cfg = r.get("config", {}) or {}
        stage = int(r["stage"]) if "stage" in r else int(cfg.get("stage", -1))
        log = Path(str(r["log_path"])) if "log_path" in r else Path(f"stage{stage}.log")
        prof_raw = r.get("profile_path")
        prof = None if prof_raw in (None, "") else _resolve_run_path(run_dir, Path(str(prof_raw)))
        out.append(CaseView(
            stage=stage, model_size=str(cfg.get("model_size", "unknown")),
            bandwidth_gbps=float(cfg.get("bandwidth_gbps", 0.0)), batch_size=int(cfg.get("batch_size", 0)),
            grad_accum_steps=int(cfg.get("grad_accum_steps", 1)), seq_len=int(cfg.get("seq_len", 0)),
            log_path=_resolve_run_path(run_dir, log), profile_path=prof,
            **{k: _opt_float(r.get(k)) for k in (
                "mean_tokens_per_s", "mean_tflops_per_s", "mean_comm_ms", "mean_fb_ms", "mean_opt_ms",
                "peak_host_rss_mb", "peak_cuda_allocated_mb", "peak_cuda_reserved_mb", "peak_cuda_max_allocated_mb",
                "peak_cuda_max_reserved_mb", "final_loss")},
            return_code=int(r.get("return_code", 0)),
            measured_state_memory_mb=_opt_mem(r.get("measured_state_memory_mb")),
            theoretical_memory_mb=_opt_mem(r.get("theoretical_memory_mb"))))
    return out


def parse_loss_log(path: Path) -> Tuple[List[int], List[float]]:
    steps, losses = [], []
    if Path(path).exists():
        for line in Path(path).read_text().splitlines():
            m = STEP_RE.search(line)
            if m:
                steps.append(int(m.group(1)))
                losses.append(float(m.group(2)))
    return steps, losses


def _filter_cases(cases: Iterable[CaseView], model_size: str) -> List[CaseView]:
    return [c for c in cases if not model_size or c.model_size == model_size]


def _filter_bandwidth(cases: Iterable[CaseView], bandwidth_gbps: Optional[float]) -> List[CaseView]:
    return [c for c in cases if bandwidth_gbps is None or abs(c.bandwidth_gbps - bandwidth_gbps) < 1e-9]


def _representative_cases_by_stage(cases: Iterable[CaseView]) -> List[CaseView]:
    """One case per stage: the unlimited-bandwidth run if present, else the fastest link."""
    best: Dict[int, CaseView] = {}
    rank = lambda c: (1 if c.bandwidth_gbps > 0 else 0, -c.bandwidth_gbps)  # noqa: E731
    for c in cases:
        if c.stage not in best or rank(c) < rank(best[c.stage]):
            best[c.stage] = c
    return [best[s] for s in sorted(best)]


# ------------------------------------------------------------------------------ memory accounting
def _case_peak_memory_mb(case: CaseView) -> Optional[float]:
    """First positive CUDA peak (max-allocated, max-reserved, allocated, reserved), else host RSS."""
    for v in (case.peak_cuda_max_allocated_mb, case.peak_cuda_max_reserved_mb, case.peak_cuda_allocated_mb,
              case.peak_cuda_reserved_mb):
        if v is not None and v > 0.0:
            return v
    return case.peak_host_rss_mb


def _profile_payload(case: CaseView) -> Optional[Dict[str, object]]:
    if case.profile_path is None or not case.profile_path.exists():
        return None
    payload = json.loads(case.profile_path.read_text())
    return payload if isinstance(payload, dict) else None


def _profile_memory_snapshots(case: CaseView) -> List[Dict[str, object]]:
    raw = (_profile_payload(case) or {}).get("memory", [])
    return [s for s in raw if isinstance(s, dict)] if isinstance(raw, list) else []


def _labelled(snaps: List[Dict[str, object]], prefix: str) -> List[Dict[str, object]]:
    chosen = [s for s in snaps if str(s.get("label", "")).startswith(prefix)]
    return chosen or snaps


def _measured_step_memory_snapshots(case: CaseView) -> List[Dict[str, object]]:
    return _labelled(_profile_memory_snapshots(case), "measured_step_")


def _training_memory_snapshots(case: CaseView) -> List[Dict[str, object]]:
    return _labelled(_profile_memory_snapshots(case), "step_")


def _measured_step_state_timeline(case: CaseView) -> List[Dict[str, object]]:
    raw = (_profile_payload(case) or {}).get("measured_step_state_timeline", [])
    out = []
    for item in raw if isinstance(raw, list) else []:
        if not isinstance(item, dict) or not item.get("label") or item.get("total_mb") is None:
            continue
        out.append({"label": str(item["label"]), **{k: float(item.get(k, 0.0)) for k in STATE_KEYS}})
    return out


def _state(item: Dict[str, object]) -> Dict[str, float]:
    return {k: float(item[k]) for k in STATE_KEYS}


def _measured_step_state_map(case: CaseView) -> Dict[str, float]:
    """label -> logical state MB.  Stage-3 timelines that left out the resident parameter shard get it added."""
    m = {str(i["label"]): float(i["total_mb"]) for i in _measured_step_state_timeline(case)}
    if case.stage == 3 and m and case.measured_state_memory_mb is not None:
        params = float(case.measured_state_memory_mb.get("params_mb", 0.0))
        total = float(case.measured_state_memory_mb.get("total_mb", 0.0))
        if abs((total - min(m.values())) - params) <= max(1.0, params * 0.05):
            m = {k: v + params for k, v in m.items()}
    return m


def _case_peak_state_breakdown(case: CaseView) -> Optional[Dict[str, float]]:
    tl = _measured_step_state_timeline(case)
    return _state(max(tl, key=lambda i: i["total_mb"])) if tl else case.measured_state_memory_mb


def _case_post_backward_state_breakdown(case: CaseView) -> Optional[Dict[str, float]]:
    for item in _measured_step_state_timeline(case):
        if str(item["label"]).endswith("_post_backward"):
            return _state(item)
    return case.measured_state_memory_mb


def _case_logical_state_breakdown(case: CaseView) -> Optional[Dict[str, float]]:
    return case.measured_state_memory_mb if case.measured_state_memory_mb is not None \
        else _case_post_backward_state_breakdown(case)


def _case_state_breakdown_at_peak_total(case: CaseView) -> Optional[Dict[str, float]]:
    """State breakdown at the snapshot whose running CUDA peak is the highest (first such label)."""
    snaps = _measured_step_memory_snapshots(case)
    if snaps:
        top = max(float(s.get("cuda_max_allocated_mb", 0.0)) for s in snaps)
        label = next(str(s.get("label", "")) for s in snaps if abs(float(s.get("cuda_max_allocated_mb", 0.0)) - top) < 1e-6)
        for item in _measured_step_state_timeline(case) if label else []:
            if item["label"] == label:
                return _state(item)
    return _case_peak_state_breakdown(case)


def _case_peak_breakdown_mb(case: CaseView) -> Optional[Tuple[float, float]]:
    """(logical state, everything else) at the measured peak."""
    peak = _case_peak_memory_mb(case)
    if peak is None:
        return None
    logical = _case_logical_state_breakdown(case)
    state = min(max(0.0 if logical is None else float(logical.get("total_mb", 0.0)), 0.0), peak)
    return state, max(peak - state, 0.0)


def _case_average_live_breakdown_mb(case: CaseView) -> Optional[Tuple[float, float]]:
    """(average logical state, average non-state) over the measured step's snapshots.

    With two or more timestamped snapshots each one holds until the next (time weighted); otherwise a
    plain mean.  Without a state timeline, the mean allocated memory over training-step snapshots is
    split against ``measured_state_memory_mb``.
    """
    state_map = _measured_step_state_map(case)
    pairs = []
    for s in _measured_step_memory_snapshots(case):
        label = str(s.get("label", ""))
        if label in state_map and "cuda_allocated_mb" in s:
            alloc = float(s["cuda_allocated_mb"])
            ts = s.get("timestamp_s")
            pairs.append((None if ts is None else float(ts), alloc, min(max(state_map[label], 0.0), alloc)))
    if pairs:
        timed = [p for p in pairs if p[0] is not None]
        if len(timed) >= 2 and timed[-1][0] - timed[0][0] > 0.0:
            span = timed[-1][0] - timed[0][0]
            st = ns = 0.0
            for (t, alloc, state), nxt in zip(timed, timed[1:]):
                dt = max(0.0, nxt[0] - t)
                st += state * dt
                ns += max(alloc - state, 0.0) * dt
            return st / span, ns / span
        return (sum(p[2] for p in pairs) / len(pairs), sum(max(p[1] - p[2], 0.0) for p in pairs) / len(pairs))
    allocs = [float(s["cuda_allocated_mb"]) for s in _training_memory_snapshots(case) if "cuda_allocated_mb" in s]
    if not allocs:
        return None
    avg = sum(allocs) / len(allocs)
    total = float(case.measured_state_memory_mb.get("total_mb", 0.0)) if case.measured_state_memory_mb else 0.0
    state = min(max(total, 0.0), avg)
    return state, max(avg - state, 0.0)


# ------------------------------------------------------------------------------ plots
def _bw_label(bw: float) -> str:
    return "unlimited" if bw <= 0 else f"{bw:g}Gbps"


def plot_loss(cases: List[CaseView], output: Path) -> Path:
    series = {}
    for c in sorted(cases, key=lambda c: (c.stage, c.bandwidth_gbps)):
        steps, losses = parse_loss_log(c.log_path)
        if steps:
            series[f"stage {c.stage}, bw {_bw_label(c.bandwidth_gbps)}, model {c.model_size}"] = list(zip(steps, losses))
    if not series:
        raise RuntimeError("No parsable loss data found in logs for the selected cases")
    return svg.line_chart(series, output, title="ZeRO Training Loss Curves", xlabel="Step", ylabel="Loss")


_BW_METRICS = {"throughput": ("mean_tokens_per_s", "Tokens / s", "Throughput vs Bandwidth"),
               "tflops": ("mean_tflops_per_s", "Approx. training TFLOPs / s", "Approx. Training TFLOPs vs Bandwidth"),
               "comm": ("mean_comm_ms", "Mean communication ms / step", "Communication Cost vs Bandwidth")}


def plot_bandwidth_metric(cases: List[CaseView], metric: str, output: Path) -> Path:
    """One line per stage over finite bandwidths; the unlimited run is drawn at an extra 'inf' tick."""
    key, ylabel, title = _BW_METRICS[metric]
    finite = sorted({c.bandwidth_gbps for c in cases if c.bandwidth_gbps > 0})
    inf_x = (finite[-1] * 1.25) if finite else 1.0
    series = {}
    for stage in sorted({c.stage for c in cases}):
        pts = [(c.bandwidth_gbps if c.bandwidth_gbps > 0 else inf_x, getattr(c, key))
               for c in cases if c.stage == stage and c.return_code == 0 and getattr(c, key) is not None]
        if pts:
            if metric != "comm" and finite:
                pts.append((0.0, 0.0))
            series[f"stage {stage}"] = pts
    if not series:
        raise RuntimeError(f"No data points available for metric '{metric}'")
    return svg.line_chart(series, output, title=title, xlabel="Bandwidth limit (Gbps)", ylabel=ylabel,
                          x_tick_labels={inf_x: "inf"})


def plot_stage_metric(cases: List[CaseView], metric: str, output: Path) -> Path:
    key = "mean_tokens_per_s" if metric == "stage-throughput" else "mean_comm_ms"
    chosen = [c for c in _representative_cases_by_stage(c for c in cases if c.return_code == 0)
              if getattr(c, key) is not None]
    if not chosen:
        raise RuntimeError(f"No metric data available for plot '{metric}'")
    return svg.bar_chart([f"stage {c.stage}" for c in chosen], {key: [getattr(c, key) for c in chosen]}, output,
                         title="Throughput by ZeRO Stage" if key == "mean_tokens_per_s" else "Communication by ZeRO Stage",
                         xlabel="ZeRO stage",
                         ylabel="Tokens / s" if key == "mean_tokens_per_s" else "Mean communication ms / step",
                         annotate=True)


def plot_grouped_stage_throughput(cases: List[CaseView], output: Path) -> Path:
    ok = [c for c in cases if c.return_code == 0 and c.mean_tokens_per_s is not None]
    if not ok:
        raise RuntimeError("No successful cases available for grouped throughput plotting")
    stages = sorted({c.stage for c in ok})
    groups = {}
    for model in sorted({c.model_size for c in ok}):
        vals = []
        for s in stages:
            pick = _representative_cases_by_stage(c for c in ok if c.model_size == model and c.stage == s)
            vals.append(float(pick[0].mean_tokens_per_s) if pick else 0.0)
        groups[model] = vals
    return svg.bar_chart([f"stage {s}" for s in stages], groups, output, xlabel="ZeRO stage", ylabel="Tokens / s",
                         title="Throughput by ZeRO Stage and Model Size")


def _stacked_by_stage(cases: List[CaseView], split, labels: Tuple[str, ...], output: Path, title: str, ylabel: str,
                      empty: str) -> Path:
    rows = []
    for c in _representative_cases_by_stage(c for c in cases if c.return_code == 0):
        parts = split(c)
        if parts is not None:
            rows.append((c.stage, parts))
    if not rows:
        raise RuntimeError(empty)
    groups = {lab: [parts[i] for _, parts in rows] for i, lab in enumerate(labels)}
    return svg.bar_chart([f"stage {s}" for s, _ in rows], groups, output, title=title, xlabel="ZeRO stage",
                         ylabel=ylabel, stacked=True)


def plot_measured_state_memory(cases: List[CaseView], output: Path) -> Path:
    def split(c):
        b = _case_logical_state_breakdown(c)
        return None if b is None else (b["params_mb"], b["grads_mb"], b["optimizer_mb"])
    return _stacked_by_stage(cases, split, ("params", "grads", "optimizer"), output,
                             "Logical ZeRO Model State Memory by Stage", "State memory (MB)",
                             "No measured state memory data available in the selected cases")


def plot_peak_memory(cases: List[CaseView], output: Path) -> Path:
    return _stacked_by_stage(cases, _case_peak_breakdown_mb, ("logical model state", "peak transient / residual"),
                             output, "Measured Step Peak GPU Memory by ZeRO Stage", "Peak memory (MB)",
                             "No peak memory data available in the selected cases")


def plot_average_memory(cases: List[CaseView], output: Path) -> Path:
    return _stacked_by_stage(cases, _case_average_live_breakdown_mb, ("model state", "avg live non-state"), output,
                             "Average Sampled GPU Memory by ZeRO Stage", "Average sampled live memory (MB)",
                             "No sampled memory data available for average-memory plotting")


def render(cases: List[CaseView], plot: str, output: Path) -> Path:
    if plot == "loss":
        return plot_loss(cases, output)
    if plot in _BW_METRICS:
        return plot_bandwidth_metric(cases, plot, output)
    if plot in ("stage-throughput", "stage-comm"):
        return plot_stage_metric(cases, plot, output)
    if plot == "grouped-stage-throughput":
        return plot_grouped_stage_throughput(cases, output)
    if plot == "memory":
        return plot_measured_state_memory(cases, output)
    if plot == "peak-memory":
        return plot_peak_memory(cases, output)
    if plot == "avg-memory":
        return plot_average_memory(cases, output)
    raise ValueError(f"Unsupported plot type: {plot}")


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Plot harness run outputs (SVG)")
    p.add_argument("--run-dir", type=str, required=True, help="experiments/results/<name>")
    p.add_argument("--plot", type=str, default="throughput", choices=PLOTS)
    p.add_argument("--output", type=str, default="analysis/figures/plot.svg",
                   help="Output path; the suffix is replaced by .svg")
    p.add_argument("--model-size", type=str, default="", help="Optional filter for one model size")
    p.add_argument("--bandwidth-gbps-filter", type=float, default=None,
                   help="Optional exact-match bandwidth filter for memory-oriented plots")
    return p.parse_args(argv)


def main(argv=None) -> None:
    args = parse_args(argv)
    summary = Path(args.run_dir) / "summary.json"
    if not summary.exists():
        raise FileNotFoundError(f"summary file not found: {summary}")
    cases = _filter_bandwidth(_filter_cases(parse_summary(summary), args.model_size), args.bandwidth_gbps_filter)
    print(f"[visualize] wrote {render(cases, args.plot, Path(args.output))}")


if __name__ == "__main__":
    main()
