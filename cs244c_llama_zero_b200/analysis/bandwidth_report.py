"""Markdown report of a bandwidth sweep run directory (fixed-workload or fit-to-memory).

Per model: the stage workload (micro-batch, global tokens per step and, for fit-to-memory runs, the
tuned peak memory against the budget), the stage ranking and winner transitions by bandwidth, the
best stage per bandwidth, and tokens/s, throughput relative to each stage's own fastest-link run,
and communication ms per step as stage x bandwidth tables.  Section titles and table layouts follow
the reference's ``analysis/bandwidth_report.py`` so reports of both implementations compare line by line.

    python -m cs244c_llama_zero_b200.analysis.bandwidth_report --run-dir experiments/results/<name>
"""

from __future__ import annotations

import argparse
import json
from collections import defaultdict
from pathlib import Path
from typing import Dict, List, Optional

from .visualize import CaseView, parse_summary


def _bw(bw: float) -> str:
    return "unlimited" if bw <= 0 else f"{bw:g} Gbps"


def _num(v: Optional[float], digits: int = 1) -> str:
    return "NA" if v is None else f"{v:.{digits}f}"


def _pct(v: Optional[float]) -> str:
    return "NA" if v is None else f"{v * 100.0:.1f}%"


def _table(headers: List[str], rows: List[List[str]]) -> str:
    out = ["| " + " | ".join(headers) + " |", "| " + " | ".join("---" for _ in headers) + " |"]
    return "\n".join(out + ["| " + " | ".join(r) + " |" for r in rows])


def _opt(v) -> Optional[float]:
    return None if v is None else float(v)


def _load_tuning(run_dir: Path) -> Optional[Dict[str, object]]:
    p = run_dir / "tuning_summary.json"
    if not p.exists():
        return None
    data = json.loads(p.read_text())
    return data if isinstance(data, dict) else None


def _ranked(cases: List[CaseView], bw: float) -> List[CaseView]:
    at = [c for c in cases if abs(c.bandwidth_gbps - bw) < 1e-9 and c.mean_tokens_per_s is not None]
    return sorted(at, key=lambda c: float(c.mean_tokens_per_s), reverse=True)


def _baseline_case(stage_cases: List[CaseView]) -> Optional[CaseView]:
    """The stage's unlimited run, else its fastest finite link."""
    if any(c.bandwidth_gbps <= 0 for c in stage_cases):
        return next(c for c in stage_cases if c.bandwidth_gbps <= 0)
    top = max(c.bandwidth_gbps for c in stage_cases)
    return next(c for c in stage_cases if c.bandwidth_gbps == top)


def _methodology(run_args: Dict[str, object], tuning: Optional[Dict[str, object]]) -> List[str]:
    lines = ["Method:"]
    if tuning is None:
        lines.append("- fixed workload: every stage uses the same per-GPU microbatch, grad accumulation, and sequence "
                     "length")
    else:
        metric = tuning.get("memory_metric", "peak_cuda_max_reserved_mb")
        if str(tuning.get("fit_mode", "memory_budget")) == "oom_boundary":
            lines.append("- fit-to-memory: each stage is first tuned at unlimited bandwidth to the largest per-GPU "
                         "microbatch that completes without OOM")
            lines.append(f"- the selected tuning profile reports `{metric}` for the largest passing microbatch")
        else:
            lines.append("- fit-to-memory: each stage is first tuned at unlimited bandwidth to the largest per-GPU "
                         f"microbatch whose measured `{metric}` stays within "
                         f"{_num(_opt(tuning.get('memory_budget_mb')))} MB")
        lines.append("- the tuned per-stage microbatch is then frozen and reused across the bandwidth sweep")
    mode = str(run_args.get("bandwidth_mode", "unknown"))
    lines.append({"socket": "- communication is forced over NCCL NET/Socket and throttled at the socket layer",
                  "simulated": "- bandwidth is simulated inside the collective interface",
                  "tc": "- bandwidth is throttled with Linux tc on the configured interface",
                  "nvlink": "- every NVLink collective and ZeRO-3 gather is paced on the device to an emulated link "
                            "of the case bandwidth (ring volumes per GPU, Gbit/s)"}.get(
        mode, "- no bandwidth throttling is applied when bandwidth is unlimited"))
    lines.append(f"- per-case metrics are averaged over logged steps after skipping "
                 f"{run_args.get('metrics_warmup_steps', 0)} warmup step(s); nominal step count is "
                 f"{run_args.get('steps', 'unknown')}")
    return lines


def _model_section(model: str, cases: List[CaseView], run_args: Dict[str, object],
                   tuning: Optional[Dict[str, object]]) -> str:
    ok = [c for c in cases if c.return_code == 0]
    if not ok:
        return f"## Model `{model}`\n\nNo successful cases.\n"
    bws = sorted({c.bandwidth_gbps for c in ok})
    stages = sorted({c.stage for c in ok})
    world = int(run_args.get("nproc_per_node", 1))
    at = {(c.stage, c.bandwidth_gbps): c for c in ok}
    first = lambda cs: min(cs, key=lambda c: (c.bandwidth_gbps > 0, c.bandwidth_gbps))  # noqa: E731

    workload_hdr = ["stage", "microbatch / gpu", "global tokens / step"]
    per_stage = dict((tuning or {}).get("per_stage", {}) or {})
    budget = _opt((tuning or {}).get("memory_budget_mb"))
    if tuning is not None:
        label = str(tuning.get("memory_metric", "peak_cuda_max_reserved_mb")).replace("peak_", "").replace(
            "_mb", "").replace("_", " ")
        workload_hdr += [f"selected {label} MB", "budget used"]
    workload = []
    for s in stages:
        sc = [c for c in ok if c.stage == s]
        rep = first(sc)
        row = [str(s), ",".join(str(b) for b in sorted({c.batch_size for c in sc})),
               str(rep.batch_size * rep.grad_accum_steps * rep.seq_len * world)]
        if tuning is not None:
            peak = _opt(per_stage.get(str(s), {}).get("selected_peak_memory_mb"))
            row += [_num(peak), _pct(peak / budget if peak is not None and budget else None)]
        workload.append(row)

    ranking, transitions, best_rows = [], [], []
    prev = None
    for bw in bws:
        r = _ranked(ok, bw)
        if not r:
            continue
        ranking.append([_bw(bw), " > ".join(f"stage {c.stage}" for c in r), str(r[0].stage),
                        _num(r[0].mean_tokens_per_s)])
        if r[0].stage != prev:
            transitions.append(f"- {_bw(bw)}: stage {r[0].stage} is the fastest stage")
        prev = r[0].stage
        best = max((c for c in ok if abs(c.bandwidth_gbps - bw) < 1e-9), key=lambda c: float(c.mean_tokens_per_s or 0.0))
        best_rows.append([_bw(bw), str(best.stage), _num(best.mean_tokens_per_s), _num(best.mean_comm_ms)])

    tput, rel, comm = [], [], []
    for s in stages:
        base = _baseline_case([c for c in ok if c.stage == s])
        base_tps = None if base is None else base.mean_tokens_per_s
        t_row, r_row, c_row = [f"stage {s}"], [f"stage {s}"], [f"stage {s}"]
        for bw in bws:
            c = at.get((s, bw))
            t_row.append(_num(None if c is None else c.mean_tokens_per_s))
            ok_ratio = c is not None and c.mean_tokens_per_s is not None and base_tps not in (None, 0.0)
            r_row.append(_pct(c.mean_tokens_per_s / base_tps) if ok_ratio else "NA")
            c_row.append(_num(None if c is None else c.mean_comm_ms))
        tput.append(t_row)
        rel.append(r_row)
        comm.append(c_row)
    hdr = ["stage"] + [_bw(b) for b in bws]
    rep = first(ok)
    parts = [f"## Model `{model}`", "",
             f"Workload: seq_len={rep.seq_len}, grad_accum_steps={rep.grad_accum_steps}, world_size={world}", "",
             "Stage workload:", _table(workload_hdr, workload), "",
             "Stage ranking by bandwidth:", _table(["bandwidth", "ranking by tokens/s", "winner", "winner tokens/s"],
                                                  ranking), "",
             "Winner transitions:", *transitions, "",
             "Best stage by bandwidth:", _table(["bandwidth", "best stage", "tokens/s", "comm ms"], best_rows), "",
             "Throughput (tokens/s):", _table(hdr, tput), "",
             "Throughput relative to the stage baseline:", _table(hdr, rel), "",
             "Communication time (ms / step):", _table(hdr, comm)]
    failed = sorted((c for c in cases if c.return_code != 0), key=lambda c: (c.stage, c.bandwidth_gbps))
    if failed:
        parts += ["", "Failed cases:"] + [f"- stage {c.stage}, {_bw(c.bandwidth_gbps)}: return_code={c.return_code} "
                                          f"log={c.log_path}" for c in failed]
    parts.append("")
    return "\n".join(parts)


def generate_report_markdown(run_dir: Path) -> str:
    run_dir = Path(run_dir)
    summary_path = run_dir / "summary.json"
    if not summary_path.exists():
        raise FileNotFoundError(f"missing summary.json under {run_dir}")
    summary = json.loads(summary_path.read_text())
    cases = parse_summary(summary_path)
    by_model: Dict[str, List[CaseView]] = defaultdict(list)
    for c in cases:
        by_model[c.model_size].append(c)
    run_args = summary.get("args", {}) if isinstance(summary.get("args", {}), dict) else {}
    tuning = _load_tuning(run_dir)
    kind = "fit-to-memory bandwidth sweep" if tuning is not None else "fixed-workload bandwidth sweep"
    parts = ["# Bandwidth Sweep Report", "", f"Run dir: `{run_dir}`", f"Run name: `{summary.get('name', run_dir.name)}`",
             f"Experiment type: {kind}",
             f"Successful cases: {sum(c.return_code == 0 for c in cases)} / {len(cases)}",
             f"Settings: bandwidth_mode={run_args.get('bandwidth_mode', 'unknown')}, "
             f"nproc_per_node={run_args.get('nproc_per_node', 'unknown')}, steps={run_args.get('steps', 'unknown')}, "
             f"metrics_warmup_steps={run_args.get('metrics_warmup_steps', 0)}", ""]
    parts += _methodology(run_args, tuning) + [""]
    parts += [_model_section(m, by_model[m], run_args, tuning) for m in sorted(by_model)]
    return "\n".join(parts).rstrip() + "\n"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Generate a markdown report for a bandwidth sweep")
    p.add_argument("--run-dir", type=str, required=True, help="experiments/results/<name>")
    p.add_argument("--output", type=str, default="", help="Defaults to <run-dir>/bandwidth_report.md")
    args = p.parse_args(argv)
    out = Path(args.output) if args.output else Path(args.run_dir) / "bandwidth_report.md"
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(generate_report_markdown(Path(args.run_dir)))
    print(f"[bandwidth-report] wrote {out}")


if __name__ == "__main__":
    main()
