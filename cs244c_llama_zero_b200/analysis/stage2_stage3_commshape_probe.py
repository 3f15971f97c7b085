"""Per-phase communication shape of stage 2 and stage 3 runs, from the per-rank profile JSON.

For every (model, bandwidth, stage) profile under ``<run-dir>/profiles`` it averages, over the
steps from ``--start-step`` on, the iteration / forward-backward / optimizer / communication times
and each communication phase's time, call count and bytes (``communication_<phase>_{ms,calls,bytes}``
with phases backward_reduce_scatter, post_allgather, forward_allgather, backward_allgather), then
prints stage-2 and stage-3 tables and a stage-3 / stage-2 comparison per bandwidth (markdown, optional
CSV).  Same quantities as the reference's ``analysis/stage2_stage3_commshape_probe.py``.
"""

from __future__ import annotations

import argparse
import csv
import json
import re
from collections import defaultdict
from pathlib import Path
from typing import Dict, List, Optional, Set, Tuple

PHASES = ("backward_reduce_scatter", "post_allgather", "forward_allgather", "backward_allgather")
BASE = ("iteration_ms", "forward_backward_ms", "optimizer_ms", "communication_ms", "tokens_per_second")


def _mean(xs: List[float]) -> Optional[float]:
    return sum(xs) / len(xs) if xs else None


def bandwidth_from_case_id(case_id: str) -> float:
    m = re.search(r"_bw(unlimited|[0-9.]+)gbps", case_id) or re.search(r"_bw(unlimited)_", case_id)
    return 0.0 if m is None or m.group(1) == "unlimited" else float(m.group(1))


def summarize_profile(payload: Dict[str, object], start_step: int) -> Optional[Dict[str, object]]:
    steps = [s for s in payload.get("steps", []) or [] if isinstance(s, dict) and int(s.get("step", 0)) >= start_step]
    if not steps:
        return None
    out: Dict[str, object] = {"stage": int(payload.get("stage", 0)),
                              "model": str((payload.get("model_config") or {}).get("name", "unknown")),
                              "samples": len(steps)}
    for k in BASE:
        out[k] = _mean([float(s.get(k, 0.0) or 0.0) for s in steps])
    for ph in PHASES:
        for f in ("ms", "calls", "bytes"):
            key = f"communication_{ph}_{f}"
            out[f"{ph}_{f}"] = 0.0 if out["stage"] == 2 and ph in PHASES[2:] else \
                _mean([float(s.get(key, 0.0) or 0.0) for s in steps])
    return out


def load_profiles(run_dir: Path, model: str = "", start_step: int = 2,
                  bandwidths: Optional[Set[float]] = None) -> Dict[Tuple[str, float, int], Dict[str, object]]:
    pdir = Path(run_dir) / "profiles"
    if not pdir.exists():
        raise FileNotFoundError(f"missing profiles directory: {pdir}")
    out = {}
    for path in sorted(pdir.glob("*.json")):
        payload = json.loads(path.read_text())
        if int(payload.get("stage", 0)) not in (2, 3):
            continue
        bw = bandwidth_from_case_id(path.stem)
        s = summarize_profile(payload, start_step)
        if s is None or (model and s["model"] != model) or (bandwidths is not None and bw not in bandwidths):
            continue
        s["profile_path"] = str(path)
        out[(str(s["model"]), bw, int(s["stage"]))] = s
    return out


def _f(v, digits=2):
    return "NA" if v is None else f"{v:.{digits}f}"


def render(cases: Dict[Tuple[str, float, int], Dict[str, object]]) -> str:
    hdr = ["model", "bw Gbps", "samples", "iter ms", "comm ms", "comm share", "fb ms", "opt ms"]
    rows: Dict[int, List[List[str]]] = defaultdict(list)
    pair: Dict[Tuple[str, float], Dict[int, Dict[str, object]]] = defaultdict(dict)
    for (model, bw, stage), s in sorted(cases.items()):
        it, cm = s["iteration_ms"], s["communication_ms"]
        row = [model, f"{bw:g}", str(s["samples"]), _f(it), _f(cm), _f(cm / it * 100, 1) + "%" if it else "NA",
               _f(s["forward_backward_ms"]), _f(s["optimizer_ms"])]
        for ph in (PHASES[:2] if stage == 2 else PHASES):
            calls = s[f"{ph}_calls"]
            row += [_f(s[f"{ph}_ms"]), _f(calls), _f((s[f"{ph}_bytes"] or 0) / 2**20),
                    _f(s[f"{ph}_ms"] / calls if calls else None)]
        rows[stage].append(row)
        pair[(model, bw)][stage] = s
    parts = []
    for stage, phases in ((2, PHASES[:2]), (3, PHASES)):
        h = hdr + [f"{ph} {f}" for ph in phases for f in ("ms", "calls", "MB", "ms/call")]
        parts += [f"## Stage {stage}", "", "| " + " | ".join(h) + " |", "| " + " | ".join("---" for _ in h) + " |"]
        parts += ["| " + " | ".join(r) + " |" for r in rows.get(stage, [])] + [""]
    parts += ["## Stage 3 / stage 2", "", "| model | bw Gbps | iter ratio | comm ratio | tokens/s ratio |",
              "| --- | --- | --- | --- | --- |"]
    for (model, bw), d in sorted(pair.items()):
        if 2 in d and 3 in d:
            r = lambda k: (d[3][k] / d[2][k]) if d[2][k] else None  # noqa: E731
            parts.append(f"| {model} | {bw:g} | {_f(r('iteration_ms'), 3)} | {_f(r('communication_ms'), 3)} | "
                         f"{_f(r('tokens_per_second'), 3)} |")
    return "\n".join(parts) + "\n"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Stage-2 vs stage-3 communication shape from profile JSON")
    p.add_argument("--run-dir", required=True)
    p.add_argument("--model-size", default="")
    p.add_argument("--start-step", type=int, default=2)
    p.add_argument("--bandwidth-gbps", nargs="+", type=float, default=None)
    p.add_argument("--output-csv", default="")
    a = p.parse_args(argv)
    cases = load_profiles(Path(a.run_dir), a.model_size, a.start_step,
                          None if a.bandwidth_gbps is None else set(a.bandwidth_gbps))
    if not cases:
        raise RuntimeError("no matching profiles found")
    print(render(cases))
    if a.output_csv:
        keys = sorted({k for s in cases.values() for k in s})
        with open(a.output_csv, "w", newline="") as fh:
            w = csv.DictWriter(fh, fieldnames=["model", "bandwidth_gbps", "stage"] + keys)
            w.writeheader()
            for (model, bw, stage), s in sorted(cases.items()):
                w.writerow({"model": model, "bandwidth_gbps": bw, **s, "stage": stage})


if __name__ == "__main__":
    main()
