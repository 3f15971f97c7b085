"""Summarise the per-collective trace that ``train_zero.py --profile-collectives`` writes into its profile JSON.

Each traced call is ``{"op", "label", "elapsed_ms", "input_bytes", "output_bytes"}`` (labels such as
``stage3.forward.allgather.layers.0``).  The report aggregates calls by (op, label), sorted by total
time, then totals time per op.  Same layout as the reference's ``analysis/collective_trace_report.py``.

    python -m cs244c_llama_zero_b200.analysis.collective_trace_report run/profiles/<case>.json
"""

from __future__ import annotations

import argparse
import json
from collections import defaultdict
from pathlib import Path
from typing import Dict, List

from cs244c_llama_zero_b200.parallel.collectives import aggregate_collective_trace

MB = 1024.0 * 1024.0


def summarize_records(records: List[Dict[str, object]]) -> List[Dict[str, object]]:
    return aggregate_collective_trace(records)


def render_profile(path: Path) -> str:
    payload = json.loads(Path(path).read_text())
    steps = payload.get("steps", []) or []
    summary = summarize_records([r for s in steps for r in s.get("collective_trace", []) or []])
    lines = [f"# {path}", "", "## Context", "", f"- stage: `{payload.get('stage')}`",
             f"- batch size / GPU: `{payload.get('microbatch_size_per_gpu')}`",
             f"- seq len: `{(payload.get('args', {}) or {}).get('seq_len')}`", f"- steps with trace: `{len(steps)}`", "",
             "## Aggregate Trace", "", "| op | label | calls | elapsed ms | input MB | output MB |",
             "| --- | --- | --- | --- | --- | --- |"]
    per_op: Dict[str, float] = defaultdict(float)
    for it in summary:
        lines.append(f"| {it['op']} | {it['label']} | {it['calls']} | {it['elapsed_ms']:.1f} | "
                     f"{it['input_bytes'] / MB:.2f} | {it['output_bytes'] / MB:.2f} |")
        per_op[str(it["op"])] += float(it["elapsed_ms"])
    lines += ["", "## By Operation", ""]
    lines += [f"- `{op}`: `{ms:.1f} ms`" for op, ms in sorted(per_op.items(), key=lambda kv: (-kv[1], kv[0]))]
    return "\n".join(lines) + "\n"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Summarize collective trace data from train_zero profile JSON")
    p.add_argument("profiles", nargs="+", help="One or more profile JSON files")
    for raw in p.parse_args(argv).profiles:
        print(render_profile(Path(raw)))


if __name__ == "__main__":
    main()
