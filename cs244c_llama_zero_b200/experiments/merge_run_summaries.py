"""Merge several harness run directories into one (e.g. a sweep resumed across machines).

Results are keyed by (stage, model, bandwidth, batch, seq_len, grad_accum); a later run directory
replaces an earlier one's result for the same key.  The merged ``summary.json`` keeps the first run's
top-level fields, records where each result came from, and (unless ``--skip-report``) gets a
``bandwidth_report.md``.  Same key and output as the reference's ``experiments/merge_run_summaries.py``.

    python -m cs244c_llama_zero_b200.experiments.merge_run_summaries --run-dirs runA runB --output-run-dir merged
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Dict, List, Optional, Tuple

from cs244c_llama_zero_b200.analysis import bandwidth_report

_KEY_FIELDS = ("stage", "model_size", "bandwidth_gbps", "batch_size", "seq_len", "grad_accum_steps")
_KEY_NAMES = ("stage", "model", "bw", "batch", "seq", "ga")


def result_key(result: Dict[str, object]) -> Tuple[object, ...]:
    cfg = result.get("config", {})
    cfg = cfg if isinstance(cfg, dict) else {}
    return tuple(cfg.get(f) for f in _KEY_FIELDS)


def key_str(key: Tuple[object, ...]) -> str:
    return "|".join(f"{n}={v}" for n, v in zip(_KEY_NAMES, key))


def load_summary(run_dir: Path) -> Dict[str, object]:
    path = run_dir / "summary.json"
    if not path.exists():
        raise FileNotFoundError(f"missing summary.json under {run_dir}")
    data = json.loads(path.read_text())
    if not isinstance(data, dict):
        raise ValueError(f"summary.json under {run_dir} must contain a JSON object")
    return data


def merge(run_dirs: List[Path], output_run_dir: Path, name: str = "", overwrite: bool = False,
          report: bool = True) -> Dict[str, object]:
    run_dirs = [Path(d).resolve() for d in run_dirs]
    out_dir = Path(output_run_dir).resolve()
    if out_dir.exists() and not overwrite:
        raise FileExistsError(f"output run dir already exists: {out_dir}")
    out_dir.mkdir(parents=True, exist_ok=True)
    summaries = [load_summary(d) for d in run_dirs]
    merged: Dict[Tuple[object, ...], Dict[str, object]] = {}
    source: Dict[Tuple[object, ...], str] = {}
    for summary, d in zip(summaries, run_dirs):
        for r in summary.get("results", []):
            if isinstance(r, dict):
                k = result_key(r)
                merged[k] = r
                source[k] = str(d)
    order = sorted(merged, key=lambda k: (-1 if k[0] is None else int(k[0]), 0.0 if k[2] is None else float(k[2]),
                                          "" if k[1] is None else str(k[1])))
    out = {**summaries[0], "name": name or out_dir.name, "num_cases": len(merged),
           "num_failures": sum(int(r.get("return_code", 0)) != 0 for r in merged.values()),
           "results": [merged[k] for k in order], "merged_from_run_dirs": [str(d) for d in run_dirs],
           "merged_result_sources": {key_str(k): s for k, s in source.items()}}
    (out_dir / "summary.json").write_text(json.dumps(out, indent=2) + "\n")
    print(f"[merge-runs] wrote {out_dir / 'summary.json'}")
    if report:
        (out_dir / "bandwidth_report.md").write_text(bandwidth_report.generate_report_markdown(out_dir))
        print(f"[merge-runs] wrote {out_dir / 'bandwidth_report.md'}")
    return out


def main(argv: Optional[List[str]] = None) -> None:
    p = argparse.ArgumentParser(description="Merge multiple harness summary.json files into one combined run dir")
    p.add_argument("--run-dirs", nargs="+", required=True, help="Run directories that contain summary.json")
    p.add_argument("--output-run-dir", type=str, required=True)
    p.add_argument("--name", type=str, default="", help="Defaults to the output directory name")
    p.add_argument("--overwrite", action="store_true")
    p.add_argument("--skip-report", action="store_true")
    a = p.parse_args(argv)
    merge([Path(d) for d in a.run_dirs], Path(a.output_run_dir), a.name, a.overwrite, not a.skip_report)


if __name__ == "__main__":
    main()
