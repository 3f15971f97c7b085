"""Remote stage-3 GPU-count scaling sweep, with the Figure-3-style chart and report rendered locally.

    python -m cs244c_llama_zero_b200.experiments.run_remote_stage3_scaling --host gpu-box \
        --config cs244c_llama_zero_b200/experiments/configs/b200_1p3b_stage3_scaling.json
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import List, Optional

from .remote import PROJECT_ROOT, add_remote_args, run_remote

DEFAULT_CONFIG = PROJECT_ROOT / "cs244c_llama_zero_b200" / "experiments" / "configs" / "b200_1p3b_stage3_scaling.json"


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Ship the repo to a remote host and run the Stage 3 GPU-scaling sweep")
    add_remote_args(p, default_config=str(DEFAULT_CONFIG), extra_flag="--extra-scaling-args", default_plots=[])
    p.add_argument("--baseline-gpu-count", type=int, default=0)
    return p.parse_args(argv)


def _post(run_dir: Path, args: argparse.Namespace) -> Optional[Path]:
    from cs244c_llama_zero_b200.analysis import stage3_scaling

    summary_path = run_dir / "summary.json"
    if args.skip_summary or not summary_path.exists():
        return None
    summary = json.loads(summary_path.read_text())
    try:
        raw = stage3_scaling.scaling_points(summary)
    except RuntimeError as exc:
        print(f"[remote-stage3] warning: {exc}")
        return None
    base = stage3_scaling.choose_baseline_gpu_count(raw, int(args.baseline_gpu_count))
    points = stage3_scaling.annotate_points(raw, base)
    if not args.skip_plots:
        stage3_scaling.plot_figure(points, run_dir / "stage3_scaling.svg", base)
    report = run_dir / "stage3_scaling_report.md"
    report.write_text(stage3_scaling.render_report(summary, points, base))
    return report


def main(argv: Optional[List[str]] = None, session=None) -> None:
    run_remote(parse_args(argv), module="run_stage3_scaling_sweep", tag="remote-stage3", postprocess=_post,
               session=session)


if __name__ == "__main__":
    main()
