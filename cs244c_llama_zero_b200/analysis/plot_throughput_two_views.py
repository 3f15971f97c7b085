"""Two views of TFLOP/s against bandwidth for a run directory: a 0-10 Gbps zoom and a full overview
(unlimited drawn at an extra 'inf' tick).  SVG output; same two views as the reference's
``analysis/plot_throughput_two_views.py``.
"""

from __future__ import annotations

import argparse
from pathlib import Path
from typing import Dict, List

from . import svg
from .visualize import CaseView, parse_summary


def cases_by_stage(cases: List[CaseView]) -> Dict[int, List[CaseView]]:
    out: Dict[int, List[CaseView]] = {}
    for c in cases:
        if c.return_code == 0 and c.mean_tflops_per_s is not None:
            out.setdefault(c.stage, []).append(c)
    return out


def plot_zoom(by_stage: Dict[int, List[CaseView]], output: Path) -> Path:
    series = {f"stage {s}": [(0.0, 0.0)] + sorted((c.bandwidth_gbps, c.mean_tflops_per_s) for c in cs
                                                   if 0.0 < c.bandwidth_gbps <= 10.0)
              for s, cs in sorted(by_stage.items())}
    return svg.line_chart(series, output, title="TFLOPs vs Bandwidth (0-10 Gbps)", xlabel="Bandwidth limit (Gbps)",
                          ylabel="Approx. training TFLOPs / s")


def plot_overview(by_stage: Dict[int, List[CaseView]], output: Path) -> Path:
    finite = sorted({c.bandwidth_gbps for cs in by_stage.values() for c in cs if c.bandwidth_gbps > 0})
    inf_x = finite[-1] * 1.25 if finite else 1.0
    series = {f"stage {s}": sorted((c.bandwidth_gbps if c.bandwidth_gbps > 0 else inf_x, c.mean_tflops_per_s)
                                   for c in cs) for s, cs in sorted(by_stage.items())}
    return svg.line_chart(series, output, title="TFLOPs vs Bandwidth", xlabel="Bandwidth limit (Gbps)",
                          ylabel="Approx. training TFLOPs / s", x_tick_labels={inf_x: "inf"})


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Draw zoomed and overview throughput-vs-bandwidth plots (SVG)")
    p.add_argument("--run-dir", required=True)
    p.add_argument("--zoom-output", required=True)
    p.add_argument("--overview-output", required=True)
    a = p.parse_args(argv)
    by_stage = cases_by_stage(parse_summary(Path(a.run_dir) / "summary.json"))
    if not by_stage:
        raise RuntimeError("no successful cases with TFLOPs in this run")
    print(f"[two-views] wrote {plot_zoom(by_stage, Path(a.zoom_output))}")
    print(f"[two-views] wrote {plot_overview(by_stage, Path(a.overview_output))}")


if __name__ == "__main__":
    main()
