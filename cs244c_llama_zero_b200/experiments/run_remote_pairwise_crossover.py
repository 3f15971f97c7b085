"""Remote pairwise crossover search: the adaptive two-stage bandwidth search on a remote host.

The remote run writes ``pairwise_report.md`` itself; it comes back with the run directory.

    python -m cs244c_llama_zero_b200.experiments.run_remote_pairwise_crossover --host gpu-box \
        --config cs244c_llama_zero_b200/experiments/configs/b200_small_pairwise_crossover_socket.json
"""

from __future__ import annotations

import argparse
from pathlib import Path
from typing import List, Optional

from .remote import PROJECT_ROOT, add_remote_args, run_remote

DEFAULT_CONFIG = (PROJECT_ROOT / "cs244c_llama_zero_b200" / "experiments" / "configs"
                  / "b200_small_pairwise_crossover_socket.json")


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Ship the repo to a remote host and run the pairwise crossover search")
    add_remote_args(p, default_config=str(DEFAULT_CONFIG), extra_flag="--extra-search-args", default_plots=[])
    return p.parse_args(argv)


def _post(run_dir: Path, args: argparse.Namespace) -> Optional[Path]:
    report = run_dir / "pairwise_report.md"
    return report if report.exists() else None


def main(argv: Optional[List[str]] = None, session=None) -> None:
    run_remote(parse_args(argv), module="run_pairwise_crossover_search", tag="remote-pairwise", postprocess=_post,
               session=session)


if __name__ == "__main__":
    main()
