"""Ship the repo to a remote GPU host, run the harness matrix there, pull results back, plot and report.

    python -m cs244c_llama_zero_b200.experiments.run_remote_bandwidth_sweep --host gpu-box \
        --config cs244c_llama_zero_b200/experiments/configs/b200_small_bandwidth_socket.json
"""

from __future__ import annotations

import argparse
from typing import List, Optional

from .remote import PROJECT_ROOT, add_remote_args, bandwidth_postprocess, run_remote

DEFAULT_CONFIG = PROJECT_ROOT / "cs244c_llama_zero_b200" / "experiments" / "configs" / "b200_bandwidth_smoke.json"
DEFAULT_PLOTS = ["throughput", "comm", "tflops", "stage-throughput", "stage-comm", "loss"]


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Ship the current repo to a clean remote workspace and run a bandwidth sweep")
    add_remote_args(p, default_config=str(DEFAULT_CONFIG), extra_flag="--extra-harness-args", default_plots=DEFAULT_PLOTS)
    return p.parse_args(argv)


def main(argv: Optional[List[str]] = None, session=None) -> None:
    run_remote(parse_args(argv), module="harness", tag="remote-sweep", postprocess=bandwidth_postprocess("remote-sweep"),
               session=session)


if __name__ == "__main__":
    main()
