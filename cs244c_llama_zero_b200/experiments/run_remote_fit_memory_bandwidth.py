"""Remote fit-to-memory bandwidth sweep: tune each stage's micro-batch on the remote GPUs, sweep, report here.

    python -m cs244c_llama_zero_b200.experiments.run_remote_fit_memory_bandwidth --host gpu-box \
        --config cs244c_llama_zero_b200/experiments/configs/b200_1p3b_fit_memory.json
"""

from __future__ import annotations

import argparse
from typing import List, Optional

from .remote import PROJECT_ROOT, add_remote_args, bandwidth_postprocess, run_remote

DEFAULT_CONFIG = PROJECT_ROOT / "cs244c_llama_zero_b200" / "experiments" / "configs" / "b200_1p3b_fit_memory.json"
DEFAULT_PLOTS = ["throughput", "comm", "stage-throughput", "peak-memory"]


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Ship the repo to a remote host and run the fit-to-memory bandwidth sweep")
    add_remote_args(p, default_config=str(DEFAULT_CONFIG), extra_flag="--extra-fit-args", default_plots=DEFAULT_PLOTS)
    return p.parse_args(argv)


def main(argv: Optional[List[str]] = None, session=None) -> None:
    run_remote(parse_args(argv), module="run_fit_memory_bandwidth", tag="remote-fit-memory",
               postprocess=bandwidth_postprocess("remote-fit-memory"), session=session)


if __name__ == "__main__":
    main()
