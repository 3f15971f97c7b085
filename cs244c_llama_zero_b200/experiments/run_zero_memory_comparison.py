"""ZeRO stage 0-3 memory comparison: one harness run over all stages at unlimited bandwidth, then memory plots.

Each stage trains a few warm-up steps and then one measured step with reset CUDA peak statistics
(``--measure-memory-step``), so the peak of that step and the live ZeRO state (params, grads,
optimizer) at each phase land in the profile JSON.  The run directory then gets three SVG charts:
logical state per stage, the measured peak split into state vs the rest, and the average live
memory split the same way.  Same flags as the reference's ``experiments/run_zero_memory_comparison.py``.

    python -m cs244c_llama_zero_b200.experiments.run_zero_memory_comparison --model-size baseline-1.3b \
        --seq-len 1024 --batch-size 8 --nproc-per-node 8
"""

from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
from typing import List, Optional

from cs244c_llama_zero_b200.analysis import visualize

from . import harness
from .common import MODEL_SIZES


def _build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Run a ZeRO stage memory comparison sweep")
    p.add_argument("--config", type=str, default="")
    p.add_argument("--name", type=str, default="", help="Run name; generated from the workload when omitted.")
    p.add_argument("--results-dir", type=str, default="experiments/results")
    p.add_argument("--model-size", type=str, default="small", choices=MODEL_SIZES)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--batch-size", type=int, default=92)
    p.add_argument("--grad-accum-steps", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--dtype", type=str, default="bfloat16", choices=["float32", "bfloat16"])
    p.add_argument("--collective-impl", type=str, default="torch", choices=harness.COLLECTIVE_IMPLS)
    p.add_argument("--nproc-per-node", type=int, default=0, help="0 = all visible GPUs.")
    p.add_argument("--profile-memory-interval", type=int, default=1)
    p.add_argument("--master-addr", type=str, default="127.0.0.1")
    p.add_argument("--master-port-base", type=int, default=29500)
    p.add_argument("--case-timeout-s", type=float, default=1800.0)
    p.add_argument("--seed", type=int, default=1337)
    p.add_argument("--measure-memory-step", action=argparse.BooleanOptionalAction, default=True,
                   help="Warm up, then record one measured step with reset CUDA peak stats.")
    p.add_argument("--memory-warmup-steps", type=int, default=None,
                   help="Defaults to steps - 1 when the measured step is enabled.")
    p.add_argument("--skip-existing", action="store_true")
    p.add_argument("--skip-plots", action="store_true")
    p.add_argument("--dry-run", action="store_true")
    return p


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    parser = _build_parser()
    prelim, _ = parser.parse_known_args(argv)
    if prelim.config:
        defaults = json.loads(Path(prelim.config).read_text()).get("defaults", {})
        if isinstance(defaults, dict):
            parser.set_defaults(**defaults)
    return parser.parse_args(argv)


def detect_visible_gpus() -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if visible:
        return len([d for d in visible.split(",") if d.strip()])
    import torch

    return int(torch.cuda.device_count())


def default_run_name(args: argparse.Namespace) -> str:
    kind = "measured_step" if args.measure_memory_step else "train"
    return f"{args.model_size}_memory_{kind}_bs{args.batch_size}_allgpus_project"


def harness_argv(args: argparse.Namespace, nproc: int, run_name: str) -> List[str]:
    steps = args.steps
    extra = ""
    if args.measure_memory_step:
        warm = args.memory_warmup_steps if args.memory_warmup_steps is not None else max(args.steps - 1, 0)
        steps = warm + 1
        extra = f"--measure-memory-step --memory-warmup-steps {warm}"
    argv = ["--name", run_name, "--results-dir", str(args.results_dir), "--stages", "0", "1", "2", "3",
            "--model-sizes", args.model_size, "--bandwidth-gbps", "0", "--nproc-per-node", str(nproc),
            "--steps", str(steps), "--seq-len", str(args.seq_len), "--batch-size", str(args.batch_size),
            "--grad-accum-steps", str(args.grad_accum_steps), "--collective-impl", args.collective_impl,
            "--data-mode", "synthetic", "--dtype", args.dtype, "--seed", str(args.seed),
            "--profile-memory-interval", str(args.profile_memory_interval), "--bandwidth-mode", "none",
            "--master-addr", args.master_addr, "--master-port-base", str(args.master_port_base),
            "--case-timeout-s", str(args.case_timeout_s)]
    if extra:
        argv += ["--extra-args", extra]
    if args.skip_existing:
        argv.append("--skip-existing")
    if args.dry_run:
        argv.append("--dry-run")
    return argv


def main(argv: Optional[List[str]] = None) -> None:
    args = parse_args(argv)
    nproc = args.nproc_per_node if args.nproc_per_node > 0 else detect_visible_gpus()
    if nproc < 1:
        raise SystemExit("No visible GPUs detected. Set CUDA_VISIBLE_DEVICES or pass --nproc-per-node.")
    if nproc == 1:
        print("[memory-sweep] warning: 1 GPU; stage-to-stage sharding effects will not be representative", flush=True)
    name = args.name or default_run_name(args)
    run_dir = Path(args.results_dir) / name
    print(f"[memory-sweep] nproc_per_node={nproc} run_name={name} output_dir={run_dir}", flush=True)
    harness.run_matrix(harness.parse_args(harness_argv(args, nproc, name)))
    if args.dry_run or args.skip_plots:
        print("[memory-sweep] run complete; skipping plot generation", flush=True)
        return
    cases = visualize._filter_cases(visualize.parse_summary(run_dir / "summary.json"), args.model_size)
    for kind, stem in (("memory", "memory"), ("peak-memory", "peak_memory"), ("avg-memory", "avg_memory")):
        print(f"[memory-sweep] wrote {visualize.render(cases, kind, run_dir / f'{stem}.svg')}", flush=True)


if __name__ == "__main__":
    main()
