"""Shared command-line groups and case construction for the tuning/sweep runners.

Each runner (fit-to-memory bandwidth sweep, stage-3 GPU-count sweep, pairwise crossover search) builds
``harness.CaseConfig`` launches of ``train_zero.py`` from the same flag groups; defaults differ per
runner and are passed in.  A ``--config`` JSON (``{"defaults": {...}, "matrix": {...}}``) supplies
parser defaults, explicit flags win.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Dict, List, Optional

from cs244c_llama_zero_b200.models.config import PRESETS

from . import harness
from .tuning import MEMORY_METRICS

MODEL_SIZES = sorted(PRESETS)


def add_run_args(p: argparse.ArgumentParser, name: str) -> None:
    p.add_argument("--config", type=str, default="")
    p.add_argument("--name", type=str, default=name)
    p.add_argument("--results-dir", type=str, default="experiments/results")
    p.add_argument("--skip-existing", action="store_true")
    p.add_argument("--dry-run", action="store_true")


def add_launch_args(p: argparse.ArgumentParser, *, nproc: Optional[int], timeout_s: float) -> None:
    if nproc is not None:
        p.add_argument("--nproc-per-node", type=int, default=nproc)
    p.add_argument("--nnodes", type=int, default=1)
    p.add_argument("--node-rank", type=int, default=0)
    p.add_argument("--master-addr", type=str, default="127.0.0.1")
    p.add_argument("--master-port-base", type=int, default=29500)
    p.add_argument("--case-timeout-s", type=float, default=timeout_s)


def add_training_args(p: argparse.ArgumentParser, *, model_size: str, steps: int, seq_len: int,
                      model_flag: str = "--model-size") -> None:
    p.add_argument(model_flag, type=str, default=model_size, choices=MODEL_SIZES)
    p.add_argument("--steps", type=int, default=steps)
    p.add_argument("--seq-len", type=int, default=seq_len)
    p.add_argument("--grad-accum-steps", type=int, default=1)
    p.add_argument("--collective-impl", type=str, default="torch", choices=harness.COLLECTIVE_IMPLS)
    p.add_argument("--data-mode", type=str, default="synthetic", choices=["synthetic", "fineweb", "random"])
    p.add_argument("--seed", type=int, default=1337)
    p.add_argument("--dtype", type=str, default="bfloat16", choices=["float32", "bfloat16"])
    p.add_argument("--max-grad-norm", type=float, default=0.0)
    p.add_argument("--stage2-grad-bucket-mb", type=float, default=64.0,
                   help="Approximate fp32 gradient bucket size for ZeRO stage 2 reduce-scatter bucketing.")
    p.add_argument("--profile-memory-interval", type=int, default=0)
    p.add_argument("--metrics-warmup-steps", type=int, default=2)
    p.add_argument("--theory-vocab-size", type=int, default=0)
    p.add_argument("--extra-args", type=str, default="")


def add_bandwidth_args(p: argparse.ArgumentParser, *, mode: str = "socket") -> None:
    p.add_argument("--bandwidth-mode", type=str, default=mode, choices=["simulated", "none", "tc", "socket", "nvlink"])
    p.add_argument("--sim-latency-ms", type=float, default=0.0)
    p.add_argument("--tc-interface", type=str, default="eth0")
    p.add_argument("--socket-interface", type=str, default="lo")
    p.add_argument("--socket-shaper-burst-bytes", type=int, default=262_144)


def add_tuning_args(p: argparse.ArgumentParser, *, max_batch: int, multiple: int,
                    fit_modes: List[str]) -> None:
    p.add_argument("--fit-mode", type=str, default="oom_boundary", choices=fit_modes,
                   help="How to decide whether a microbatch size fits during tuning.")
    p.add_argument("--memory-metric", type=str, default="peak_cuda_max_allocated_mb", choices=list(MEMORY_METRICS))
    p.add_argument("--min-batch-size", type=int, default=1)
    p.add_argument("--max-batch-size", type=int, default=max_batch)
    p.add_argument("--initial-batch-size", type=int, default=0,
                   help="Initial microbatch guess for tuning. 0 uses the midpoint of the search interval.")
    p.add_argument("--batch-size-multiple", type=int, default=multiple)
    p.add_argument("--growth-factor", type=float, default=2.0)
    p.add_argument("--tuning-memory-warmup-steps", type=int, default=2)


def parse_with_config(parser: argparse.ArgumentParser, argv: Optional[List[str]],
                      matrix_keys=("stages", "model_sizes", "bandwidth_gbps")) -> argparse.Namespace:
    prelim, _ = parser.parse_known_args(argv)
    if prelim.config:
        payload = json.loads(Path(prelim.config).read_text())
        overrides: Dict[str, object] = dict(payload.get("defaults", {}) or {})
        matrix = payload.get("matrix", {}) or {}
        for key in matrix_keys:
            if key in matrix:
                overrides[key] = matrix[key]
        known = {a.dest for a in parser._actions}
        parser.set_defaults(**{k: v for k, v in overrides.items() if k in known})
    return parser.parse_args(argv)


def make_case(args: argparse.Namespace, *, stage: int, batch_size: int, bandwidth_gbps: float, steps: int,
              metrics_warmup_steps: int, bandwidth_mode: str, extra_args: str,
              nproc_per_node: Optional[int] = None) -> harness.CaseConfig:
    """A ``CaseConfig`` whose unspecified fields come from ``args`` (bandwidth fields default to off)."""
    return harness.CaseConfig(
        stage=int(stage), model_size=str(args.model_size), bandwidth_gbps=float(bandwidth_gbps),
        nproc_per_node=int(nproc_per_node if nproc_per_node is not None else args.nproc_per_node),
        steps=int(steps), seq_len=int(args.seq_len), batch_size=int(batch_size),
        grad_accum_steps=int(args.grad_accum_steps), collective_impl=str(args.collective_impl),
        data_mode=str(args.data_mode), seed=int(args.seed), dtype=str(args.dtype),
        max_grad_norm=float(args.max_grad_norm), stage2_grad_bucket_mb=float(args.stage2_grad_bucket_mb),
        profile_memory_interval=int(args.profile_memory_interval), metrics_warmup_steps=int(metrics_warmup_steps),
        bandwidth_mode=str(bandwidth_mode), sim_latency_ms=float(getattr(args, "sim_latency_ms", 0.0)),
        tc_interface=str(getattr(args, "tc_interface", "eth0")),
        socket_interface=str(getattr(args, "socket_interface", "lo")),
        socket_shaper_burst_bytes=int(getattr(args, "socket_shaper_burst_bytes", 262_144)),
        theory_vocab_size=int(args.theory_vocab_size), extra_args=str(extra_args))


def write_json(path: Path, payload: Dict[str, object]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(payload, indent=2) + "\n")
