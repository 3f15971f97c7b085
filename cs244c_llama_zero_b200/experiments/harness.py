"""Experiment harness: run a matrix of ZeRO stages x model sizes x bandwidths through ``train_zero.py``.

Record formats are the reference's (``experiments/harness.py:31-82, 208-213, 697-712``) so runs of either
implementation can be merged, plotted and reported by the same tools:

* ``CaseConfig`` / ``CaseResult`` field names, ``case_id`` = ``s{stage}_m{model}_bw{unlimited|Xgbps}_np{n}_sl{S}_bs{B}_ga{G}_seed{seed}``,
* run directory: ``summary.json``, ``cases/<id>.json``, ``logs/<id>.log``, ``profiles/<id>.json``,
* the step-line regex (``STEP_RE``), warm-up skipping, memory parsing preferring the measured step,
* theoretical state memory (fp32 params/grads + 8 B/param Adam, ideal 1/W sharding per stage),
* exit code 124 on timeout and 125 when socket shaping was requested but NCCL did not use sockets.

A JSON config ``{"defaults": {...}, "matrix": {...}}`` supplies parser defaults; explicit flags win.
Bandwidth modes: ``simulated`` (sleep-based), ``none``, ``tc`` (``infra/throttle.sh``), ``socket``
(``infra/socket_shaper.c`` preloaded, NCCL forced onto sockets).

    python -m cs244c_llama_zero_b200.experiments.harness --config cs244c_llama_zero_b200/experiments/configs/b200_small_stages.json
"""

from __future__ import annotations

import argparse
import itertools
import json
import os
import re
import shlex
import shutil
import subprocess
import sys
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Dict, List, Optional

PROJECT_ROOT = Path(__file__).resolve().parents[2]
SOCKET_SHAPER_SOURCE = PROJECT_ROOT / "infra" / "socket_shaper.c"
SOCKET_SHAPER_SO = PROJECT_ROOT / "infra" / "socket_shaper.so"
if str(PROJECT_ROOT) not in sys.path:
    sys.path.insert(0, str(PROJECT_ROOT))

from cs244c_llama_zero_b200.models import build_config, estimate_num_parameters  # noqa: E402

STEP_RE = re.compile(
    r"\[step\s+(\d+)\]\s+loss=([0-9.eE+\-]+).*?tokens/s=([0-9,]+).*?grad_norm=([0-9.eE+\-a-zA-Z]+)"
    r".*?fb_ms=([0-9.eE+\-]+).*?comm_ms=([0-9.eE+\-]+).*?opt_ms=([0-9.eE+\-]+)(?:.*?tflops=([0-9.eE+\-]+))?"
)

RC_TIMEOUT = 124
RC_SOCKET_VERIFY = 125
COLLECTIVE_IMPLS = ["ring", "torch", "nvls", "p2p"]


@dataclass
class CaseConfig:
    stage: int
    model_size: str
    bandwidth_gbps: float
    nproc_per_node: int
    steps: int
    seq_len: int
    batch_size: int
    grad_accum_steps: int
    collective_impl: str
    data_mode: str
    seed: int
    dtype: str
    max_grad_norm: float
    stage2_grad_bucket_mb: float
    profile_memory_interval: int
    metrics_warmup_steps: int
    bandwidth_mode: str
    sim_latency_ms: float
    tc_interface: str
    socket_interface: str
    socket_shaper_burst_bytes: int
    theory_vocab_size: int
    extra_args: str


@dataclass
class CaseResult:
    case_id: str
    config: Dict[str, object]
    command: str
    return_code: int
    elapsed_s: float
    log_path: str
    profile_path: str
    final_loss: Optional[float]
    logged_steps: int
    mean_tokens_per_s: Optional[float]
    mean_tflops_per_s: Optional[float]
    mean_comm_ms: Optional[float]
    mean_fb_ms: Optional[float]
    mean_opt_ms: Optional[float]
    peak_host_rss_mb: Optional[float]
    peak_cuda_allocated_mb: Optional[float]
    peak_cuda_reserved_mb: Optional[float]
    peak_cuda_max_allocated_mb: Optional[float]
    peak_cuda_max_reserved_mb: Optional[float]
    measured_state_memory_mb: Optional[Dict[str, float]]
    theoretical_param_count: int
    theoretical_memory_mb: Dict[str, float]
    notes: str = ""
    # Extra (not in the reference's record): the same idealised state memory with the run's dtype
    # (bf16 params and grads plus an fp32 master copy next to the Adam moments).
    theoretical_memory_dtype_mb: Optional[Dict[str, float]] = None


@dataclass(frozen=True)
class LaunchConfig:
    nnodes: int
    node_rank: int
    master_addr: str
    master_port_base: int
    case_timeout_s: float


def _build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Experiment harness for ZeRO stages 0-3")
    p.add_argument("--config", type=str, default="")
    p.add_argument("--name", type=str, default="week3_matrix")
    p.add_argument("--results-dir", type=str, default="experiments/results")
    p.add_argument("--skip-existing", action="store_true")
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--stages", nargs="+", type=int, default=[0, 1, 2, 3])
    p.add_argument("--model-sizes", nargs="+", default=["tiny"])
    p.add_argument("--bandwidth-gbps", nargs="+", type=float, default=[0.0])
    p.add_argument("--nproc-per-node", type=int, default=2)
    p.add_argument("--nnodes", type=int, default=1)
    p.add_argument("--node-rank", type=int, default=0)
    p.add_argument("--master-addr", type=str, default="127.0.0.1")
    p.add_argument("--master-port-base", type=int, default=29500)
    p.add_argument("--case-timeout-s", type=float, default=1800.0)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--batch-size", type=int, default=4)
    p.add_argument("--grad-accum-steps", type=int, default=1)
    p.add_argument("--collective-impl", type=str, default="torch", choices=COLLECTIVE_IMPLS)
    p.add_argument("--data-mode", type=str, default="synthetic", choices=["synthetic", "fineweb", "random"])
    p.add_argument("--seed", type=int, default=1337)
    p.add_argument("--dtype", type=str, default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--max-grad-norm", type=float, default=0.0)
    p.add_argument("--stage2-grad-bucket-mb", type=float, default=64.0)
    p.add_argument("--profile-memory-interval", type=int, default=0)
    p.add_argument("--metrics-warmup-steps", type=int, default=0,
                   help="Ignore this many logged training steps when computing mean step metrics.")
    p.add_argument("--bandwidth-mode", type=str, default="simulated",
                   choices=["simulated", "none", "tc", "socket", "nvlink"],
                   help="nvlink: device-paced emulated link for --collective-impl nvls|p2p (Gbit/s)")
    p.add_argument("--sim-latency-ms", type=float, default=0.0)
    p.add_argument("--tc-interface", type=str, default="eth0")
    p.add_argument("--socket-interface", type=str, default="lo")
    p.add_argument("--socket-shaper-burst-bytes", type=int, default=262_144)
    p.add_argument("--theory-vocab-size", type=int, default=0,
                   help="If >0, use this vocab size for theoretical memory; otherwise inferred from data mode.")
    p.add_argument("--extra-args", type=str, default="")
    return p


def _apply_config_to_parser(parser: argparse.ArgumentParser, config_path: str) -> None:
    payload = json.loads(Path(config_path).read_text())
    overrides: Dict[str, object] = dict(payload.get("defaults", {}) or {})
    matrix = payload.get("matrix", {}) or {}
    for key in ("stages", "model_sizes", "bandwidth_gbps"):
        if key in matrix:
            overrides[key] = matrix[key]
    if overrides:
        parser.set_defaults(**overrides)


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    parser = _build_parser()
    prelim, _ = parser.parse_known_args(argv)
    if prelim.config:
        _apply_config_to_parser(parser, prelim.config)
    return parser.parse_args(argv)


def _merge_config_file(args: argparse.Namespace) -> argparse.Namespace:
    """Overwrite ``args`` with a config file's values (config wins; used by programmatic callers)."""
    if not args.config:
        return args
    payload = json.loads(Path(args.config).read_text())
    for key, value in (payload.get("defaults", {}) or {}).items():
        if hasattr(args, key):
            setattr(args, key, value)
    for key in ("stages", "model_sizes", "bandwidth_gbps"):
        if key in (payload.get("matrix", {}) or {}):
            setattr(args, key, payload["matrix"][key])
    return args


def _case_id(case: CaseConfig) -> str:
    bw = "unlimited" if case.bandwidth_gbps <= 0 else f"{case.bandwidth_gbps:g}gbps"
    return (f"s{case.stage}_m{case.model_size}_bw{bw}_np{case.nproc_per_node}_sl{case.seq_len}_bs{case.batch_size}"
            f"_ga{case.grad_accum_steps}_seed{case.seed}")


def _launch_config_from_args(args: argparse.Namespace) -> LaunchConfig:
    return LaunchConfig(int(args.nnodes), int(args.node_rank), str(args.master_addr), int(args.master_port_base),
                        float(args.case_timeout_s))


def _build_cases(args: argparse.Namespace) -> List[CaseConfig]:
    shared = dict(
        nproc_per_node=int(args.nproc_per_node), steps=int(args.steps), seq_len=int(args.seq_len),
        batch_size=int(args.batch_size), grad_accum_steps=int(args.grad_accum_steps),
        collective_impl=str(args.collective_impl), data_mode=str(args.data_mode), seed=int(args.seed),
        dtype=str(args.dtype), max_grad_norm=float(args.max_grad_norm),
        stage2_grad_bucket_mb=float(args.stage2_grad_bucket_mb),
        profile_memory_interval=int(args.profile_memory_interval),
        metrics_warmup_steps=int(args.metrics_warmup_steps), bandwidth_mode=str(args.bandwidth_mode),
        sim_latency_ms=float(args.sim_latency_ms), tc_interface=str(args.tc_interface),
        socket_interface=str(args.socket_interface), socket_shaper_burst_bytes=int(args.socket_shaper_burst_bytes),
        theory_vocab_size=int(args.theory_vocab_size), extra_args=str(args.extra_args),
    )
    return [CaseConfig(stage=int(s), model_size=str(m), bandwidth_gbps=float(bw), **shared)
            for s, m, bw in itertools.product(args.stages, args.model_sizes, args.bandwidth_gbps)]


def _theory_vocab(case: CaseConfig) -> int:
    if case.theory_vocab_size > 0:
        return case.theory_vocab_size
    if case.model_size.startswith("baseline-"):
        return 32_000
    return 8_192 if case.data_mode in ("synthetic", "random") else 128_256


def _theoretical_memory(case: CaseConfig) -> tuple:
    """Idealised ZeRO state memory with fp32 params and grads (4 + 4 B) and Adam moments (8 B)."""
    cfg = build_config(case.model_size, vocab_size=_theory_vocab(case), max_seq_len=case.seq_len)
    n = estimate_num_parameters(cfg)
    w = max(1, case.nproc_per_node)
    shard = {0: (1, 1, 1), 1: (1, 1, w), 2: (1, w, w), 3: (w, w, w)}
    if case.stage not in shard:
        raise ValueError(f"Unsupported stage: {case.stage}")
    dp, dg, do = shard[case.stage]
    mb = 1024.0 * 1024.0
    params, grads, opt = 4.0 * n / dp / mb, 4.0 * n / dg / mb, 8.0 * n / do / mb
    return n, {"params_mb": params, "grads_mb": grads, "optimizer_mb": opt, "total_mb": params + grads + opt}


def _theoretical_memory_dtype(case: CaseConfig, n_params: int) -> Dict[str, float]:
    """State memory with the run's dtype: params and grads at its element size, Adam moments fp32 (8 B)
    plus an fp32 master copy (4 B) when the params are not fp32; ideal 1/W sharding per stage."""
    elem = {"float32": 4, "bfloat16": 2, "float16": 2}.get(case.dtype, 4)
    w = max(1, case.nproc_per_node)
    dp, dg, do = {0: (1, 1, 1), 1: (1, 1, w), 2: (1, w, w), 3: (w, w, w)}[case.stage]
    mb = 1024.0 * 1024.0
    opt_bytes = 8.0 + (4.0 if elem != 4 else 0.0)
    params, grads, opt = elem * n_params / dp / mb, elem * n_params / dg / mb, opt_bytes * n_params / do / mb
    return {"params_mb": params, "grads_mb": grads, "optimizer_mb": opt, "total_mb": params + grads + opt}


def _parse_step_metrics(log_text: str, metrics_warmup_steps: int = 0) -> Dict[str, object]:
    losses: List[float] = []
    rows: List[Dict[str, Optional[float]]] = []
    for line in log_text.splitlines():
        m = STEP_RE.search(line)
        if not m:
            continue
        losses.append(float(m.group(2)))
        rows.append({"tokens_per_s": float(m.group(3).replace(",", "")),
                     "tflops_per_s": None if m.group(8) is None else float(m.group(8)),
                     "fb_ms": float(m.group(5)), "comm_ms": float(m.group(6)), "opt_ms": float(m.group(7))})
    if metrics_warmup_steps > 0:
        rows = rows[metrics_warmup_steps:]

    def mean(key: str) -> Optional[float]:
        vals = [float(r[key]) for r in rows if r[key] is not None]
        return sum(vals) / len(vals) if vals else None

    return {"final_loss": losses[-1] if losses else None, "logged_steps": len(losses),
            "mean_tokens_per_s": mean("tokens_per_s"), "mean_tflops_per_s": mean("tflops_per_s"),
            "mean_comm_ms": mean("comm_ms"), "mean_fb_ms": mean("fb_ms"), "mean_opt_ms": mean("opt_ms")}


_MEMORY_KEYS = ("peak_host_rss_mb", "peak_cuda_allocated_mb", "peak_cuda_reserved_mb", "peak_cuda_max_allocated_mb",
                "peak_cuda_max_reserved_mb")


def _parse_profile_memory(profile_path: Path) -> Dict[str, object]:
    """Peak memory of a run; the measured step's peaks take precedence over snapshot maxima."""
    out: Dict[str, object] = {key: None for key in _MEMORY_KEYS}
    out["measured_state_memory_mb"] = None
    if not profile_path.exists():
        return out
    payload = json.loads(profile_path.read_text())
    state = payload.get("state_memory_breakdown_mb")
    if isinstance(state, dict):
        out["measured_state_memory_mb"] = {str(k): float(v) for k, v in state.items()}
    measured = payload.get("measured_step_memory") if isinstance(payload.get("measured_step_memory"), dict) else {}
    m_alloc = measured.get("peak_allocated_mb")
    m_res = measured.get("peak_reserved_mb")
    m_alloc = None if m_alloc is None else float(m_alloc)
    m_res = None if m_res is None else float(m_res)
    snapshots = payload.get("memory", []) or []

    def peak(key: str) -> Optional[float]:
        vals = [float(s[key]) for s in snapshots if key in s]
        return max(vals) if vals else None

    def prefer(measured_value: Optional[float], key: str) -> Optional[float]:
        return measured_value if measured_value is not None else peak(key)

    out.update({
        "peak_host_rss_mb": peak("host_maxrss_mb") if snapshots else None,
        "peak_cuda_allocated_mb": prefer(m_alloc, "cuda_allocated_mb"),
        "peak_cuda_reserved_mb": prefer(m_res, "cuda_reserved_mb"),
        "peak_cuda_max_allocated_mb": prefer(m_alloc, "cuda_max_allocated_mb"),
        "peak_cuda_max_reserved_mb": prefer(m_res, "cuda_max_reserved_mb"),
    })
    return out


def _apply_tc(case: CaseConfig) -> None:
    subprocess.run([str(PROJECT_ROOT / "infra" / "throttle.sh"), "apply", case.tc_interface,
                    f"{case.bandwidth_gbps:g}gbit", "1mb", "10ms"], check=True, cwd=PROJECT_ROOT)


def _clear_tc(case: CaseConfig) -> None:
    subprocess.run([str(PROJECT_ROOT / "infra" / "throttle.sh"), "delete", case.tc_interface], check=False,
                   cwd=PROJECT_ROOT)


def _master_port_for_case(launch: LaunchConfig, case_index: int) -> int:
    return launch.master_port_base + case_index


def _ensure_socket_shaper_built() -> Path:
    if sys.platform != "linux":
        raise RuntimeError("bandwidth-mode=socket is only supported on Linux")
    from infra.build_socket_shaper import build_socket_shaper

    return build_socket_shaper(SOCKET_SHAPER_SOURCE, SOCKET_SHAPER_SO)


def _build_launch_env(case: CaseConfig, socket_shaper_path: Optional[Path] = None,
                      socket_shaper_shared_name: Optional[str] = None) -> Dict[str, str]:
    env = os.environ.copy()
    env["PYTHONUNBUFFERED"] = "1"
    env["ZERO_COLLECTIVE_CUDA_SYNC"] = "1"
    for key in ("ZERO_SIM_BW_GBPS", "ZERO_SIM_LATENCY_MS", "ZERO_SOCKET_SHAPER_BW_GBPS", "ZERO_SOCKET_SHAPER_LATENCY_MS",
                "ZERO_SOCKET_SHAPER_BURST_BYTES", "ZERO_SOCKET_SHAPER_SHARED_NAME", "ZERO_NVLINK_BW_GBPS",
                "ZERO_NVLINK_LATENCY_MS"):
        env.pop(key, None)
    if case.bandwidth_mode == "simulated":
        if case.bandwidth_gbps > 0:
            env["ZERO_SIM_BW_GBPS"] = str(case.bandwidth_gbps)
        if case.sim_latency_ms > 0:
            env["ZERO_SIM_LATENCY_MS"] = str(case.sim_latency_ms)
    if case.bandwidth_mode == "nvlink":
        # Paced on the device by the NVLink collective runtime (parallel/comm/pacing.py).
        if case.bandwidth_gbps > 0:
            env["ZERO_NVLINK_BW_GBPS"] = str(case.bandwidth_gbps)
        if case.sim_latency_ms > 0:
            env["ZERO_NVLINK_LATENCY_MS"] = str(case.sim_latency_ms)
    if case.bandwidth_mode == "socket":
        if socket_shaper_path is None:
            raise ValueError("socket shaper path is required for bandwidth-mode=socket")
        env["ZERO_SOCKET_SHAPER_BW_GBPS"] = str(case.bandwidth_gbps)
        if case.sim_latency_ms > 0:
            env["ZERO_SOCKET_SHAPER_LATENCY_MS"] = str(case.sim_latency_ms)
        env["ZERO_SOCKET_SHAPER_BURST_BYTES"] = str(case.socket_shaper_burst_bytes)
        if socket_shaper_shared_name:
            env["ZERO_SOCKET_SHAPER_SHARED_NAME"] = socket_shaper_shared_name
        env.update({"NCCL_P2P_DISABLE": "1", "NCCL_SHM_DISABLE": "1", "NCCL_IB_DISABLE": "1",
                    "NCCL_SOCKET_IFNAME": case.socket_interface, "GLOO_SOCKET_IFNAME": case.socket_interface,
                    "NCCL_DEBUG": "INFO", "NCCL_DEBUG_SUBSYS": "INIT,NET"})
        preload = [str(socket_shaper_path)] + ([env["LD_PRELOAD"].strip()] if env.get("LD_PRELOAD", "").strip() else [])
        env["LD_PRELOAD"] = ":".join(preload)
    return env


def _verify_socket_transport_log(log_text: str) -> bool:
    return ("Using network Socket" in log_text) or ("via NET/Socket/" in log_text)


def _build_train_zero_cmd(case: CaseConfig, profile_path: Path, launch: LaunchConfig, case_index: int) -> List[str]:
    cmd = [
        sys.executable, "-m", "torch.distributed.run",
        "--nnodes", str(launch.nnodes), "--node_rank", str(launch.node_rank),
        "--nproc_per_node", str(case.nproc_per_node), "--master_addr", launch.master_addr,
        "--master_port", str(_master_port_for_case(launch, case_index)),
        str(PROJECT_ROOT / "train_zero.py"),
        "--zero-stage", str(case.stage), "--collective-impl", case.collective_impl, "--data-mode", case.data_mode,
        "--model-size", case.model_size, "--seq-len", str(case.seq_len), "--batch-size", str(case.batch_size),
        "--grad-accum-steps", str(case.grad_accum_steps), "--max-steps", str(case.steps), "--seed", str(case.seed),
        "--dtype", case.dtype, "--max-grad-norm", str(case.max_grad_norm),
        "--stage2-grad-bucket-mb", str(case.stage2_grad_bucket_mb), "--log-interval", "1",
        "--checkpoint-interval", "0", "--profile-json", str(profile_path), "--profile-rank0-only",
    ]
    if _theory_vocab(case) != 8_192 and case.data_mode in ("synthetic", "random"):
        cmd.extend(["--synthetic-vocab-size", str(_theory_vocab(case))])
    if case.profile_memory_interval > 0:
        cmd.extend(["--profile-memory-interval", str(case.profile_memory_interval)])
    if case.extra_args.strip():
        cmd.extend(shlex.split(case.extra_args))
    return cmd


def _combine_process_output(stdout, stderr) -> str:
    def text(v) -> str:
        if v is None:
            return ""
        return v.decode("utf-8", errors="replace") if isinstance(v, bytes) else v

    return text(stdout) + "\n" + text(stderr)


def _empty_metrics() -> Dict[str, object]:
    return {"final_loss": None, "logged_steps": 0, "mean_tokens_per_s": None, "mean_tflops_per_s": None,
            "mean_comm_ms": None, "mean_fb_ms": None, "mean_opt_ms": None}


def _run_case(case: CaseConfig, run_dir: Path, skip_existing: bool, dry_run: bool, launch: LaunchConfig,
              case_index: int) -> CaseResult:
    case_id = _case_id(case)
    (run_dir / "cases").mkdir(parents=True, exist_ok=True)
    result_path = run_dir / "cases" / f"{case_id}.json"
    if skip_existing and result_path.exists():
        return CaseResult(**json.loads(result_path.read_text()))
    for sub in ("logs", "profiles"):
        (run_dir / sub).mkdir(parents=True, exist_ok=True)
    log_path = run_dir / "logs" / f"{case_id}.log"
    profile_path = run_dir / "profiles" / f"{case_id}.json"
    cmd = _build_train_zero_cmd(case, profile_path, launch, case_index)
    shaper = _ensure_socket_shaper_built() if case.bandwidth_mode == "socket" and not dry_run else None
    env = _build_launch_env(case, shaper, f"zero_socket_{os.getpid()}_{case_index}" if shaper else None) \
        if not (dry_run and case.bandwidth_mode == "socket") else dict(os.environ)
    command = " ".join(shlex.quote(x) for x in cmd)
    n_params, theory = _theoretical_memory(case)

    def finish(rc: int, elapsed: float, metrics: Dict[str, object], mem: Dict[str, object], notes: str) -> CaseResult:
        result = CaseResult(case_id=case_id, config=asdict(case), command=command, return_code=rc, elapsed_s=elapsed,
                            log_path=str(log_path), profile_path=str(profile_path), **metrics, **mem,
                            theoretical_param_count=n_params, theoretical_memory_mb=theory, notes=notes,
                            theoretical_memory_dtype_mb=_theoretical_memory_dtype(case, n_params))
        result_path.write_text(json.dumps(asdict(result), indent=2))
        return result

    if dry_run:
        mem = {key: None for key in _MEMORY_KEYS}
        mem["measured_state_memory_mb"] = None
        return finish(0, 0.0, _empty_metrics(), mem, "dry_run")
    use_tc = case.bandwidth_mode == "tc" and case.bandwidth_gbps > 0
    if use_tc:
        _apply_tc(case)
    t0 = time.perf_counter()
    notes = ""
    try:
        done = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=PROJECT_ROOT,
                              timeout=launch.case_timeout_s if launch.case_timeout_s > 0 else None)
        log_text = _combine_process_output(done.stdout, done.stderr)
        rc = done.returncode
    except subprocess.TimeoutExpired as exc:
        log_text = _combine_process_output(exc.stdout, exc.stderr) + \
            f"\n[harness] timeout after {launch.case_timeout_s:.1f}s\n"
        rc = RC_TIMEOUT
        notes = f"timeout_after_s={launch.case_timeout_s:.1f}"
    finally:
        if use_tc:
            _clear_tc(case)
    elapsed = time.perf_counter() - t0
    if rc == 0 and case.bandwidth_mode == "socket" and not _verify_socket_transport_log(log_text):
        rc = RC_SOCKET_VERIFY
        notes = "socket_transport_verification_failed"
        log_text += "\n[harness] expected NCCL NET/Socket transport markers were missing from the log\n"
    log_path.write_text(log_text)
    return finish(rc, elapsed, _parse_step_metrics(log_text, case.metrics_warmup_steps),
                  _parse_profile_memory(profile_path), notes)


def _build_summary(results: List[CaseResult], args: argparse.Namespace) -> Dict[str, object]:
    return {
        "name": args.name,
        "args": vars(args),
        "theoretical_memory_note": (
            "Memory estimates are idealized ZeRO state-memory terms (params, grads, optimizer states), fp32-based, "
            "and do not include activations, temporary buffers, or framework overhead."),
        "profiled_tflops_note": (
            "Training TFLOPs/s is derived from the train_zero TFLOPs mode: estimated cluster step FLOPs by default, "
            "or torch.profiler-derived FLOPs when profile mode is explicitly enabled."),
        "num_cases": len(results),
        "num_failures": sum(1 for r in results if r.return_code != 0),
        "results": [asdict(r) for r in results],
    }


def run_matrix(args: argparse.Namespace) -> Dict[str, object]:
    launch = _launch_config_from_args(args)
    if args.bandwidth_mode == "tc" and shutil.which("tc") is None:
        raise FileNotFoundError("bandwidth mode 'tc' requires the 'tc' command to be installed")
    if args.bandwidth_mode == "nvlink" and args.collective_impl not in ("nvls", "p2p"):
        raise ValueError("bandwidth mode 'nvlink' paces the NVLink collective kernels: use --collective-impl nvls or p2p")
    run_dir = Path(args.results_dir) / args.name
    run_dir.mkdir(parents=True, exist_ok=True)
    cases = _build_cases(args)
    print(f"[harness] prepared {len(cases)} cases")
    results: List[CaseResult] = []
    for idx, case in enumerate(cases, start=1):
        print(f"[harness] ({idx}/{len(cases)}) {_case_id(case)}")
        result = _run_case(case, run_dir, args.skip_existing, args.dry_run, launch, idx - 1)
        results.append(result)
        if result.return_code != 0:
            print(f"[harness] case failed: {result.case_id} (see {result.log_path})")
    summary = _build_summary(results, args)
    (run_dir / "summary.json").write_text(json.dumps(summary, indent=2))
    print(f"[harness] wrote {run_dir / 'summary.json'}")
    return summary


def main(argv: Optional[List[str]] = None) -> None:
    run_matrix(parse_args(argv))


if __name__ == "__main__":
    main()
