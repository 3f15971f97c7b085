"""Experiment harness: case matrix, record formats, log/profile parsing, env, timeouts (subprocess mocked)."""

from __future__ import annotations

import json
import subprocess
from pathlib import Path

import pytest

from cs244c_llama_zero_b200.experiments import harness


def _args(tmp_path: Path, *extra: str):
    return harness.parse_args(["--results-dir", str(tmp_path), "--name", "t", *extra])


def test_case_matrix_is_cartesian_product(tmp_path):
    args = _args(tmp_path, "--stages", "0", "3", "--model-sizes", "tiny", "small", "--bandwidth-gbps", "0", "1.5")
    cases = harness._build_cases(args)
    assert len(cases) == 8
    assert {(c.stage, c.model_size, c.bandwidth_gbps) for c in cases} == {
        (s, m, b) for s in (0, 3) for m in ("tiny", "small") for b in (0.0, 1.5)}


def test_case_id_format(tmp_path):
    case = harness._build_cases(_args(tmp_path, "--stages", "2", "--bandwidth-gbps", "2.5"))[0]
    assert harness._case_id(case) == "s2_mtiny_bw2.5gbps_np2_sl128_bs4_ga1_seed1337"
    case.bandwidth_gbps = 0.0
    assert "_bwunlimited_" in harness._case_id(case)


def test_config_file_supplies_defaults_and_cli_wins(tmp_path):
    cfg = tmp_path / "cfg.json"
    cfg.write_text(json.dumps({"defaults": {"seq_len": 256, "batch_size": 8},
                               "matrix": {"stages": [1], "model_sizes": ["small"], "bandwidth_gbps": [0, 10]}}))
    args = harness.parse_args(["--config", str(cfg), "--batch-size", "2"])
    assert args.seq_len == 256 and args.batch_size == 2
    assert args.stages == [1] and args.model_sizes == ["small"] and args.bandwidth_gbps == [0, 10]
    merged = harness._merge_config_file(harness.parse_args(["--config", str(cfg), "--batch-size", "2"]))
    assert merged.batch_size == 8


def test_step_metrics_parsing_with_warmup_skip():
    log = "\n".join([
        "[step 00001] loss=9.0000 avg100=9.0 tokens/s=1,000 grad_norm=1.0 fb_ms=10.0 comm_ms=5.0 opt_ms=1.0 tflops=0.5",
        "noise",
        "[step 00002] loss=8.0000 avg100=8.5 tokens/s=3,000 grad_norm=nan fb_ms=20.0 comm_ms=7.0 opt_ms=3.0",
    ])
    m = harness._parse_step_metrics(log)
    assert m["logged_steps"] == 2 and m["final_loss"] == 8.0
    assert m["mean_tokens_per_s"] == 2000.0 and m["mean_tflops_per_s"] == 0.5
    w = harness._parse_step_metrics(log, metrics_warmup_steps=1)
    assert w["mean_tokens_per_s"] == 3000.0 and w["mean_comm_ms"] == 7.0 and w["mean_tflops_per_s"] is None


def test_profile_memory_prefers_measured_step(tmp_path):
    path = tmp_path / "p.json"
    path.write_text(json.dumps({
        "memory": [{"host_maxrss_mb": 5.0, "cuda_allocated_mb": 10.0, "cuda_reserved_mb": 20.0,
                    "cuda_max_allocated_mb": 30.0, "cuda_max_reserved_mb": 40.0}],
        "measured_step_memory": {"peak_allocated_mb": 12.0, "peak_reserved_mb": 22.0},
        "state_memory_breakdown_mb": {"params_mb": 1, "grads_mb": 2, "optimizer_mb": 3, "total_mb": 6},
    }))
    m = harness._parse_profile_memory(path)
    assert m["peak_cuda_allocated_mb"] == 12.0 and m["peak_cuda_max_reserved_mb"] == 22.0
    assert m["peak_host_rss_mb"] == 5.0 and m["measured_state_memory_mb"]["total_mb"] == 6.0
    assert harness._parse_profile_memory(tmp_path / "missing.json")["peak_cuda_allocated_mb"] is None


def test_theoretical_memory_shrinks_with_stage(tmp_path):
    cases = harness._build_cases(_args(tmp_path, "--nproc-per-node", "4"))
    totals = [harness._theoretical_memory(c)[1]["total_mb"] for c in cases]
    assert totals[0] > totals[1] > totals[2] > totals[3]


def test_command_and_env(tmp_path):
    args = _args(tmp_path, "--stages", "2", "--bandwidth-gbps", "1", "--bandwidth-mode", "simulated",
                 "--extra-args", "--tflops-mode off")
    case = harness._build_cases(args)[0]
    cmd = harness._build_train_zero_cmd(case, tmp_path / "p.json", harness._launch_config_from_args(args), 3)
    assert cmd[cmd.index("--master_port") + 1] == str(29500 + 3)
    assert cmd[cmd.index("--zero-stage") + 1] == "2" and cmd[-2:] == ["--tflops-mode", "off"]
    env = harness._build_launch_env(case)
    assert env["ZERO_SIM_BW_GBPS"] == "1.0" and env["ZERO_COLLECTIVE_CUDA_SYNC"] == "1"
    case.bandwidth_mode = "socket"
    env = harness._build_launch_env(case, Path("/x/shaper.so"), "shared")
    assert env["LD_PRELOAD"].startswith("/x/shaper.so") and env["NCCL_P2P_DISABLE"] == "1"
    assert env["ZERO_SOCKET_SHAPER_SHARED_NAME"] == "shared" and "ZERO_SIM_BW_GBPS" not in env
    assert harness._verify_socket_transport_log("... via NET/Socket/0 ...")
    assert not harness._verify_socket_transport_log("via P2P/IPC")


def test_timeout_returns_124_and_profile_metrics(tmp_path, monkeypatch):
    args = _args(tmp_path, "--stages", "0", "--bandwidth-mode", "none")
    case = harness._build_cases(args)[0]

    def fake_timeout(*a, **k):
        raise subprocess.TimeoutExpired(cmd="x", timeout=1, output="[step 00001] loss=1.0 avg100=1.0 tokens/s=10 "
                                        "grad_norm=0.1 fb_ms=1 comm_ms=1 opt_ms=1")

    monkeypatch.setattr(harness.subprocess, "run", fake_timeout)
    res = harness._run_case(case, tmp_path / "run", False, False, harness._launch_config_from_args(args), 0)
    assert res.return_code == 124 and res.notes.startswith("timeout_after_s") and res.logged_steps == 1

    def fake_ok(cmd, **k):
        prof = Path(cmd[cmd.index("--profile-json") + 1])
        prof.write_text(json.dumps({"memory": [], "measured_step_memory": {"peak_allocated_mb": 7.0,
                                                                           "peak_reserved_mb": 8.0}}))
        return subprocess.CompletedProcess(cmd, 0, stdout="[step 00001] loss=2.0 avg100=2.0 tokens/s=5 grad_norm=1 "
                                                          "fb_ms=1 comm_ms=2 opt_ms=3\n", stderr="")

    monkeypatch.setattr(harness.subprocess, "run", fake_ok)
    args.name = "t2"
    res = harness._run_case(case, tmp_path / "run2", False, False, harness._launch_config_from_args(args), 0)
    assert res.return_code == 0 and res.peak_cuda_allocated_mb == 7.0 and res.mean_comm_ms == 2.0
    again = harness._run_case(case, tmp_path / "run2", True, False, harness._launch_config_from_args(args), 0)
    assert again == res


def test_dry_run_writes_summary(tmp_path):
    args = _args(tmp_path, "--dry-run", "--stages", "0", "1")
    summary = harness.run_matrix(args)
    assert summary["num_cases"] == 2 and summary["num_failures"] == 0
    data = json.loads((tmp_path / "t" / "summary.json").read_text())
    assert {"name", "args", "theoretical_memory_note", "profiled_tflops_note", "num_cases", "num_failures",
            "results"} <= set(data)
    assert data["results"][0]["notes"] == "dry_run"


@pytest.mark.parametrize("bw,expect", [(0.0, None), (2.0, "2.0")])
def test_simulated_env_only_when_limited(tmp_path, bw, expect):
    case = harness._build_cases(_args(tmp_path, "--bandwidth-gbps", str(bw)))[0]
    assert harness._build_launch_env(case).get("ZERO_SIM_BW_GBPS") == expect


def test_dtype_aware_theoretical_memory_sits_beside_the_fp32_one(tmp_path):
    args = _args(tmp_path, "--stages", "0", "3", "--dtype", "bfloat16", "--nproc-per-node", "4")
    s0, s3 = harness._build_cases(args)
    n, fp32 = harness._theoretical_memory(s0)
    bf = harness._theoretical_memory_dtype(s0, n)
    mb = 1024.0 * 1024.0
    assert bf["params_mb"] == 2 * n / mb and bf["grads_mb"] == 2 * n / mb and bf["optimizer_mb"] == 12 * n / mb
    assert fp32["params_mb"] == 4 * n / mb  # the reference's fp32 definition is kept unchanged
    bf3 = harness._theoretical_memory_dtype(s3, n)
    assert bf3["total_mb"] == bf["total_mb"] / 4
    res = harness._run_case(s0, tmp_path / "run", False, True, harness._launch_config_from_args(args), 0)
    assert res.theoretical_memory_dtype_mb == bf
    legacy = {k: v for k, v in json.loads((tmp_path / "run" / "cases" / f"{res.case_id}.json").read_text()).items()
              if k != "theoretical_memory_dtype_mb"}
    assert harness.CaseResult(**legacy).theoretical_memory_dtype_mb is None  # older records still load
