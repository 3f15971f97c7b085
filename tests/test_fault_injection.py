"""Failure detection with host-made faults (gloo ranks on CPU; no GPU is faulted, trapped or hung).

A rank that exits, raises or stops joining between steps must end the job promptly with a non-zero
exit code (the survivors' next collective fails: closed connection or the short process-group
timeout), and the experiment harness must record that exit code for the case.
"""

from __future__ import annotations

import os
import subprocess
import sys
import time
from pathlib import Path

import pytest

from cs244c_llama_zero_b200.experiments import harness
from cs244c_llama_zero_b200.train.faults import FaultInjected, FaultInjector, parse_faults

from .dist_utils import find_free_port

ROOT = Path(__file__).resolve().parents[1]


def _train_zero(fault: str, stage: int = 2, extra=()) -> subprocess.CompletedProcess:
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(find_free_port()), str(ROOT / "train_zero.py"), "--zero-stage", str(stage),
           "--model-size", "tiny", "--dim", "32", "--n-layers", "1", "--n-heads", "2", "--n-kv-heads", "1",
           "--ffn-dim", "64", "--seq-len", "16", "--batch-size", "2", "--max-steps", "6", "--log-interval", "1",
           "--checkpoint-interval", "0", "--data-mode", "synthetic", "--synthetic-vocab-size", "97",
           "--collective-impl", "torch", "--pg-timeout-s", "10", *extra]
    env = dict(os.environ, ZB_FAULT=fault, ZB_FAULT_STALL_S="120", CUDA_VISIBLE_DEVICES="")
    return subprocess.run(cmd, capture_output=True, text=True, timeout=240, env=env, cwd=ROOT)


def test_parse_and_local_injection():
    assert [(f.kind, f.rank, f.step) for f in parse_faults("kill_rank:1@3, raise_rank:0@2")] == [
        ("kill_rank", 1, 3), ("raise_rank", 0, 2)]
    with pytest.raises(ValueError):
        parse_faults("explode:1@2")
    inj = FaultInjector(0, "raise_rank:0@2,kill_rank:1@1")
    inj.at_step(1)  # the kill directive is for rank 1
    with pytest.raises(FaultInjected):
        inj.at_step(2)
    assert not FaultInjector(3, "raise_rank:0@2")


@pytest.mark.parametrize("fault", ["kill_rank:1@3", "raise_rank:1@3", "stall_rank:1@3"])
def test_rank_failure_ends_job_with_error(fault):
    t0 = time.perf_counter()
    done = _train_zero(fault)
    elapsed = time.perf_counter() - t0
    assert done.returncode != 0, done.stdout[-2000:]
    assert "[step 00002]" in done.stdout  # steps before the fault completed
    assert "[step 00006]" not in done.stdout
    assert f"injecting {fault.split(':')[0]} at step 3" in done.stderr
    assert elapsed < 200


def test_harness_records_failed_case(tmp_path, monkeypatch):
    args = harness.parse_args(["--results-dir", str(tmp_path), "--name", "f", "--stages", "2", "--bandwidth-mode",
                               "none", "--master-port-base", str(find_free_port()),
                               "--steps", "5", "--seq-len", "16", "--batch-size", "2", "--extra-args",
                               "--dim 32 --n-layers 1 --n-heads 2 --n-kv-heads 1 --ffn-dim 64 --pg-timeout-s 10"])
    case = harness._build_cases(args)[0]
    monkeypatch.setenv("ZB_FAULT", "kill_rank:1@2")
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "")
    launch = harness._launch_config_from_args(args)
    result = harness._run_case(case, tmp_path / "run", False, False, launch, 0)
    assert result.return_code != 0 and result.logged_steps >= 1


def test_skip_signal_directive_arms_the_nvlink_collectives(monkeypatch):
    import torch

    from cs244c_llama_zero_b200.parallel.comm import nvlink

    assert [(f.kind, f.rank, f.step) for f in parse_faults("skip_signal:1@4")] == [("skip_signal", 1, 4)]
    monkeypatch.setattr(nvlink, "_world", lambda: 2)
    coll = nvlink.NvlinkCollectives(device=torch.device("cpu"))
    launched = []

    class Ctx:
        def __getattr__(self, name):
            return lambda *a: launched.append(name)

    class Buf:
        ctx = Ctx()

    monkeypatch.setattr(coll, "_locate", lambda t: (Buf(), 0))
    inj = FaultInjector(rank=1, spec="skip_signal:1@4")
    inj.at_step(3, coll)
    assert coll._skip == 0
    inj.at_step(4, coll)
    flat = torch.ones(16)
    assert coll.allreduce_scaled_(flat, 0.5) is flat and launched == []  # left out: no kernel, data untouched
    assert torch.equal(flat, torch.ones(16))
    coll.allreduce_scaled_(flat, 0.5)
    assert launched == ["allreduce_f32"]
    with pytest.raises(ValueError, match="nvls"):
        FaultInjector(rank=0, spec="skip_signal:0@1").at_step(1, object())


def test_device_error_record_maps_to_exceptions():
    from cs244c_llama_zero_b200 import ops
    from cs244c_llama_zero_b200.parallel.comm.nvlink import CommTimeoutError

    ops.raise_for_device_errors([0, 0, 0, 0])
    with pytest.raises(CommTimeoutError, match="collective barrier"):
        ops.raise_for_device_errors([4, 1, 7, 48])
    with pytest.raises(ops.DeviceWaitError, match="gemm pipeline wait") as info:
        ops.raise_for_device_errors([1, 2, 3, 1])
    assert not isinstance(info.value, CommTimeoutError)
    with pytest.raises(ops.DeviceWaitError, match="paced link hold"):
        ops.raise_for_device_errors([5, 0, 0, 1])


def test_async_loss_raises_on_a_recorded_expiry():
    import torch

    from cs244c_llama_zero_b200.ops import DeviceWaitError
    from cs244c_llama_zero_b200.train.session import AsyncLoss

    ok = AsyncLoss(torch.tensor([1.5]), None, torch.zeros(4, dtype=torch.int32))
    assert ok.item() == 1.5 and ok.nbytes == 20
    bad = AsyncLoss(torch.tensor([1.5]), None, torch.tensor([3, 0, 0, 1], dtype=torch.int32))
    with pytest.raises(DeviceWaitError):
        bad.item()
