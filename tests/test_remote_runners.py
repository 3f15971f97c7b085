"""Remote runners end to end over a loopback "host": ssh runs the command locally, scp copies files.

The remote workspace is a temp directory on this machine, so bundling, unpacking, running the
experiment module (dry run), pulling the run directory back, reporting and cleanup all execute for real.
"""

from __future__ import annotations

import json
import shutil
import subprocess
from pathlib import Path

import pytest

from cs244c_llama_zero_b200.experiments import remote, run_remote_bandwidth_sweep, run_remote_stage3_scaling


class LoopbackRunner:
    def __init__(self):
        self.calls = []

    def __call__(self, cmd, **kw):
        self.calls.append(list(cmd))
        if cmd[0] == "ssh":
            done = subprocess.run(["bash", "-c", cmd[-1]], capture_output=True, text=True)
            if kw.get("check") and done.returncode != 0:
                raise subprocess.CalledProcessError(done.returncode, cmd, done.stdout, done.stderr)
            return done
        if cmd[0] == "scp":
            src, dst = (c.split(":", 1)[1] if c.startswith("root@") else c for c in cmd[-2:])
            shutil.copy(src, dst)
            return subprocess.CompletedProcess(cmd, 0, "", "")
        return subprocess.run(cmd, **{k: v for k, v in kw.items() if k != "check"}, check=kw.get("check", False))


def _session(runner):
    return remote.RemoteSession("loopback", runner=runner, log=lambda s: None)


def test_bundle_excludes_results_and_builds():
    paths = remote.bundle_paths(remote.PROJECT_ROOT)
    assert "bench.py" in paths and "setup.py" in paths
    assert not any(p.endswith(".so") or p.startswith(("build/", "baseline/_ref/")) for p in paths)
    ignored = remote.subprocess.run(["git", "check-ignore", "--stdin"], input="\n".join(paths), text=True,
                                    capture_output=True, cwd=remote.PROJECT_ROOT).stdout.split()
    assert ignored == []  # nothing git ignores (scratch folders, results) goes into the bundle


def test_remote_bandwidth_sweep_dry_run_roundtrip(tmp_path):
    runner = LoopbackRunner()
    base = tmp_path / "remote_base"
    local = tmp_path / "local"
    run_remote_bandwidth_sweep.main(["--host", "loopback", "--remote-base-dir", str(base), "--local-results-dir",
                                     str(local), "--dry-run", "--remote-python", "python"], session=_session(runner))
    run_dir = local / "loopback" / "b200_bandwidth_smoke"
    summary = json.loads((run_dir / "summary.json").read_text())
    assert summary["num_cases"] == 8 and summary["results"][0]["notes"] == "dry_run"
    meta = json.loads((run_dir / "remote_run_metadata.json").read_text())
    assert meta["module"] == "harness" and meta["run_name"] == "b200_bandwidth_smoke"
    assert (run_dir / "bandwidth_report.md").exists()
    assert list(base.iterdir()) == []  # remote workspace removed
    assert any(c[0] == "scp" for c in runner.calls)


def test_remote_refuses_existing_local_dir(tmp_path):
    (tmp_path / "loopback" / "b200_bandwidth_smoke").mkdir(parents=True)
    with pytest.raises(FileExistsError):
        run_remote_bandwidth_sweep.main(["--host", "loopback", "--local-results-dir", str(tmp_path)],
                                        session=_session(LoopbackRunner()))


def test_remote_stage3_postprocess_renders_report(tmp_path):
    run_dir = tmp_path / "run"
    run_dir.mkdir()
    (run_dir / "summary.json").write_text(json.dumps({"args": {"model_size": "m"}, "scaling_points": [
        {"gpu_count": 1, "mean_tflops_per_s": 10.0, "per_gpu_tflops_per_s": 10.0},
        {"gpu_count": 2, "mean_tflops_per_s": 21.0, "per_gpu_tflops_per_s": 10.5}]}))
    args = run_remote_stage3_scaling.parse_args(["--host", "h"])
    report = run_remote_stage3_scaling._post(run_dir, args)
    assert report is not None and "Stage 3 GPU Scaling" in report.read_text()
    assert (run_dir / "stage3_scaling.svg").exists()
