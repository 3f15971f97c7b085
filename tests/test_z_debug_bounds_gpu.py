"""The debug-bounds build (``_C_debug``, ``-DB200_DEBUG_BOUNDS``): the kernel numerics and canary
tests pass against it, and none of its range checks on hand-indexed global accesses fires (the
module fixture of those tests asserts that the device error record stays clean).

Collected near the end of the suite because it re-runs other test files in a child process."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.gpu
def test_kernel_suite_passes_under_the_debug_bounds_build():
    if not list((ROOT / "cs244c_llama_zero_b200" / "ops").glob("_C_debug*.so")):
        pytest.fail("the debug-bounds extension is not built: ZB_DEBUG_BOUNDS=1 python setup.py build_ext "
                    "--inplace --build-temp build/debug_bounds")
    env = dict(os.environ, ZB_DEBUG_BOUNDS="1")
    cmd = [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "-m", "gpu",
           "tests/test_kernels_gpu.py", "tests/test_race_checks_gpu.py", "-k", "not replay"]
    done = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    assert done.returncode == 0, done.stdout[-4000:] + done.stderr[-2000:]
    assert " passed" in done.stdout


def test_debug_flag_selects_the_debug_module(monkeypatch):
    from cs244c_llama_zero_b200 import ops

    monkeypatch.setenv("ZB_DEBUG_BOUNDS", "1")
    assert ops.extension_module_name() == "_C_debug"
    monkeypatch.setenv("ZB_DEBUG_BOUNDS", "0")
    assert ops.extension_module_name() == "_C"
