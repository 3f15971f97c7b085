#!/usr/bin/env python3
"""Run the reference project's own test suite against this package.

The reference keeps its modules at the top level (``model``, ``zero``, ``collectives``,
``profiler``, ``data``, ``experiments``, ``analysis``); this package namespaces them under
``cs244c_llama_zero_b200``.  The script copies the reference's test files into a temporary
directory (nothing of them is kept in this repository), rewrites their import lines with the module
map below, and runs them with pytest against this package.  A test that passes shows that a user
of the reference gets the same behaviour from the same call here.

Deliberate differences are listed in ``EXPECTED_DIFFERENCES`` with the reason; they are reported,
not counted as failures.

    python scripts/run_reference_tests.py --reference-root <reference checkout> [-- <pytest args>]
"""

from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = "cs244c_llama_zero_b200"

# reference module -> this package's module (longest prefix first)
MODULE_MAP = [
    ("data.fineweb", f"{PKG}.data.datasets"),
    ("model.config", f"{PKG}.models.config"),
    ("model.llama", f"{PKG}.models.llama"),
    ("model", f"{PKG}.models"),
    ("zero.common", f"{PKG}.parallel.zero.common"),
    ("zero", f"{PKG}.parallel.zero"),
    ("collectives", f"{PKG}.parallel.collectives"),
    ("profiler", f"{PKG}.profiler"),
    ("data", f"{PKG}.data"),
    ("experiments", f"{PKG}.experiments"),
    ("analysis", f"{PKG}.analysis"),
]

# test id suffix -> why this package differs on purpose
EXPECTED_DIFFERENCES = {
    "test_stage2_releases_full_grads_and_keeps_shard_world2":
        "stage 2 keeps its fp32 gradient shard allocated between steps (grad_shard is never None)",
    "test_stage2_memory_trace_records_internal_labels_world1":
        "the flat fp32 gradient buffer is a persistent (symmetric) allocation, so it stays live after the step",
    "test_stage2_logical_state_breakdown_keeps_grad_shard_after_step_world1":
        "same: live gradient memory after the step is the persistent buffers, not zero",
}

TEST_DIRS = ("tests", "zero/tests", "collectives/tests")
LINKS = ("infra", "scripts", "train.py", "train_zero.py")  # paths the reference tests reach from their root


def rewrite(source: str) -> str:
    def sub(match: re.Match) -> str:
        kw, mod = match.group(1), match.group(2)
        for ref, ours in MODULE_MAP:
            if mod == ref or mod.startswith(ref + "."):
                return f"{kw} {ours}{mod[len(ref):]}"
        return match.group(0)

    out = re.sub(r"^(from|import)\s+([A-Za-z_][\w.]*)", sub, source, flags=re.M)
    # scripts the tests launch by path live inside the package here
    out = re.sub(r'"experiments/(\w+)\.py"', rf'"-m", "{PKG}.experiments.\1"', out)
    return out


def stage(reference_root: Path, dest: Path) -> list:
    files = []
    for rel in TEST_DIRS:
        src = reference_root / rel
        if not src.is_dir():
            continue
        out_dir = dest / rel.replace("/", "_")
        out_dir.mkdir(parents=True, exist_ok=True)
        for f in sorted(src.glob("*.py")):
            if f.name == "conftest.py":
                continue
            (out_dir / f.name).write_text(rewrite(f.read_text()))
            files.append(out_dir / f.name)
    for name in LINKS:
        link = dest / name
        if not link.exists():
            os.symlink(ROOT / name, link)
    return files


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--reference-root", required=True, type=Path)
    p.add_argument("--keep", action="store_true", help="keep the staged copy and print its path")
    p.add_argument("pytest_args", nargs="*")
    args = p.parse_args(argv)
    tmp = Path(tempfile.mkdtemp(prefix="reftests_"))
    try:
        files = stage(args.reference_root.resolve(), tmp)
        if not files:
            print(f"no reference tests found under {args.reference_root}", file=sys.stderr)
            return 2
        env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT)] + [os.environ.get("PYTHONPATH", "")]))
        cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-rf", *map(str, files),
               *args.pytest_args]
        done = subprocess.run(cmd, cwd=tmp, env=env, capture_output=True, text=True)
        print(done.stdout[-4000:])
        failed = re.findall(r"^FAILED (\S+)", done.stdout, flags=re.M)
        unexpected = [f for f in failed if not any(f.endswith(k) for k in EXPECTED_DIFFERENCES)]
        for f in failed:
            why = next((v for k, v in EXPECTED_DIFFERENCES.items() if f.endswith(k)), None)
            if why:
                print(f"expected difference: {f.split('::')[-1]} - {why}")
        if unexpected:
            print(f"{len(unexpected)} unexpected failure(s)")
            return 1
        if done.returncode not in (0, 1):
            print(done.stderr[-2000:])
            return done.returncode
        print("reference suite: all tests pass apart from the listed deliberate differences")
        return 0
    finally:
        if args.keep:
            print(f"staged in {tmp}")
        else:
            shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    sys.exit(main())
