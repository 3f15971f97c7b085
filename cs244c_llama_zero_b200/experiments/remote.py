"""Run an experiment on a remote GPU host over ssh: ship the repo, run, pull results back, report.

Steps of one remote run (every remote command goes through ``ssh user@host``):

1. bundle the working tree (``git ls-files --cached --others --exclude-standard``, minus result
   directories and built artefacts) into a tar.gz,
2. ``mktemp -d`` a fresh workspace under ``--remote-base-dir`` and ``scp`` the bundle there, unpack,
3. optionally ``pip install -r requirements.txt`` and build the CUDA extension in place,
4. run the experiment module (``python -m cs244c_llama_zero_b200.experiments.<module> --config ... --name ...``),
   streaming its output,
5. tar the remote run directory, ``scp`` it back into ``--local-results-dir/<host>/<name>``,
6. render the plots / reports locally and write ``remote_run_metadata.json``,
7. remove the remote workspace (unless ``--keep-remote-workdir``), also when a step failed.

The four CLIs (``run_remote_bandwidth_sweep``, ``run_remote_fit_memory_bandwidth``,
``run_remote_pairwise_crossover``, ``run_remote_stage3_scaling``) differ only in the module they run
and the reports they render.  Flags follow the reference's ``experiments/run_remote_*.py``.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import shlex
import shutil
import subprocess
import sys
import tarfile
import tempfile
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence

PROJECT_ROOT = Path(__file__).resolve().parents[2]
# git-ignored paths (scratch folders among them) are already left out by --exclude-standard
EXCLUDED_PREFIXES = ("experiments/results/", "build/", "baseline/_ref/")
EXCLUDED_SUFFIXES = (".so", ".o", ".pyc", ".ncu-rep")
PLOT_FILES = {"throughput": "throughput.svg", "comm": "comm.svg", "tflops": "tflops.svg",
              "stage-throughput": "stage_throughput.svg", "stage-comm": "stage_comm.svg", "loss": "loss.svg",
              "memory": "memory.svg", "peak-memory": "peak_memory.svg", "avg-memory": "avg_memory.svg"}

Runner = Callable[..., subprocess.CompletedProcess]


def sanitize(token: str) -> str:
    return re.sub(r"[^A-Za-z0-9._-]+", "_", token).strip("._") or "run"


def add_remote_args(p: argparse.ArgumentParser, *, default_config: str, extra_flag: str,
                    default_plots: Sequence[str]) -> None:
    p.add_argument("--host", type=str, required=True)
    p.add_argument("--user", type=str, default="root")
    p.add_argument("--port", type=int, default=22)
    p.add_argument("--ssh-option", action="append", default=[], help="Repeated raw ssh -o options")
    p.add_argument("--config", type=str, default=default_config)
    p.add_argument("--name-override", type=str, default="")
    p.add_argument(extra_flag, dest="extra_args", type=str, default="",
                   help="Extra arguments appended to the remote experiment command")
    p.add_argument("--remote-base-dir", type=str, default="/workspace/zero-b200-runs")
    p.add_argument("--remote-python", type=str, default="python3")
    p.add_argument("--install-deps", action="store_true")
    p.add_argument("--build-extension", action="store_true",
                   help="Build the sm_100a extension in the remote workspace before running")
    p.add_argument("--keep-remote-workdir", action="store_true")
    p.add_argument("--local-results-dir", type=str, default="experiments/results/remote")
    p.add_argument("--overwrite-local", action="store_true")
    p.add_argument("--skip-plots", action="store_true")
    p.add_argument("--skip-summary", action="store_true")
    p.add_argument("--plots", nargs="+", default=list(default_plots), choices=sorted(PLOT_FILES))
    p.add_argument("--dry-run", action="store_true")


def bundle_paths(root: Path, runner: Runner = subprocess.run) -> List[str]:
    listed = runner(["git", "ls-files", "--cached", "--others", "--exclude-standard", "-z"], cwd=root, check=True,
                    text=True, capture_output=True).stdout
    keep = []
    for rel in (x for x in listed.split("\0") if x):
        if rel.startswith(EXCLUDED_PREFIXES) or rel.endswith(EXCLUDED_SUFFIXES) or "__pycache__/" in rel:
            continue
        keep.append(rel)
    if not keep:
        raise RuntimeError("bundle would be empty")
    return keep


def create_bundle(root: Path, rel_paths: Sequence[str]) -> Path:
    fd, name = tempfile.mkstemp(suffix=".tar.gz")
    os.close(fd)
    with tarfile.open(name, "w:gz", format=tarfile.PAX_FORMAT) as tar:
        for rel in rel_paths:
            if (root / rel).exists():
                tar.add(root / rel, arcname=rel, recursive=False)
    return Path(name)


@dataclass
class RemoteSession:
    host: str
    user: str = "root"
    port: int = 22
    ssh_options: List[str] = field(default_factory=list)
    runner: Runner = subprocess.run
    log: Callable[[str], None] = print

    @property
    def target(self) -> str:
        return f"{self.user}@{self.host}"

    def ssh_cmd(self, remote: str) -> List[str]:
        cmd = ["ssh", "-p", str(self.port)]
        for opt in self.ssh_options:
            cmd += ["-o", opt]
        return cmd + [self.target, remote]

    def scp_cmd(self, src: str, dst: str) -> List[str]:
        cmd = ["scp", "-P", str(self.port)]
        for opt in self.ssh_options:
            cmd += ["-o", opt]
        return cmd + [src, dst]

    def ssh(self, remote: str, *, check: bool = True, stream: bool = False) -> str:
        if stream:
            done = self.runner(self.ssh_cmd(remote), cwd=PROJECT_ROOT, check=False, text=True)
            if check and done.returncode != 0:
                raise RuntimeError(f"remote command failed with exit code {done.returncode}: {remote}")
            return ""
        done = self.runner(self.ssh_cmd(remote), cwd=PROJECT_ROOT, check=check, text=True, capture_output=True)
        return (done.stdout or "").strip()

    def upload(self, local: Path, remote: str) -> None:
        self.runner(self.scp_cmd(str(local), f"{self.target}:{remote}"), cwd=PROJECT_ROOT, check=True)

    def download(self, remote: str, local: Path) -> None:
        self.runner(self.scp_cmd(f"{self.target}:{remote}", str(local)), cwd=PROJECT_ROOT, check=True)

    def make_workspace(self, base_dir: str, name: str) -> str:
        base = base_dir.rstrip("/")
        return self.ssh(f"mkdir -p {shlex.quote(base)} && mktemp -d {shlex.quote(base)}/{shlex.quote(sanitize(name))}.XXXXXX")

    def pull_dir(self, remote_dir: str, local_dir: Path) -> None:
        archive = f"{remote_dir.rstrip('/')}.tar.gz"
        local_dir.mkdir(parents=True, exist_ok=True)
        fd, tmp = tempfile.mkstemp(suffix=".tar.gz")
        os.close(fd)
        try:
            self.ssh(f"tar -C {shlex.quote(remote_dir)} -czf {shlex.quote(archive)} .")
            self.download(archive, Path(tmp))
            shutil.unpack_archive(tmp, str(local_dir), filter="data")
        finally:
            self.ssh(f"rm -f {shlex.quote(archive)}", check=False)
            Path(tmp).unlink(missing_ok=True)


def _config_defaults(config: Path) -> Dict[str, object]:
    data = json.loads(config.read_text())
    defaults = data.get("defaults", {})
    return defaults if isinstance(defaults, dict) else {}


def run_remote(args: argparse.Namespace, *, module: str, tag: str,
               postprocess: Callable[[Path, argparse.Namespace], Optional[Path]],
               session: Optional[RemoteSession] = None) -> Path:
    """Ship, run ``module`` with ``--config``/``--name``, pull back, post-process; returns the local run dir."""
    config = Path(args.config).resolve()
    if not config.exists():
        raise FileNotFoundError(f"missing config: {config}")
    try:
        config_rel = config.relative_to(PROJECT_ROOT.resolve())
    except ValueError as exc:
        raise ValueError(f"config must live under the repo root: {config}") from exc
    defaults = _config_defaults(config)
    name = sanitize(args.name_override or str(defaults.get("name", config.stem)))
    results_dir = str(defaults.get("results_dir", "experiments/results")).rstrip("/")
    local_dir = (PROJECT_ROOT / args.local_results_dir / sanitize(args.host) / name).resolve()
    if local_dir.exists():
        if not args.overwrite_local:
            raise FileExistsError(f"local run dir already exists: {local_dir}")
        shutil.rmtree(local_dir)
    session = session or RemoteSession(args.host, args.user, args.port, list(args.ssh_option))
    bundle = create_bundle(PROJECT_ROOT, bundle_paths(PROJECT_ROOT, session.runner))
    workspace = ""
    t0 = time.time()
    try:
        workspace = session.make_workspace(args.remote_base_dir, name)
        ws = shlex.quote(workspace)
        session.upload(bundle, f"{workspace}/repo_bundle.tar.gz")
        session.ssh(f"tar -xzf {ws}/repo_bundle.tar.gz -C {ws} && rm -f {ws}/repo_bundle.tar.gz", stream=True)
        py = shlex.quote(args.remote_python)
        if args.install_deps:
            session.ssh(f"cd {ws} && {py} -m pip install -r requirements.txt", stream=True)
        if getattr(args, "build_extension", False):
            session.ssh(f"cd {ws} && {py} setup.py build_ext --inplace", stream=True)
        session.ssh(f"cd {ws} && {py} -c \"import torch; print('torch', torch.__version__, 'cuda', "
                    f"torch.cuda.device_count())\"", stream=True)
        cmd = [args.remote_python, "-m", f"cs244c_llama_zero_b200.experiments.{module}", "--config", str(config_rel),
               "--name", name] + shlex.split(args.extra_args or "")
        if args.dry_run:
            cmd.append("--dry-run")
        session.ssh(f"cd {ws} && " + " ".join(shlex.quote(c) for c in cmd), stream=True)
        remote_run_dir = f"{workspace}/{results_dir}/{name}"
        session.pull_dir(remote_run_dir, local_dir)
        report = postprocess(local_dir, args)
        meta = {"host": args.host, "user": args.user, "port": args.port, "config": str(config_rel), "run_name": name,
                "module": module, "remote_workspace": workspace, "remote_run_dir": remote_run_dir,
                "local_run_dir": str(local_dir), "report_path": None if report is None else str(report),
                "elapsed_s": time.time() - t0}
        (local_dir / "remote_run_metadata.json").write_text(json.dumps(meta, indent=2) + "\n")
        session.log(f"[{tag}] local results: {local_dir}")
        return local_dir
    finally:
        bundle.unlink(missing_ok=True)
        if workspace and not args.keep_remote_workdir:
            session.ssh(f"rm -rf {shlex.quote(workspace)}", check=False)


def render_plots(run_dir: Path, plots: Sequence[str], tag: str) -> None:
    from cs244c_llama_zero_b200.analysis import visualize

    summary = run_dir / "summary.json"
    if not summary.exists():
        return
    cases = visualize.parse_summary(summary)
    for plot in plots:
        try:
            visualize.render(cases, plot, run_dir / PLOT_FILES[plot])
        except (RuntimeError, ValueError) as exc:
            print(f"[{tag}] warning: plot {plot} failed: {exc}", file=sys.stderr)


def bandwidth_postprocess(tag: str) -> Callable[[Path, argparse.Namespace], Optional[Path]]:
    def post(run_dir: Path, args: argparse.Namespace) -> Optional[Path]:
        from cs244c_llama_zero_b200.analysis import bandwidth_report

        if not args.skip_plots:
            render_plots(run_dir, args.plots, tag)
        if args.skip_summary or not (run_dir / "summary.json").exists():
            return None
        out = run_dir / "bandwidth_report.md"
        out.write_text(bandwidth_report.generate_report_markdown(run_dir))
        return out
    return post
