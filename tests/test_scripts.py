"""Operational scripts on CPU: gloo sanity / all-reduce benchmark (2 ranks), loopback shaper check, repo bundle."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _torchrun(script: str, port: int, *args: str) -> str:
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(port), str(ROOT / "scripts" / script), *args]
    return subprocess.run(cmd, check=True, capture_output=True, text=True, timeout=300, cwd=ROOT).stdout


def test_distributed_sanity_gloo():
    assert "all_reduce_sum=3.0" in _torchrun("distributed_sanity.py", 29631)


def test_benchmark_allreduce_gloo():
    line = [ln for ln in _torchrun("benchmark_allreduce.py", 29632, "--numel", "4096", "--iters", "2").splitlines()
            if ln.startswith("{")][-1]
    rec = json.loads(line)
    assert rec["world_size"] == 2 and rec["payload_mb"] == 4096 * 4 / 1e6 and rec["mean_ms"] > 0


def test_validate_socket_shaper(tmp_path):
    out = tmp_path / "v.json"
    subprocess.run([sys.executable, str(ROOT / "scripts" / "validate_bandwidth.py"), "socket", "--bw-gbps", "0.2",
                    "--bytes", "4000000", "--tolerance", "0.5", "--json-output", str(out)], check=True,
                   capture_output=True, timeout=300)
    rec = json.loads(out.read_text())
    assert rec["passed"] and rec["shaped_gbps"] < rec["unshaped_gbps"]


def test_repo_bundle_roundtrip(tmp_path):
    archive = tmp_path / "b.tar.gz"
    subprocess.run(["bash", str(ROOT / "scripts" / "repo_bundle.sh"), "pack", str(archive)], check=True,
                   capture_output=True)
    dest = tmp_path / "unpacked"
    subprocess.run(["bash", str(ROOT / "scripts" / "repo_bundle.sh"), "unpack", str(archive), str(dest)], check=True,
                   capture_output=True)
    assert (dest / "bench.py").exists() and not (dest / ".git").exists()


def test_reference_suite_runner_maps_imports_and_stages(tmp_path):
    sys.path.insert(0, str(ROOT / "scripts"))
    try:
        import run_reference_tests as rrt
    finally:
        sys.path.pop(0)
    src = ("from model.config import ModelConfig\nfrom zero import ZeROStage2Optimizer\nimport analysis.visualize\n"
           "from data.fineweb import PackedFineWebDataset\nfrom experiments import harness\nimport torch\n"
           "cmd = [sys.executable, \"experiments/merge_run_summaries.py\"]\n")
    out = rrt.rewrite(src)
    assert "from cs244c_llama_zero_b200.models.config import ModelConfig" in out
    assert "from cs244c_llama_zero_b200.parallel.zero import ZeROStage2Optimizer" in out
    assert "import cs244c_llama_zero_b200.analysis.visualize" in out
    assert "from cs244c_llama_zero_b200.data.datasets import PackedFineWebDataset" in out
    assert "from cs244c_llama_zero_b200.experiments import harness" in out and "import torch\n" in out
    assert '"-m", "cs244c_llama_zero_b200.experiments.merge_run_summaries"' in out
    fake = tmp_path / "ref"
    (fake / "tests").mkdir(parents=True)
    (fake / "tests" / "test_x.py").write_text("from model import build_tiny_config\n\ndef test_ok():\n    assert build_tiny_config()\n")
    (fake / "tests" / "conftest.py").write_text("")
    staged = rrt.stage(fake, tmp_path / "staged")
    assert [p.name for p in staged] == ["test_x.py"]
    assert "cs244c_llama_zero_b200.models" in staged[0].read_text()
    assert (tmp_path / "staged" / "train_zero.py").exists()


def test_bench_roofline_entry():
    import types

    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    from cs244c_llama_zero_b200.models import build_config
    from cs244c_llama_zero_b200.profiler import executed_train_flops

    cfg = build_config("baseline-small", vocab_size=32000, max_seq_len=1024)
    sess = types.SimpleNamespace(model_cfg=cfg, engine=types.SimpleNamespace(recompute=False))
    args = bench.parse_args(["--batch-size", "8", "--seq-len", "1024"])
    assert args.extra_list == ["baseline-1.3b"] and set(args.extra_list) <= set(bench.CONFIG_SHAPES)
    e = bench.roofline_entry(sess, 8, 1024, 2, 10.0, 1400.0)
    flops = executed_train_flops(cfg, 8, 1024)
    assert abs(e["executed_tflops_per_gpu"] - flops / 0.01 / 1e12) < 1e-6
    assert abs(e["roofline_fraction"] - flops / 0.01 / 1.4e15) < 1e-9
    assert 0.3 < e["roofline_fraction"] < 0.8  # ~5.4 TFLOP in 10 ms on a 1.4 PFLOP/s part


def test_bench_config_shapes_match_the_presets():
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    from cs244c_llama_zero_b200.models import build_config

    for size, shape in bench.CONFIG_SHAPES.items():
        cfg = build_config(size, vocab_size=32000, max_seq_len=shape["seq"])
        for key in ("dim", "n_layers", "n_heads", "n_kv_heads", "ffn_dim"):
            assert getattr(cfg, key) == shape[key], (size, key)


def test_clock_sampler_summary_from_samples():
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    cs = bench.ClockSampler([0])
    cs.samples = [(0, 1965.0, 1965.0, []), (0, 1900.0, 1965.0, ["sw_power_cap"]), (0, 300.0, 1965.0, [])]
    s = cs.summary()
    assert s["sm_mhz"] == 1932.5 and s["sm_max_mhz"] == 1965.0 and s["reasons"] == ["sw_power_cap"]


def test_bench_cuda_graph_default_follows_world_size(monkeypatch):
    """``--cuda-graph auto`` (the default) captures stages 0-2 at one GPU only; on/off force it."""
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    assert bench.parse_args([]).cuda_graph is True
    assert bench.parse_args(["--cuda-graph", "off"]).cuda_graph is False
    monkeypatch.setenv("WORLD_SIZE", "8")
    assert bench.parse_args(["--gpus", "8"]).cuda_graph is False
    assert bench.parse_args(["--gpus", "8", "--cuda-graph"]).cuda_graph is True
