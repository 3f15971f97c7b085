"""Micro-batch search, stage-3 batch prediction, crossover search rule, run merging, reports and charts (CPU).

Expected probe orders and predictions are the reference's own test vectors
(tests/test_fit_memory_bandwidth.py, tests/test_stage3_scaling_sweep.py,
tests/test_pairwise_crossover_search.py there): each probe is a training launch, so the order matters.
"""

from __future__ import annotations

import json
import subprocess
import sys
from argparse import Namespace
from pathlib import Path

import pytest

from cs244c_llama_zero_b200.analysis import bandwidth_report, collective_trace_report, stage3_scaling, visualize
from cs244c_llama_zero_b200.experiments import (run_fit_memory_bandwidth, run_pairwise_crossover_search,
                                                run_stage3_scaling_sweep, tuning)
from cs244c_llama_zero_b200.experiments.run_pairwise_crossover_search import PairwisePoint, choose_next_finite_bandwidth

ROOT = Path(__file__).resolve().parents[1]


def _trial(batch: int, fits: bool = True, peak: float | None = None) -> tuning.TuningTrial:
    return tuning.TuningTrial(batch_size=batch, fits=fits, peak_memory_mb=peak if peak is not None else
                              (float(batch * 100) if fits else None), return_code=0 if fits else 1,
                              reason="ok" if fits else "over_budget", case_id=f"c{batch}", log_path="",
                              profile_path="", mean_tokens_per_s=None)


# ------------------------------------------------------------------------------ boundary search
@pytest.mark.parametrize("lo,hi,mult,init,limit,best,seen", [
    (1, 16, 1, 0, 10, 10, [8, 16, 12, 10, 11]),
    (4, 32, 4, 0, 18, 16, [16, 32, 24, 20]),
    (4, 512, 4, 256, 84, 84, [256, 128, 64, 96, 80, 88, 84]),
])
def test_search_probe_order(lo, hi, mult, init, limit, best, seen):
    probes = []

    def evaluator(b):
        probes.append(b)
        return _trial(b, b <= limit)

    top, trials = tuning.search_max_batch_size(lo, hi, mult, 2.0, init, evaluator)
    assert top.batch_size == best and probes == seen
    assert [t.batch_size for t in trials] == sorted(seen)


def test_search_caps_at_max_and_raises_when_nothing_fits():
    top, trials = tuning.search_max_batch_size(1, 20, 1, 2.0, 0, lambda b: _trial(b, True))
    assert top.batch_size == 20 and [t.batch_size for t in trials] == [10, 20]
    with pytest.raises(RuntimeError, match="no fitting batch size"):
        tuning.search_max_batch_size(1, 8, 1, 2.0, 0, lambda b: _trial(b, False))
    with pytest.raises(ValueError):
        tuning.search_max_batch_size(0, 8, 1, 2.0, 0, lambda b: _trial(b))


def test_reference_name_aliases():
    assert run_fit_memory_bandwidth._select_max_batch_size is tuning.search_max_batch_size
    assert run_stage3_scaling_sweep._predict_initial_batch_size is tuning.predict_initial_batch_size


# ------------------------------------------------------------------------------ stage-3 prediction
def _pred_args(mult=1, max_batch=128, strategy="predictive"):
    return Namespace(min_batch_size=1, max_batch_size=max_batch, batch_size_multiple=mult, initial_batch_size=0,
                     tuning_strategy=strategy)


def test_predict_shard_ratio_fallback():
    pred, info = tuning.predict_initial_batch_size(
        _pred_args(mult=4), gpu_count=4, previous_selected_batch_size=20, previous_gpu_count=2,
        selected_trials_by_gpu_count={2: _trial(20, peak=22_000.0)},
        trial_history_by_gpu_count={2: [_trial(20, peak=22_000.0)]})
    assert pred == 40 and info["kind"] == "shard_ratio"


def test_predict_memory_model():
    sel = {1: _trial(50, peak=10_000.0), 2: _trial(70, peak=10_000.0)}
    hist = {1: [_trial(20, peak=7_000.0), _trial(40, peak=9_000.0), sel[1]],
            2: [_trial(40, peak=7_000.0), _trial(60, peak=9_000.0), sel[2]]}
    pred, info = tuning.predict_initial_batch_size(_pred_args(mult=2), gpu_count=4, previous_selected_batch_size=70,
                                                   previous_gpu_count=2, selected_trials_by_gpu_count=sel,
                                                   trial_history_by_gpu_count=hist)
    assert pred == 80 and info["kind"] == "memory_model" and info["budget_mb"] == 10_000.0


def test_predict_prefers_shard_ratio_with_one_gpu_count():
    sel = {1: _trial(19, peak=22_000.0)}
    hist = {1: [_trial(16, peak=20_800.0), _trial(18, peak=21_600.0), sel[1]]}
    pred, info = tuning.predict_initial_batch_size(_pred_args(), gpu_count=2, previous_selected_batch_size=19,
                                                   previous_gpu_count=1, selected_trials_by_gpu_count=sel,
                                                   trial_history_by_gpu_count=hist)
    assert pred == 38 and info["kind"] == "shard_ratio"


def test_predict_exponential_uses_configured_guess():
    pred, info = tuning.predict_initial_batch_size(_pred_args(strategy="exponential"), gpu_count=2,
                                                   previous_selected_batch_size=12, previous_gpu_count=1,
                                                   selected_trials_by_gpu_count={}, trial_history_by_gpu_count={})
    assert pred == 12 and info["kind"] == "configured_initial_guess"


def test_least_squares_line():
    assert tuning.least_squares_line([(0.0, 1.0), (1.0, 3.0), (2.0, 5.0)]) == pytest.approx((2.0, 1.0))
    assert tuning.least_squares_line([(1.0, 1.0)]) is None
    assert tuning.least_squares_line([(1.0, 1.0), (1.0, 2.0)]) is None


# ------------------------------------------------------------------------------ crossover rule
def _pt(bw, ratio):
    return PairwisePoint(bw, 100.0, 100.0 * ratio, 0.0, 0.0, 0.0, 0.0, ratio, 3 if ratio >= 1.0 else 2)


def test_crossover_prefers_sign_flip():
    nxt = choose_next_finite_bandwidth({0.01: _pt(0.01, 1.5), 0.1: _pt(0.1, 0.8), 0.5: _pt(0.5, 0.6)},
                                       tolerance_ratio=1.25)
    assert nxt == (0.01 * 0.1) ** 0.5


def test_crossover_targets_parity_without_flip():
    nxt = choose_next_finite_bandwidth({0.01: _pt(0.01, 2.0), 0.1: _pt(0.1, 1.1), 0.5: _pt(0.5, 1.8)},
                                       tolerance_ratio=1.25)
    assert nxt == (0.1 * 0.5) ** 0.5


def test_crossover_stops_when_tight():
    assert choose_next_finite_bandwidth({0.4: _pt(0.4, 1.1), 0.45: _pt(0.45, 0.95)}, tolerance_ratio=1.25) is None
    sampled = {0.01: _pt(0.01, 1.5), 0.1: _pt(0.1, 0.8)}
    lo, hi = run_pairwise_crossover_search.best_flip_bracket(sampled)
    assert (lo.bandwidth_gbps, hi.bandwidth_gbps) == (0.01, 0.1)
    assert run_pairwise_crossover_search.nearest_parity_point(sampled).bandwidth_gbps == 0.1
    assert run_pairwise_crossover_search.seed_bandwidths(0.01, 1.0, [0.5, -1]) == [1.0, 0.5, 0.1, 0.01]


# ------------------------------------------------------------------------------ runners (dry run, no GPU)
def test_fit_memory_dry_run_writes_tuning(tmp_path):
    args = run_fit_memory_bandwidth.parse_args(["--results-dir", str(tmp_path), "--name", "fm", "--dry-run",
                                                "--stages", "0", "3", "--max-batch-size", "16"])
    out = run_fit_memory_bandwidth.run(args, gpu_total_memory_mb=1000.0)
    data = json.loads((tmp_path / "fm" / "tuning_summary.json").read_text())
    assert data == json.loads(json.dumps(out))
    assert data["per_stage"]["3"]["selected_batch_size"] == 16
    assert [t["batch_size"] for t in data["per_stage"]["0"]["trials"]] == [8, 16]


def test_stage3_fixed_batch_dry_run(tmp_path):
    args = run_stage3_scaling_sweep.parse_args(["--results-dir", str(tmp_path), "--name", "s3", "--dry-run",
                                                "--gpu-counts", "2", "1", "--fixed-batch-size", "4"])
    summary = run_stage3_scaling_sweep.run(args, per_gpu_total_memory_mb=1000.0)
    assert summary["gpu_counts"] == [1, 2] and summary["scaling_mode"] == "fixed_batch"
    assert summary["per_gpu_count"]["2"]["fit_status"] == "fit"


def test_stage3_tuned_dry_run_uses_predictor(tmp_path):
    args = run_stage3_scaling_sweep.parse_args(["--results-dir", str(tmp_path), "--name", "s3t", "--dry-run",
                                                "--gpu-counts", "1", "2", "--max-batch-size", "8"])
    summary = run_stage3_scaling_sweep.run(args, per_gpu_total_memory_mb=1000.0)
    assert summary["per_gpu_count"]["1"]["tuning_prediction"]["kind"] == "configured_initial_guess"
    assert summary["per_gpu_count"]["2"]["tuning_prediction"]["kind"] == "shard_ratio"


def test_scaling_efficiency_annotation():
    pts = [{"gpu_count": 4, "mean_tflops_per_s": 30.0}, {"gpu_count": 1, "mean_tflops_per_s": 10.0}]
    run_stage3_scaling_sweep.add_scaling_efficiency(pts)
    assert [p["gpu_count"] for p in pts] == [1, 4]
    assert pts[1]["speedup_vs_base"] == 3.0 and pts[1]["scaling_efficiency_vs_base"] == 0.75


def test_pairwise_validates_arguments(tmp_path):
    args = run_pairwise_crossover_search.parse_args(["--results-dir", str(tmp_path), "--stage-a", "2",
                                                     "--stage-b", "2"])
    with pytest.raises(ValueError):
        run_pairwise_crossover_search.run(args, gpu_total_memory_mb=1.0)


def test_pairwise_fixed_batches_dry_run(tmp_path):
    args = run_pairwise_crossover_search.parse_args(["--results-dir", str(tmp_path), "--name", "pw", "--dry-run",
                                                     "--stage-a-batch-size", "4", "--stage-b-batch-size", "8"])
    out = run_pairwise_crossover_search.run(args, gpu_total_memory_mb=1.0)
    assert out["per_stage"]["3"]["selection_mode"] == "fixed_batch_size"


# ------------------------------------------------------------------------------ merge + reports
def _result(stage, bw, tps, comm, batch=4, rc=0, **extra):
    return {"config": {"stage": stage, "model_size": "small", "bandwidth_gbps": bw, "batch_size": batch,
                       "seq_len": 128, "grad_accum_steps": 1}, "log_path": f"logs/s{stage}_{bw}.log",
            "profile_path": "", "mean_tokens_per_s": tps, "mean_comm_ms": comm, "return_code": rc, **extra}


def test_merge_prefers_later_runs(tmp_path):
    args = {"bandwidth_mode": "socket", "nproc_per_node": 4, "steps": 4, "metrics_warmup_steps": 1}
    for name, results in (("a", [_result(0, 0.0, 100.0, 10.0)]),
                          ("b", [_result(0, 0.0, 110.0, 9.0), _result(3, 0.0, 150.0, 20.0, batch=8)])):
        (tmp_path / name).mkdir()
        (tmp_path / name / "summary.json").write_text(json.dumps({"name": name, "args": args, "results": results}))
    subprocess.run([sys.executable, "-m", "cs244c_llama_zero_b200.experiments.merge_run_summaries", "--run-dirs",
                    str(tmp_path / "a"), str(tmp_path / "b"), "--output-run-dir", str(tmp_path / "merged")],
                   check=True, cwd=ROOT)
    merged = json.loads((tmp_path / "merged" / "summary.json").read_text())
    assert merged["name"] == "merged" and merged["num_cases"] == 2
    assert [r["mean_tokens_per_s"] for r in merged["results"]] == [110.0, 150.0]
    assert (tmp_path / "merged" / "bandwidth_report.md").exists()


def test_bandwidth_report_fixed_workload(tmp_path):
    results = [_result(0, 0.0, 100.0, 5.0), _result(0, 5.0, 80.0, 8.0), _result(1, 0.0, 120.0, 6.0),
               _result(1, 5.0, 60.0, 12.0)]
    (tmp_path / "summary.json").write_text(json.dumps({"name": "bw", "results": results, "args": {
        "bandwidth_mode": "simulated", "nproc_per_node": 4, "steps": 20, "metrics_warmup_steps": 1}}))
    report = bandwidth_report.generate_report_markdown(tmp_path)
    for needle in ("# Bandwidth Sweep Report", "Experiment type: fixed-workload bandwidth sweep",
                   "Successful cases: 4 / 4", "metrics_warmup_steps=1", "Best stage by bandwidth:",
                   "Stage ranking by bandwidth:", "| unlimited | 1 | 120.0 | 6.0 |", "| 5 Gbps | 0 | 80.0 | 8.0 |",
                   "| stage 0 | 100.0% | 80.0% |", "| stage 1 | 100.0% | 50.0% |",
                   "- 5 Gbps: stage 0 is the fastest stage"):
        assert needle in report, needle


def test_bandwidth_report_fit_to_memory(tmp_path):
    results = [_result(0, 0.0, 500.0, 40.0, batch=1), _result(0, 1.0, 250.0, 80.0, batch=1),
               _result(3, 0.0, 900.0, 60.0), _result(3, 1.0, 200.0, 140.0)]
    (tmp_path / "summary.json").write_text(json.dumps({"name": "fm", "results": results, "args": {
        "bandwidth_mode": "socket", "nproc_per_node": 4, "steps": 8, "metrics_warmup_steps": 2}}))
    (tmp_path / "tuning_summary.json").write_text(json.dumps({
        "memory_budget_mb": 22000.0, "memory_metric": "peak_cuda_max_reserved_mb", "per_stage": {
            "0": {"selected_batch_size": 1, "selected_peak_memory_mb": 21000.0},
            "3": {"selected_batch_size": 4, "selected_peak_memory_mb": 20500.0}}}))
    report = bandwidth_report.generate_report_markdown(tmp_path)
    assert "Experiment type: fit-to-memory bandwidth sweep" in report
    assert "fit-to-memory: each stage is first tuned" in report
    assert "selected cuda max reserved MB" in report
    assert "| 0 | 1 | 512 | 21000.0 | 95.5% |" in report and "| 3 | 4 | 2048 | 20500.0 | 93.2% |" in report


def _view(**kw):
    base = dict(stage=2, model_size="tiny", bandwidth_gbps=0.0, batch_size=1, grad_accum_steps=1, seq_len=1,
                log_path=Path("/nonexistent/x.log"), profile_path=None, mean_tokens_per_s=None,
                mean_tflops_per_s=None, mean_comm_ms=None, mean_fb_ms=None, mean_opt_ms=None, peak_host_rss_mb=None,
                peak_cuda_allocated_mb=None, peak_cuda_reserved_mb=None, peak_cuda_max_allocated_mb=None,
                peak_cuda_max_reserved_mb=None, final_loss=None, return_code=0, measured_state_memory_mb=None,
                theoretical_memory_mb=None)
    base.update(kw)
    return visualize.CaseView(**base)


def test_parse_summary_schemas_and_path_rebase(tmp_path):
    run = tmp_path / "remote_run"
    (run / "logs").mkdir(parents=True)
    (run / "logs" / "case.log").write_text("ok\n")
    (run / "summary.json").write_text(json.dumps({"results": [
        {"config": {"stage": 3, "model_size": "tiny", "bandwidth_gbps": 5.0},
         "log_path": "experiments/results/remote_run/logs/case.log", "mean_tokens_per_s": 123.0,
         "peak_cuda_max_reserved_mb": 444.0, "measured_state_memory_mb": {"total_mb": 205.0}, "return_code": 0},
        {"stage": 2, "log_path": "stage2.log", "return_code": 0}]}))
    a, b = visualize.parse_summary(run / "summary.json")
    assert (a.stage, a.model_size, a.bandwidth_gbps, a.batch_size, a.grad_accum_steps) == (3, "tiny", 5.0, 0, 1)
    assert a.log_path == run / "logs" / "case.log" and a.profile_path is None
    assert a.peak_cuda_max_reserved_mb == 444.0 and a.measured_state_memory_mb == {"total_mb": 205.0}
    assert (b.stage, b.model_size, b.bandwidth_gbps) == (2, "unknown", 0.0)
    assert visualize.parse_loss_log(tmp_path / "missing.log") == ([], [])


def test_peak_memory_rules(tmp_path):
    assert visualize._case_peak_memory_mb(_view(peak_host_rss_mb=512.0, peak_cuda_allocated_mb=0.0)) == 512.0
    assert visualize._case_peak_memory_mb(_view(peak_cuda_max_allocated_mb=333.0, peak_cuda_max_reserved_mb=444.0)) \
        == 333.0
    state = {"params_mb": 50.0, "grads_mb": 25.0, "optimizer_mb": 75.0, "total_mb": 150.0}
    assert visualize._case_peak_breakdown_mb(_view(peak_cuda_max_allocated_mb=333.0,
                                                   measured_state_memory_mb=state)) == (150.0, 183.0)


def test_average_live_breakdown(tmp_path):
    prof = tmp_path / "p.json"
    prof.write_text(json.dumps({"memory": [
        {"label": "start", "cuda_allocated_mb": 80.0}, {"label": "step_1_start", "cuda_allocated_mb": 200.0},
        {"label": "step_1_post_backward", "cuda_allocated_mb": 260.0},
        {"label": "step_1_end", "cuda_allocated_mb": 220.0}]}))
    v = _view(profile_path=prof, measured_state_memory_mb={"params_mb": 50.0, "grads_mb": 20.0, "optimizer_mb": 30.0,
                                                           "total_mb": 100.0})
    assert visualize._case_average_live_breakdown_mb(v) == pytest.approx((100.0, 126.66666666666666))
    prof.write_text(json.dumps({
        "memory": [{"label": "measured_step_1_start", "timestamp_s": 0.0, "cuda_allocated_mb": 10.0},
                   {"label": "measured_step_1_mid", "timestamp_s": 9.0, "cuda_allocated_mb": 30.0},
                   {"label": "measured_step_1_end", "timestamp_s": 10.0, "cuda_allocated_mb": 10.0}],
        "measured_step_state_timeline": [{"label": f"measured_step_1_{p}", "total_mb": 8.0}
                                         for p in ("start", "mid", "end")]}))
    assert visualize._case_average_live_breakdown_mb(v) == pytest.approx((8.0, 4.0))


def test_state_breakdowns_from_timeline(tmp_path):
    prof = tmp_path / "p.json"
    prof.write_text(json.dumps({
        "memory": [{"label": "a", "cuda_allocated_mb": 50.0, "cuda_max_allocated_mb": 80.0},
                   {"label": "b", "cuda_allocated_mb": 60.0, "cuda_max_allocated_mb": 90.0}],
        "measured_step_state_timeline": [
            {"label": "a", "params_mb": 10.0, "grads_mb": 6.0, "optimizer_mb": 5.0, "total_mb": 21.0},
            {"label": "b", "params_mb": 10.0, "grads_mb": 4.0, "optimizer_mb": 5.0, "total_mb": 19.0}]}))
    v = _view(profile_path=prof)
    assert visualize._case_state_breakdown_at_peak_total(v)["total_mb"] == 19.0
    assert visualize._case_peak_state_breakdown(v)["total_mb"] == 21.0


def test_representative_and_svg_plots(tmp_path):
    cases = [_view(stage=0, bandwidth_gbps=5.0, mean_tokens_per_s=50.0),
             _view(stage=0, bandwidth_gbps=0.0, mean_tokens_per_s=90.0, peak_cuda_max_allocated_mb=300.0,
                   measured_state_memory_mb={"params_mb": 1.0, "grads_mb": 1.0, "optimizer_mb": 1.0,
                                             "total_mb": 3.0}),
             _view(stage=1, bandwidth_gbps=2.0, mean_tokens_per_s=40.0),
             _view(stage=1, bandwidth_gbps=5.0, mean_tokens_per_s=60.0, peak_cuda_max_allocated_mb=200.0)]
    picked = visualize._representative_cases_by_stage(cases)
    assert [(c.stage, c.bandwidth_gbps) for c in picked] == [(0, 0.0), (1, 5.0)]
    for kind in ("throughput", "stage-throughput", "grouped-stage-throughput", "peak-memory"):
        out = visualize.render(cases, kind, tmp_path / f"{kind}.png")
        assert out.suffix == ".svg" and out.read_text().startswith("<svg")


def test_stage3_scaling_report(tmp_path):
    summary = {"args": {"model_size": "medium", "seq_len": 256}, "per_gpu_count": {"1": {"fit_status": "no_fit"}},
               "scaling_points": [
                   {"gpu_count": 4, "selected_batch_size": 2, "global_tokens_per_step": 2048, "mean_tflops_per_s": 36.0,
                    "per_gpu_tflops_per_s": 9.0, "peak_cuda_max_allocated_mb": 18000.0},
                   {"gpu_count": 2, "selected_batch_size": 1, "selected_peak_memory_mb": 23000.0,
                    "global_tokens_per_step": 512, "mean_tflops_per_s": 14.0, "per_gpu_tflops_per_s": 7.0}]}
    pts = stage3_scaling.scaling_points(summary)
    assert [p["gpu_count"] for p in pts] == [2, 4] and pts[0]["peak_memory_mb"] == 23000.0
    base = stage3_scaling.choose_baseline_gpu_count(pts, 0)
    ann = stage3_scaling.annotate_points(pts, base)
    assert ann[1]["superlinear_gain_vs_perfect_linear"] == pytest.approx(36.0 / 28.0)
    report = stage3_scaling.render_report(summary, ann, base)
    assert "ZeRO paper" in report and "Strongest superlinear gain" in report and "`1`" in report
    fig = stage3_scaling.plot_figure(ann, tmp_path / "fig.svg", base)
    assert fig.exists() and (tmp_path / "fig_per_gpu.svg").exists()


def test_collective_trace_report(tmp_path):
    prof = tmp_path / "p.json"
    prof.write_text(json.dumps({"stage": 3, "microbatch_size_per_gpu": 2, "args": {"seq_len": 64}, "steps": [
        {"collective_trace": [
            {"op": "allgather", "label": "l0", "elapsed_ms": 2.0, "input_bytes": 4, "output_bytes": 16},
            {"op": "allgather", "label": "l0", "elapsed_ms": 3.0, "input_bytes": 4, "output_bytes": 16},
            {"op": "reduce_scatter", "label": "l1", "elapsed_ms": 1.5, "input_bytes": 16, "output_bytes": 4}]}]}))
    text = collective_trace_report.render_profile(prof)
    assert "| allgather | l0 | 2 | 5.0 |" in text and "- `allgather`: `5.0 ms`" in text
