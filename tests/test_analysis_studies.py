"""Analysis studies on synthetic run directories: step-latency fit, comm-shape probe, bucket inflation,
two-view throughput plots and the ZeRO memory diagram."""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from cs244c_llama_zero_b200.analysis import (memory_parallelism_diagram, plot_throughput_two_views,
                                             stage2_bucket_inflation_probe, stage2_stage3_commshape_probe,
                                             stage2_stage3_step_latency)


def _run(tmp: Path, name: str, stage: int, batch: int, points) -> Path:
    d = tmp / name
    d.mkdir()
    res = [{"config": {"stage": stage, "model_size": "small", "bandwidth_gbps": bw, "batch_size": batch,
                       "seq_len": 128, "grad_accum_steps": 1}, "mean_tokens_per_s": tps, "mean_tflops_per_s": tps / 100,
            "return_code": 0, "log_path": "x.log"} for bw, tps in points]
    (d / "summary.json").write_text(json.dumps({"args": {"nproc_per_node": 4}, "results": res}))
    return d


def test_step_latency_fit_recovers_model(tmp_path):
    # tokens/step = 4 * 128 * 4 = 2048 (stage 2), 8192 (stage 3); t = a + b / bw
    def pts(tokens, a, b):
        return [(0.0, tokens / a)] + [(bw, tokens / (a + b / bw)) for bw in (1.0, 2.0, 5.0)]

    r2 = _run(tmp_path, "s2", 2, 4, pts(2048, 0.5, 2.0))
    r3 = _run(tmp_path, "s3", 3, 16, pts(8192, 1.0, 3.0))
    res = stage2_stage3_step_latency.analyse([str(r2)], [str(r3)])
    assert res["stage2"]["a_s"] == pytest.approx(0.5) and res["stage2"]["b_s_gbps"] == pytest.approx(2.0)
    assert res["stage3"]["b_s_gbps"] == pytest.approx(3.0)
    assert res["token_ratio_stage3_over_stage2"] == 4.0
    assert res["latency_ratio_unlimited"] == pytest.approx(2.0)
    assert res["throughput_ratio_low_bw"] == pytest.approx(4.0 * 2.0 / 3.0)
    assert stage2_stage3_step_latency.plot(res, tmp_path / "lat.svg").exists()
    with pytest.raises(ValueError):
        stage2_stage3_step_latency.fit_bandwidth_model([])


def test_commshape_probe(tmp_path):
    prof = tmp_path / "run" / "profiles"
    prof.mkdir(parents=True)

    def step(n, **kw):
        base = {"step": n, "iteration_ms": 10.0, "forward_backward_ms": 6.0, "optimizer_ms": 1.0,
                "communication_ms": 3.0, "tokens_per_second": 100.0}
        base.update(kw)
        return base

    for stage, extra in ((2, {"communication_backward_reduce_scatter_ms": 2.0,
                              "communication_backward_reduce_scatter_calls": 1.0,
                              "communication_backward_reduce_scatter_bytes": float(2 ** 21)}),
                         (3, {"communication_forward_allgather_ms": 4.0, "communication_forward_allgather_calls": 15.0,
                              "iteration_ms": 20.0, "tokens_per_second": 50.0})):
        payload = {"stage": stage, "model_config": {"name": "small"}, "steps": [step(1), step(2, **extra), step(3, **extra)]}
        (prof / f"s{stage}_msmall_bw1gbps_np4_sl128_bs4_ga1_seed1.json").write_text(json.dumps(payload))
    cases = stage2_stage3_commshape_probe.load_profiles(tmp_path / "run", start_step=2)
    assert set(cases) == {("small", 1.0, 2), ("small", 1.0, 3)}
    assert cases[("small", 1.0, 2)]["backward_reduce_scatter_bytes"] == 2 ** 21
    assert cases[("small", 1.0, 2)]["forward_allgather_ms"] == 0.0
    text = stage2_stage3_commshape_probe.render(cases)
    assert "## Stage 3 / stage 2" in text and "| small | 1 | 2.000 |" in text
    assert stage2_stage3_commshape_probe.bandwidth_from_case_id("s2_mx_bwunlimited_np4") == 0.0


def test_bucket_inflation():
    ranges = stage2_bucket_inflation_probe.bucket_ranges([4, 4, 4, 10, 2], 8)
    assert ranges == [(0, 8), (8, 12), (12, 22), (22, 24)]
    rows = stage2_bucket_inflation_probe.inflation_rows([4, 4, 4, 4], world=2, bucket_numel=8)
    # shard size 8: bucket 0 = rank 0's shard only -> packed 2 x 8 = 16 elements for 8 logical
    assert [r.inflation for r in rows] == [2.0, 2.0]
    assert stage2_bucket_inflation_probe.inflation_rows([3, 5], world=2, bucket_numel=100)[0].inflation == 1.0


def test_two_views_and_memory_diagram(tmp_path):
    run = _run(tmp_path, "bw", 0, 4, [(0.0, 500.0), (1.0, 200.0), (5.0, 400.0), (20.0, 480.0)])
    by = plot_throughput_two_views.cases_by_stage(
        plot_throughput_two_views.parse_summary(run / "summary.json"))
    assert plot_throughput_two_views.plot_zoom(by, tmp_path / "z.svg").exists()
    assert "inf" in plot_throughput_two_views.plot_overview(by, tmp_path / "o.svg").read_text()
    b = memory_parallelism_diagram.per_device_bytes(psi=1000, n_d=4, k=12)
    assert b["Baseline"]["total"] == 16000 and b["P_os"]["total"] == 4000 + 3000
    assert b["P_os+g"]["total"] == 2000 + 14000 / 4 and b["P_os+g+p"]["total"] == 4000
    assert memory_parallelism_diagram.render_svg(1000, 16, 12, "t").count("<rect") > 16
