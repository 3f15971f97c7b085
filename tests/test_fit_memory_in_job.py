"""CPU tests of the in-job fit-to-memory runner's memory model (the GPU run itself is an experiment)."""

from cs244c_llama_zero_b200.experiments.fit_memory_in_job import fit_line, parse_args, predict_max_batch


def test_line_through_two_probes_and_prediction():
    slope, base = fit_line([(1, 130_000.0), (2, 137_500.0)])
    assert abs(slope - 7_500.0) < 1e-9 and abs(base - 122_500.0) < 1e-9
    # 0.88 * 183_359 MiB = 161_355.9 -> (161_355.9 - 122_500) / 7_500 = 5.18 -> 5
    assert predict_max_batch(slope, base, 183_359.0, 0.88, 256) == 5
    assert predict_max_batch(slope, base, 100_000.0, 0.88, 256) == 0  # the state alone does not fit
    assert predict_max_batch(0.0, base, 183_359.0, 0.88, 64) == 64


def test_defaults_are_the_7b_baseline_config():
    a = parse_args([])
    assert a.model_size == "baseline-7b" and a.seq_len == 2048 and a.stages == "0,1,2,3"
