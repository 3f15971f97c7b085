"""CPU unit tests: model (eager oracle backend), presets, data packing, flat-param helpers, profiler, tracing.

The golden loss and the parameter-count ranges are the reference's own test vectors
(tests/test_model.py, tests/test_config.py there); matching them pins the same initialisation order
and the same loss definition (in-model label shift, mean over all shifted tokens).
"""

from __future__ import annotations

import math
import time

import pytest
import torch

from cs244c_llama_zero_b200.data import PackedFineWebDataset, RankShardIterableDataset, SyntheticPatternDataset
from cs244c_llama_zero_b200.models import (LlamaForCausalLM, ModelConfig, build_config, build_medium_config,
                                           build_small_config, build_tiny_config, estimate_num_parameters)
from cs244c_llama_zero_b200.models.llama import RotaryEmbedding, apply_rotary_pos_emb
from cs244c_llama_zero_b200.parallel.collectives import LocalCollectives, TracingCollectives, aggregate_collective_trace
from cs244c_llama_zero_b200.profiler import (FlopTracker, MemoryTracker, TimerRegistry, estimate_transformer_train_flops,
                                             flops_to_tflops_per_second, overlap_efficiency)


def _tiny() -> ModelConfig:
    return ModelConfig(name="unit_test", vocab_size=128, max_seq_len=16, dim=64, n_layers=2, n_heads=4, n_kv_heads=2,
                       ffn_dim=128, dropout=0.0)


GOLDEN_IDS = torch.tensor([[3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7, 9, 3],
                           [2, 7, 1, 8, 2, 8, 1, 8, 2, 8, 4, 5, 9, 0, 4, 5]])


def test_forward_shape_and_backward():
    cfg = _tiny()
    model = LlamaForCausalLM(cfg)
    x = torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len))
    out = model(input_ids=x, labels=x)
    assert out.logits.shape == (2, cfg.max_seq_len, cfg.vocab_size) and torch.isfinite(out.loss)
    out.loss.backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in model.parameters())


def test_chunked_loss_golden_value():
    torch.manual_seed(123)
    model = LlamaForCausalLM(_tiny())
    model.set_loss_chunk_size(4)
    out = model(input_ids=GOLDEN_IDS, labels=GOLDEN_IDS, return_logits=False)
    assert out.logits is None
    torch.testing.assert_close(out.loss.detach(), torch.tensor(4.901787757873535), atol=1e-6, rtol=0.0)


def test_chunked_loss_and_checkpointing_match_full():
    torch.manual_seed(123)
    full = LlamaForCausalLM(_tiny())
    other = LlamaForCausalLM(_tiny())
    other.load_state_dict(full.state_dict())
    other.set_loss_chunk_size(4)
    other.set_activation_checkpointing(True)
    x = torch.randint(0, 128, (2, 16))
    a = full(input_ids=x, labels=x, return_logits=False).loss
    b = other(input_ids=x, labels=x, return_logits=False).loss
    a.backward()
    b.backward()
    torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)
    for (n, p), q in zip(full.named_parameters(), other.parameters()):
        torch.testing.assert_close(p.grad, q.grad, atol=1e-6, rtol=1e-5, msg=n)


def test_causal_mask_and_rope_norm():
    torch.manual_seed(0)
    model = LlamaForCausalLM(_tiny()).eval()
    x = torch.randint(0, 128, (1, 16))
    y = x.clone()
    y[0, -1] = (y[0, -1] + 1) % 128
    with torch.no_grad():
        la, lb = model(input_ids=x).logits, model(input_ids=y).logits
    torch.testing.assert_close(la[:, :-1], lb[:, :-1])
    rope = RotaryEmbedding(dim=16, base=500_000.0)
    q = torch.randn(1, 2, 16, 16)
    cos, sin = rope(16, q.device, q.dtype)
    qr, _ = apply_rotary_pos_emb(q, q, cos, sin)
    torch.testing.assert_close(qr.norm(dim=-1), q.norm(dim=-1), atol=1e-5, rtol=1e-5)


def test_model_learns_deterministic_task():
    torch.manual_seed(7)
    cfg = ModelConfig(name="overfit", vocab_size=64, max_seq_len=16, dim=48, n_layers=2, n_heads=4, n_kv_heads=2,
                      ffn_dim=128, dropout=0.0)
    model = LlamaForCausalLM(cfg)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3, weight_decay=0.0)
    batch = torch.stack([torch.arange(s, s + 17) % 64 for s in (0, 3, 9, 15)])[:, :-1]
    losses = []
    for _ in range(40):
        opt.zero_grad(set_to_none=True)
        loss = model(input_ids=batch, labels=batch).loss
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < 0.7 * losses[0]


def test_generate_extends_sequence():
    torch.manual_seed(1)
    model = LlamaForCausalLM(_tiny()).eval()
    out = model.generate(GOLDEN_IDS[:1, :4], max_new_tokens=5)
    assert out.shape == (1, 9) and torch.equal(out[:, :4], GOLDEN_IDS[:1, :4])


def test_presets_and_parameter_counts():
    tiny, small, medium = build_tiny_config(), build_small_config(), build_medium_config()
    n = [estimate_num_parameters(c) for c in (tiny, small, medium)]
    assert n[0] < n[1] < n[2]
    assert 40e6 <= n[0] <= 60e6 and 250e6 <= n[1] <= 400e6 and 1.1e9 <= n[2] <= 1.5e9
    s = build_config("baseline-small", vocab_size=32000)
    assert (s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.ffn_dim) == (768, 12, 12, 4, 2048)
    m = LlamaForCausalLM(build_config("tiny", vocab_size=512, max_seq_len=32))
    assert estimate_num_parameters(m.cfg) == sum(p.numel() for p in m.parameters())
    with pytest.raises(ValueError):
        build_config("nope")


def test_data_packing_synthetic_and_rank_shard():
    class Tok:
        def encode(self, text, add_special_tokens=False):
            return [ord(c) % 32 for c in text]

    chunks = list(PackedFineWebDataset(text_iterable=[{"text": "abcd"}, {"text": "efgh"}, {"text": "ijkl"}],
                                       tokenizer=Tok(), seq_len=4, eos_token_id=1))
    assert len(chunks) >= 2 and all(c.shape == (5,) for c in chunks)
    syn = SyntheticPatternDataset(seq_len=8, vocab_size=10)
    first = next(iter(syn))
    assert first.shape == (9,) and torch.equal(first, torch.arange(9) % 10)
    shard = list(RankShardIterableDataset(list(range(10)), rank=1, world_size=3))
    assert shard == [1, 4, 7]


def test_profiler_pieces():
    assert overlap_efficiency(step_ms=15.0, compute_ms=10.0, communication_ms=5.0) == 0.0
    assert overlap_efficiency(step_ms=10.0, compute_ms=10.0, communication_ms=5.0) == 1.0
    reg = TimerRegistry(device=None)
    t = reg.timer("sleep")
    t.start()
    time.sleep(0.01)
    t.stop()
    s = reg.summarize()["sleep"]
    assert s.count == 1 and s.total_ms > 0
    mem = MemoryTracker(device=None)
    mem.record("before")
    mem.record("after")
    assert [d["label"] for d in mem.as_dicts()] == ["before", "after"]
    ft = FlopTracker(device=None)
    layer = torch.nn.Linear(16, 8)
    x = torch.randn(4, 16)
    _, flops = ft.measure("linear_step", lambda: layer(x).square().mean().backward())
    assert flops > 0 and ft.as_dicts()[0]["label"] == "linear_step"
    assert flops_to_tflops_per_second(total_flops=flops, step_time_s=0.5) > 0
    cfg = build_tiny_config(vocab_size=1024, max_seq_len=64)
    f0 = estimate_transformer_train_flops(cfg, batch_size=4, seq_len=64, grad_accum_steps=2, world_size=4, stage=0)
    f3 = estimate_transformer_train_flops(cfg, batch_size=4, seq_len=64, grad_accum_steps=2, world_size=4, stage=3)
    assert 0 < f0 < f3


def test_tracing_collectives_and_aggregation():
    traced = TracingCollectives(LocalCollectives())
    shard = torch.arange(4, dtype=torch.bfloat16)
    with traced.label_scope("stage2.step.allgather.updated_param_shard"):
        out = traced.allgather(shard)
    rec = traced.consume_trace()
    assert out.numel() == 4 and len(rec) == 1 and traced.consume_trace() == []
    assert rec[0]["op"] == "allgather" and rec[0]["label"] == "stage2.step.allgather.updated_param_shard"
    assert rec[0]["input_bytes"] == 8 and rec[0]["output_bytes"] == 8
    summary = aggregate_collective_trace([
        {"op": "allgather", "label": "l0", "elapsed_ms": 2.0, "input_bytes": 4, "output_bytes": 16},
        {"op": "allgather", "label": "l0", "elapsed_ms": 3.0, "input_bytes": 4, "output_bytes": 16},
        {"op": "reduce_scatter", "label": "l1", "elapsed_ms": 1.5, "input_bytes": 16, "output_bytes": 4}])
    assert summary == [
        {"op": "allgather", "label": "l0", "calls": 2, "elapsed_ms": 5.0, "input_bytes": 8.0, "output_bytes": 32.0},
        {"op": "reduce_scatter", "label": "l1", "calls": 1, "elapsed_ms": 1.5, "input_bytes": 16.0,
         "output_bytes": 4.0}]


def test_nvtx_ranges_are_balanced_and_off_by_default(monkeypatch):
    from cs244c_llama_zero_b200.profiler import nvtx

    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    monkeypatch.setattr(torch.cuda.nvtx, "mark", lambda name: calls.append(("mark", name)))
    was = nvtx.enabled()
    try:
        nvtx.enable(False)
        with nvtx.nvtx_range("off"):
            nvtx.mark("off")
        assert calls == []
        nvtx.enable(True)
        with nvtx.nvtx_range("step"):
            with nvtx.nvtx_range("forward"):
                nvtx.mark("m")
        with pytest.raises(RuntimeError):
            with nvtx.nvtx_range("raises"):
                raise RuntimeError("x")
        assert calls == [("push", "step"), ("push", "forward"), ("mark", "m"), ("pop",), ("pop",),
                         ("push", "raises"), ("pop",)]
    finally:
        nvtx.enable(was)


def test_peak_lookup_and_roofline_fraction(tmp_path, monkeypatch):
    import json as _json

    from cs244c_llama_zero_b200.profiler import flops as F

    monkeypatch.delenv("ZB_PEAK_TFLOPS", raising=False)
    assert F.peak_bf16_tflops(str(tmp_path)) == (F.FALLBACK_PEAK_BF16_TFLOPS, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(_json.dumps({"bf16_tflops": 1646.4, "bf16_tflops_sustained": 1388.8}))
    assert F.peak_bf16_tflops(str(tmp_path)) == (1388.8, "measured")
    monkeypatch.setenv("ZB_PEAK_TFLOPS", "1000")
    assert F.peak_bf16_tflops(str(tmp_path)) == (1000.0, "ZB_PEAK_TFLOPS")
    assert F.roofline_fraction(5e14, 1.0, 1000.0) == pytest.approx(0.5)
    assert F.roofline_fraction(1.0, 0.0, 1000.0) is None


def test_rope_tables_frequency_major_layout():
    """The q|k|v GEMM's RoPE epilogue reads the same angles frequency-major: [head_dim/2, seq_len]."""
    import torch

    from cs244c_llama_zero_b200.ops.functional import rope_tables, rope_tables_t

    cos, sin = rope_tables(64, 32, 10000.0, torch.device("cpu"))
    cos_t, sin_t = rope_tables_t(64, 32, 10000.0, torch.device("cpu"))
    assert cos.shape == (64, 16) and cos_t.shape == (16, 64) and cos_t.is_contiguous()
    assert torch.equal(cos_t, cos.t()) and torch.equal(sin_t, sin.t())
    pos, i = 37, 5
    angle = pos * 10000.0 ** (-2 * i / 32)
    assert abs(float(cos_t[i, pos]) - math.cos(angle)) < 1e-5 and abs(float(sin_t[i, pos]) - math.sin(angle)) < 1e-5
