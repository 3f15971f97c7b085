"""TrainSession on CPU: synchronous and asynchronous loss readback give the same training run."""

from __future__ import annotations

import math

import torch

from cs244c_llama_zero_b200.train import AsyncLoss, SessionConfig, TrainSession


def _session(stage: int) -> TrainSession:
    torch.manual_seed(0)
    cfg = SessionConfig(model_size="baseline-tiny", vocab_size=97, seq_len=16, batch_size=2, zero_stage=stage,
                        learning_rate=1e-2, model_overrides={"dim": 32, "n_layers": 1, "n_heads": 2, "n_kv_heads": 1,
                                                             "ffn_dim": 64})
    return TrainSession(cfg)


def test_async_loss_matches_sync_steps():
    g = torch.Generator().manual_seed(3)
    batches = [torch.randint(0, 97, (2, 16), generator=g)] * 4  # one batch, so the loss must fall
    for stage in (0, 3):
        sync, asyn = _session(stage), _session(stage)
        want = [float(sync.train_step(b)) for b in batches]
        handles = [asyn.train_step_async(b) for b in batches]
        assert all(isinstance(h, AsyncLoss) for h in handles)
        got = [h.item() for h in handles]
        assert all(math.isfinite(x) for x in got)
        assert got == want, (stage, got, want)
        assert want[-1] < want[0]  # it trains


def test_graph_mode_is_eager_on_cpu_and_clock_can_pause():
    from cs244c_llama_zero_b200.parallel.zero.base import CommClock

    torch.manual_seed(0)
    cfg = SessionConfig(model_size="baseline-tiny", vocab_size=97, seq_len=16, batch_size=2, zero_stage=2,
                        learning_rate=1e-2, cuda_graph=True,
                        model_overrides={"dim": 32, "n_layers": 1, "n_heads": 2, "n_kv_heads": 1, "ffn_dim": 64})
    sess = TrainSession(cfg)
    assert sess.graph_unsupported_reason() is None
    b = torch.randint(0, 97, (2, 16), generator=torch.Generator().manual_seed(1))
    assert math.isfinite(float(sess.train_step(b))) and sess._graph is None
    clock = CommClock(torch.device("cpu"))
    clock.timing = False
    with clock.measure("allreduce", 64):
        pass
    assert clock.calls["allreduce"] == 1 and clock.ms("allreduce") == 0.0
