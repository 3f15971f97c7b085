"""ZeRO engines vs single-process AdamW on the gathered global batch (CPU/gloo ranks).

Mirrors the reference's strategy (``zero/tests/test_zero_stages.py:72-544``): each rank
trains on its local batch; a replica trains on the all-gathered global batch with
``torch.optim.AdamW``; parameters must agree after every step.
"""

from __future__ import annotations

import os

from contextlib import nullcontext

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
from cs244c_llama_zero_b200.parallel import TorchCollectives, TracingCollectives
from cs244c_llama_zero_b200.parallel.zero import (
    ZeROStage0DDP,
    ZeROStage1Optimizer,
    ZeROStage2Optimizer,
    ZeROStage3Optimizer,
)
from cs244c_llama_zero_b200.parallel.zero.common import (
    build_flat_param_metadata,
    flatten_param_shard_fp32,
    flatten_params_fp32,
)
from cs244c_llama_zero_b200.profiler import MemoryTracker

from .dist_utils import find_free_port, init_gloo

ENGINES = {0: ZeROStage0DDP, 1: ZeROStage1Optimizer, 2: ZeROStage2Optimizer, 3: ZeROStage3Optimizer}


def _cfg(dropout: float = 0.0) -> ModelConfig:
    return ModelConfig(name="zero_test", vocab_size=97, max_seq_len=8, dim=32, n_layers=2, n_heads=4,
                       n_kv_heads=2, ffn_dim=96, dropout=dropout)


def _local_batch(step: int, rank: int, batch: int, seq: int, vocab: int) -> torch.Tensor:
    base = torch.arange(batch * seq, dtype=torch.long).view(batch, seq)
    return (base + step * 13 + rank * 7) % vocab


def _full(engine):
    return engine.summon_full_params() if hasattr(engine, "summon_full_params") else nullcontext()


def _assert_close(a: LlamaForCausalLM, b: LlamaForCausalLM, msg: str) -> None:
    for (na, pa), (nb, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert na == nb
        torch.testing.assert_close(pa, pb, atol=2e-5, rtol=2e-5, msg=f"{msg} :: {na}")


def test_flatten_param_shard_matches_full_slice() -> None:
    model = LlamaForCausalLM(_cfg())
    meta = build_flat_param_metadata(model)
    flat = flatten_params_fp32(meta)
    for lo, hi in [(0, 17), (11, 57), (meta.total_numel - 23, meta.total_numel)]:
        torch.testing.assert_close(flatten_param_shard_fp32(meta, lo, hi), flat[lo:hi])


def _stage_worker(rank: int, world: int, port: int, stage: int, max_grad_norm: float, impl: str,
                  grad_accum: int) -> None:
    init_gloo(rank, world, port)
    try:
        cfg = _cfg()
        torch.manual_seed(1234)
        model = LlamaForCausalLM(cfg)
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
        ref = LlamaForCausalLM(cfg)
        ref.load_state_dict(model.state_dict())
        hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
        coll = None
        if impl == "torch":
            coll = TorchCollectives()
        elif impl == "tracing":
            coll = TracingCollectives(TorchCollectives())
        engine = ENGINES[stage](model=model, collectives=coll, **hp)
        opt = torch.optim.AdamW(ref.parameters(), **hp)
        for step in range(3):
            micro = [_local_batch(step * 10 + m, rank, 3, cfg.max_seq_len, cfg.vocab_size) for m in range(grad_accum)]
            engine.zero_grad()
            engine.prepare_forward()
            for ids in micro:
                loss = model(input_ids=ids, labels=ids).loss
                engine.backward(loss / grad_accum)
            engine.step(max_grad_norm=max_grad_norm)

            opt.zero_grad(set_to_none=True)
            for ids in micro:
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                g = torch.cat(parts)
                (ref(input_ids=g, labels=g).loss / grad_accum).backward()
            if max_grad_norm > 0:
                torch.nn.utils.clip_grad_norm_(ref.parameters(), max_norm=max_grad_norm)
            opt.step()
            with _full(engine):
                _assert_close(model, ref, f"stage={stage} step={step} rank={rank}")
        if impl == "tracing":
            trace = engine.collectives.consume_trace()
            assert trace and all("op" in r and "label" in r for r in trace)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _spawn(fn, world: int, *args) -> None:
    mp.spawn(fn, args=(world, find_free_port(), *args), nprocs=world, join=True)


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
@pytest.mark.parametrize("world", [2, 3])
def test_stages_match_reference_global_batch(stage: int, world: int) -> None:
    _spawn(_stage_worker, world, stage, 0.0, "ring", 1)


@pytest.mark.parametrize("stage", [2, 3])
def test_sharded_stage_with_clipping_world3(stage: int) -> None:
    _spawn(_stage_worker, 3, stage, 0.5, "ring", 1)


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_stages_with_torch_collectives_and_grad_accum(stage: int) -> None:
    _spawn(_stage_worker, 2, stage, 0.3, "torch", 2)


@pytest.mark.parametrize("stage", [2, 3])
def test_stages_with_tracing_collectives(stage: int) -> None:
    _spawn(_stage_worker, 2, stage, 0.0, "tracing", 1)


def _materialization_worker(rank: int, world: int, port: int) -> None:
    init_gloo(rank, world, port)
    try:
        model = LlamaForCausalLM(_cfg())
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
        engine = ZeROStage3Optimizer(model=model, lr=1e-3, weight_decay=0.0)
        assert any(p.numel() == 0 for p in model.parameters())
        with engine.summon_full_params():
            assert all(p.numel() > 0 for p in model.parameters())
            with engine.summon_full_params():
                assert all(p.numel() > 0 for p in model.parameters())
            assert all(p.numel() > 0 for p in model.parameters())
        assert any(p.numel() == 0 for p in model.parameters())
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_stage3_summon_full_params_round_trip() -> None:
    _spawn(_materialization_worker, 2)


def _dropout_worker(rank: int, world: int, port: int) -> None:
    """Stage 3 recomputes each module in backward; RNG replay must reproduce dropout masks."""
    init_gloo(rank, world, port)
    try:
        cfg = _cfg(dropout=0.2)
        torch.manual_seed(99)
        m3 = LlamaForCausalLM(cfg)
        for p in m3.parameters():
            dist.broadcast(p.data, src=0)
        m0 = LlamaForCausalLM(cfg)
        m0.load_state_dict(m3.state_dict())
        hp = dict(lr=1e-3, weight_decay=0.0)
        e3 = ZeROStage3Optimizer(model=m3, **hp)
        e0 = ZeROStage0DDP(model=m0, **hp)
        for step in range(2):
            ids = _local_batch(step, rank, 2, cfg.max_seq_len, cfg.vocab_size)
            for engine, model in ((e3, m3), (e0, m0)):
                torch.manual_seed(1000 + step * 10 + rank)
                engine.zero_grad()
                engine.prepare_forward()
                model.train()
                engine.backward(model(input_ids=ids, labels=ids).loss)
                engine.step()
            with e3.summon_full_params():
                _assert_close(m3, m0, f"dropout step={step}")
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_stage3_matches_stage0_with_dropout() -> None:
    _spawn(_dropout_worker, 2)


def _checkpoint_worker(rank: int, world: int, port: int, stage: int) -> None:
    init_gloo(rank, world, port)
    try:
        cfg = _cfg()
        torch.manual_seed(5)
        hp = dict(lr=1e-3, weight_decay=0.01)

        def build():
            torch.manual_seed(5)
            m = LlamaForCausalLM(cfg)
            for p in m.parameters():
                dist.broadcast(p.data, src=0)
            return m, ENGINES[stage](model=m, **hp)

        def train_step(engine, model, step):
            ids = _local_batch(step, rank, 2, cfg.max_seq_len, cfg.vocab_size)
            engine.zero_grad()
            engine.prepare_forward()
            engine.backward(model(input_ids=ids, labels=ids).loss)
            engine.step()

        m_a, e_a = build()
        for s in range(2):
            train_step(e_a, m_a, s)
        state = e_a.state_dict()
        with _full(e_a):
            model_state = {k: v.clone() for k, v in m_a.state_dict().items()}
        m_b, e_b = build()
        with _full(e_b):
            m_b.load_state_dict(model_state)
        e_b.load_state_dict(state)
        for s in range(2, 4):
            train_step(e_a, m_a, s)
            train_step(e_b, m_b, s)
        with _full(e_a), _full(e_b):
            _assert_close(m_a, m_b, f"checkpoint stage={stage}")
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_checkpoint_restore_continues_identically(stage: int) -> None:
    _spawn(_checkpoint_worker, 2, stage)


def _memory_worker(rank: int, world: int, port: int) -> None:
    init_gloo(rank, world, port)
    try:
        cfg = _cfg()
        model = LlamaForCausalLM(cfg)
        e2 = ZeROStage2Optimizer(model=model, lr=1e-3)
        timeline = []
        e2.memory_tracker = MemoryTracker(device=torch.device("cpu"))
        e2.memory_trace_active = True
        e2.memory_state_timeline = timeline
        e2.zero_grad()
        ids = _local_batch(0, rank, 2, cfg.max_seq_len, cfg.vocab_size)
        e2.backward(model(input_ids=ids, labels=ids).loss)
        e2.step()
        labels = [t["label"] for t in timeline]
        assert labels.index("measured_step_stage2_pre_reduce_scatter") < labels.index(
            "measured_step_stage2_post_reduce_scatter"
        ) < labels.index("measured_step_stage2_pre_allgather") < labels.index("measured_step_stage2_post_allgather")
        assert all(p.grad is None for p in model.parameters())
        logical = e2.memory_state_breakdown_mb()
        live = e2.live_model_state_breakdown_mb()
        assert logical["grads_mb"] < live["grads_mb"]
        e0 = ZeROStage0DDP(model=LlamaForCausalLM(cfg), lr=1e-3)
        assert logical["optimizer_mb"] < e0.memory_state_breakdown_mb()["optimizer_mb"]
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_stage2_memory_accounting_and_trace_order() -> None:
    _spawn(_memory_worker, 2)


class _FusedStepCollectives(TorchCollectives):
    """Stands in for the NVLink kernel of the one-kernel stage-2 step with the same maths in torch."""

    supports_fused_step = True

    def __init__(self):
        self.fused_calls = 0
        self.rs_calls = 0

    def locate_symmetric(self, t):
        return ("ctx", 0)

    def reduce_scatter_accumulate_(self, acc, flat, scale):
        self.rs_calls += 1
        return super().reduce_scatter_accumulate_(acc, flat, scale)

    def allreduce_scaled_(self, flat, scale):
        self.rs_calls += 1
        return super().allreduce_scaled_(flat, scale)

    def reduce_scatter_adamw_allgather(self, params_flat, grads_flat, master, exp_avg, exp_avg_sq, grad_scale, cfg,
                                       step, dev_scalars=None, sq_out=None):
        from cs244c_llama_zero_b200.parallel.zero.optim import adamw_update_

        self.fused_calls += 1
        shard = torch.zeros(master.numel())
        self.reduce_scatter_into(shard, grads_flat)
        shard.mul_(grad_scale)
        if sq_out is not None:
            sq_out.zero_().add_(shard.pow(2).sum())
        out = torch.empty(master.numel(), dtype=params_flat.dtype)
        adamw_update_(master, exp_avg, exp_avg_sq, shard, cfg, step, param_out=out)
        self.allgather_into(params_flat, out)
        return True


def _fused_step_worker(rank: int, world: int, port: int, stage: int, grad_accum: int) -> None:
    init_gloo(rank, world, port)
    try:
        cfg = _cfg()
        torch.manual_seed(1234)
        model = LlamaForCausalLM(cfg)
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
        ref = LlamaForCausalLM(cfg)
        ref.load_state_dict(model.state_dict())
        hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
        coll = _FusedStepCollectives()
        engine = ENGINES[stage](model=model, collectives=coll, **hp)
        engine._fused_step, engine._fused_sq = True, torch.zeros(1)  # what the NVLink setup enables on GPUs
        opt = torch.optim.AdamW(ref.parameters(), **hp)
        for step in range(3):
            micro = [_local_batch(step * 10 + m, rank, 3, cfg.max_seq_len, cfg.vocab_size) for m in range(grad_accum)]
            engine.zero_grad()
            engine.prepare_forward()
            for ids in micro:
                engine.backward(model(input_ids=ids, labels=ids).loss / grad_accum)
            stats = engine.step_with_stats(max_grad_norm=0.0)
            opt.zero_grad(set_to_none=True)
            for ids in micro:
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                g = torch.cat(parts)
                (ref(input_ids=g, labels=g).loss / grad_accum).backward()
            want_norm = torch.sqrt(sum(p.grad.float().pow(2).sum() for p in ref.parameters()))
            opt.step()
            _assert_close(model, ref, f"fused stage={stage} step={step} rank={rank}")
            torch.testing.assert_close(torch.tensor(stats["grad_norm"]), want_norm, rtol=1e-4, atol=1e-6)
        assert coll.fused_calls == 3 and coll.rs_calls == 0  # one fused collective per step, whatever grad_accum
        assert engine.step_count == 3
        engine.zero_grad()
        ids = _local_batch(99, rank, 3, cfg.max_seq_len, cfg.vocab_size)
        engine.backward(model(input_ids=ids, labels=ids).loss)
        engine.step(max_grad_norm=0.5)  # clipping takes the two-kernel path
        assert coll.fused_calls == 3 and coll.rs_calls == 1 and engine.step_count == 4
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("stage,grad_accum", [(1, 1), (2, 1), (2, 2)])
def test_fused_step_plumbing_matches_reference(stage: int, grad_accum: int) -> None:
    _spawn(_fused_step_worker, 2, stage, grad_accum)


def test_stage2_on_one_rank_matches_stage0_with_grad_accum() -> None:
    """On one rank stage 2's gradient shard is the flat gradient buffer itself (no copy); training
    must equal stage 0 step for step, with several micro-batches per step."""
    cfg = _cfg()
    runs = []
    for stage in (0, 2):
        torch.manual_seed(1234)
        model = LlamaForCausalLM(cfg)
        engine = ENGINES[stage](model=model, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
        norms = []
        for step in range(3):
            engine.zero_grad()
            engine.prepare_forward()
            for m in range(2):
                ids = _local_batch(step * 10 + m, 0, 3, cfg.max_seq_len, cfg.vocab_size)
                engine.backward(model(input_ids=ids, labels=ids).loss / 2)
            norms.append(engine.step(max_grad_norm=0.5))
        runs.append((model, norms))
        if stage == 2:
            assert engine.grad_shard.data_ptr() == engine.space.grads.data_ptr()
    _assert_close(runs[0][0], runs[1][0], "stage 2 vs stage 0 on one rank")
    torch.testing.assert_close(torch.tensor(runs[1][1]), torch.tensor(runs[0][1]))


class _RoutedGradCollectives(TorchCollectives):
    """Gloo stand-in for routed stage 2: a rank cannot add into another process's memory here, so
    pushes land in a local full-size outbox and the barrier reduce-scatters it into the owners' shards
    (what the NVLink pushes + barrier produce on GPUs)."""

    supports_routed_grads = True

    def __init__(self):
        self.outbox = None
        self.shard = None
        self.pushes = 0

    def alloc(self, numel, dtype):
        self.shard = torch.zeros(numel, dtype=dtype)
        return self.shard

    def shard_bases(self, t):
        return [1000 + r for r in range(dist.get_world_size())]

    def routed_push(self, src, flat0, chunk, bases):
        world = len(bases)
        if self.outbox is None:
            self.outbox = torch.zeros(chunk * world)
        self.outbox[flat0:flat0 + src.numel()] += src
        self.pushes += 1

    def barrier(self):
        if self.outbox is not None:
            part = torch.zeros_like(self.shard)
            self.reduce_scatter_into(part, self.outbox)
            self.shard += part
            self.outbox.zero_()
        dist.barrier()


def _routed_worker(rank: int, world: int, port: int, max_grad_norm: float, grad_accum: int) -> None:
    init_gloo(rank, world, port)
    try:
        cfg = _cfg()
        torch.manual_seed(1234)
        model = LlamaForCausalLM(cfg)
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
        ref = LlamaForCausalLM(cfg)
        ref.load_state_dict(model.state_dict())
        hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
        coll = _RoutedGradCollectives()
        ZeROStage2Optimizer._routed_requested = lambda self: True  # what NVLink collectives enable on GPUs
        engine = ZeROStage2Optimizer(model=model, collectives=coll, **hp)
        assert engine._routed and engine.space.grads is None and engine.grad_shard is coll.shard
        opt = torch.optim.AdamW(ref.parameters(), **hp)
        for step in range(3):
            micro = [_local_batch(step * 10 + m, rank, 3, cfg.max_seq_len, cfg.vocab_size) for m in range(grad_accum)]
            engine.zero_grad()
            engine.prepare_forward()
            for ids in micro:
                engine.backward(model(input_ids=ids, labels=ids).loss / grad_accum)
            norm = engine.step(max_grad_norm=max_grad_norm)
            opt.zero_grad(set_to_none=True)
            for ids in micro:
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                g = torch.cat(parts)
                (ref(input_ids=g, labels=g).loss / grad_accum).backward()
            want = torch.sqrt(sum(p.grad.float().pow(2).sum() for p in ref.parameters()))
            if max_grad_norm > 0:
                torch.nn.utils.clip_grad_norm_(ref.parameters(), max_norm=max_grad_norm)
            opt.step()
            _assert_close(model, ref, f"routed step={step} rank={rank}")
            torch.testing.assert_close(torch.tensor(norm), want, rtol=1e-4, atol=1e-6)
        assert coll.pushes > 0 and engine.step_count == 3
        live = engine.live_model_state_breakdown_mb()
        assert live["grads_mb"] == pytest.approx(engine.space.chunk * 4 / 2 ** 20)  # the shard only
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("max_grad_norm,grad_accum", [(0.0, 1), (0.5, 2)])
def test_routed_stage2_matches_reference(max_grad_norm: float, grad_accum: int) -> None:
    _spawn(_routed_worker, 2, max_grad_norm, grad_accum)


class _RingCollectives(TorchCollectives):
    """Gloo stand-in for the stage-2 gradient ring: a bucket reduce all-reduces the bucket, adds this
    rank's slice of the averaged sum into its gradient segment and clears the bucket (what the NVLink
    bucket kernel produces on GPUs)."""

    supports_bucket_reduce = True

    def __init__(self):
        self.reduces = []

    def alloc(self, numel, dtype):
        return torch.zeros(numel, dtype=dtype)

    def bucket_reduce_(self, bucket, acc, scale, blocks=0):
        total = bucket.clone()
        dist.all_reduce(total)
        part = acc.numel()
        r = dist.get_rank()
        acc += scale * total[r * part:(r + 1) * part]
        bucket.zero_()
        self.reduces.append(bucket.numel())
        return True


def _ring_worker(rank: int, world: int, port: int, max_grad_norm: float, grad_accum: int) -> None:
    init_gloo(rank, world, port)
    try:
        cfg = _cfg()
        torch.manual_seed(1234)
        model = LlamaForCausalLM(cfg)
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
        ref = LlamaForCausalLM(cfg)
        ref.load_state_dict(model.state_dict())
        hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
        coll = _RingCollectives()
        ZeROStage2Optimizer._ring_requested = lambda self: True  # what NVLink collectives enable on GPUs
        engine = ZeROStage2Optimizer(model=model, collectives=coll, **hp)
        assert engine._ring and engine.space.grads is None and len(engine._ring_slots) == 2
        blocks = [b for b in engine._ring_buckets if b[4] >= 0]
        assert len(blocks) == cfg.n_layers
        opt = torch.optim.AdamW(ref.parameters(), **hp)
        for step in range(3):
            micro = [_local_batch(step * 10 + m, rank, 3, cfg.max_seq_len, cfg.vocab_size) for m in range(grad_accum)]
            engine.zero_grad()
            engine.prepare_forward()
            for ids in micro:
                engine.backward(model(input_ids=ids, labels=ids).loss / grad_accum)
            norm = engine.step(max_grad_norm=max_grad_norm)
            opt.zero_grad(set_to_none=True)
            for ids in micro:
                parts = [torch.empty_like(ids) for _ in range(world)]
                dist.all_gather(parts, ids)
                g = torch.cat(parts)
                (ref(input_ids=g, labels=g).loss / grad_accum).backward()
            want = torch.sqrt(sum(p.grad.float().pow(2).sum() for p in ref.parameters()))
            if max_grad_norm > 0:
                torch.nn.utils.clip_grad_norm_(ref.parameters(), max_norm=max_grad_norm)
            opt.step()
            _assert_close(model, ref, f"ring step={step} rank={rank}")
            torch.testing.assert_close(torch.tensor(norm), want, rtol=1e-4, atol=1e-6)
        # every bucket reduced once per backward; the buckets tile the flat space and the shard holds
        # one W-th of each
        assert len(coll.reduces) == 3 * grad_accum * len(engine._ring_buckets)
        cursor = 0
        for lo, hi, part, off, _ in engine._ring_buckets:
            assert lo == cursor and world * part >= hi - lo
            cursor = hi
        assert cursor >= engine.space.numel
        assert engine.grad_shard.numel() == sum(b[2] for b in engine._ring_buckets)
        live = engine.live_model_state_breakdown_mb()
        # the shard plus the ring's slots and edge buffers (no full gradient buffer)
        assert live["grads_mb"] == pytest.approx((engine.grad_shard.numel() * 4 + engine._ring_bytes()) / 2 ** 20)
        # checkpoint round trip: a fresh engine restored from the state continues identically
        state = engine.state_dict()
        assert state["layout"] == "ring_interleaved_v1"
        torch.manual_seed(99)
        model2 = LlamaForCausalLM(cfg)
        engine2 = ZeROStage2Optimizer(model=model2, collectives=_RingCollectives(), **hp)
        engine2.load_state_dict(state)
        for (n, a), (_, b) in zip(model.named_parameters(), model2.named_parameters()):
            assert torch.equal(a, b), n
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("max_grad_norm,grad_accum", [(0.0, 1), (0.5, 2)])
def test_ring_stage2_matches_reference(max_grad_norm: float, grad_accum: int) -> None:
    _spawn(_ring_worker, 2, max_grad_norm, grad_accum)


def test_stage2_gradient_mode_auto_policy(monkeypatch) -> None:
    """``ZB_STAGE2_GRADS=auto`` picks the gradient ring only when the full fp32 gradient buffer would
    reach the size threshold; ``ring`` / ``full`` force it; collectives without the bucket kernel
    and single-GPU runs never get it."""
    from types import SimpleNamespace

    from cs244c_llama_zero_b200.parallel.zero.common import build_flat_param_metadata

    model = LlamaForCausalLM(_cfg())
    stub = SimpleNamespace(world_size=2, device=torch.device("cuda", 0), meta=build_flat_param_metadata(model),
                           collectives=SimpleNamespace(supports_bucket_reduce=True),
                           RING_AUTO_MIN_BYTES=ZeROStage2Optimizer.RING_AUTO_MIN_BYTES)
    want = ZeROStage2Optimizer._ring_requested
    monkeypatch.delenv("ZB_STAGE2_GRADS", raising=False)
    assert not want(stub)  # a small model keeps the full buffer
    stub.RING_AUTO_MIN_BYTES = 1
    assert want(stub)
    monkeypatch.setenv("ZB_STAGE2_GRADS", "full")
    assert not want(stub)
    monkeypatch.setenv("ZB_STAGE2_GRADS", "ring")
    stub.RING_AUTO_MIN_BYTES = 1 << 60
    assert want(stub)
    stub.collectives = SimpleNamespace()
    assert not want(stub)
    stub.collectives = SimpleNamespace(supports_bucket_reduce=True)
    stub.world_size = 1
    assert not want(stub)


def _bf16_wire_worker(rank: int, world: int, port: int, stage: int) -> None:
    init_gloo(rank, world, port)
    os.environ["ZB_GRAD_COMM"] = "bf16"
    try:
        cfg = _cfg()
        torch.manual_seed(1234)
        model = LlamaForCausalLM(cfg)
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
        ref = LlamaForCausalLM(cfg)
        ref.load_state_dict(model.state_dict())
        hp = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.05)
        engine = ENGINES[stage](model=model, collectives=TorchCollectives(), **hp)
        opt = torch.optim.AdamW(ref.parameters(), **hp)
        for step in range(3):
            ids = _local_batch(step * 10, rank, 3, cfg.max_seq_len, cfg.vocab_size)
            engine.zero_grad()
            engine.prepare_forward()
            engine.backward(model(input_ids=ids, labels=ids).loss)
            engine.step(max_grad_norm=0.0)
            opt.zero_grad(set_to_none=True)
            parts = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(parts, ids)
            g = torch.cat(parts)
            ref(input_ids=g, labels=g).loss.backward()
            opt.step()
        assert engine._bf16_wire is not None and engine._bf16_wire.dtype == torch.bfloat16
        # bf16 gradients on the wire.  AdamW normalises each element's gradient, so an update differs
        # from the fp32 one by a small part of lr, except where rounding the cross-rank sum of nearly
        # cancelling contributions flips a tiny gradient's sign (at most 2 lr per step there).
        lr = hp["lr"]
        for (n, a), (_, b) in zip(model.named_parameters(), ref.named_parameters()):
            d = (a - b).abs()
            assert d.max().item() <= 3 * 2 * lr + 1e-6, (n, d.max().item())
            assert (d > 0.3 * lr).float().mean().item() <= 0.02, (n, (d > 0.3 * lr).float().mean().item())
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("stage", [0, 1, 2])
def test_bf16_gradient_wire_format(stage: int) -> None:
    """``ZB_GRAD_COMM=bf16``: gradients reduced in bf16 (the reference's dtype) train like fp32."""
    _spawn(_bf16_wire_worker, 2, stage)
