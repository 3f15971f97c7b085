"""ZeRO-2 gradient ring (the default stage-2 gradient path with the NVLink collectives).

* ``bucket_reduce_``: one bucket of every rank's gradient, each rank's slice of the sum accumulated
  into its gradient segment, the bucket cleared afterwards, accumulation over two calls;
* ``adamw_allgather_segments``: AdamW on an interleaved shard against the formula, and the bf16
  all-gather writing exactly the valid part of every slice; multicast and peer loads for both;
* the push reduce-scatter (peer stores into a landing area, several pieces per call) against NCCL,
  and the push variant of the bucket reduce;
* the stage-2 engine in ring mode (no full gradient buffer) against the NCCL engine with its full
  buffer, with clipping and two micro-batches per step, with switch and push reductions.

Both run as two processes on two GPUs.
"""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from .dist_utils import find_free_port

pytestmark = pytest.mark.gpu


def _init(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _bucket_worker(rank: int, world: int, port: int) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200 import ops
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero.optim import AdamWConfig

        ops.load_extension().reset_device_errors()
        dev = torch.device("cuda", rank)
        for multicast in (True, False):
            coll = NvlinkCollectives(device=dev, use_multicast=multicast)
            # bucket reduce: rank r's slice of the summed bucket into its segment, bucket cleared
            bucket_buf = coll.alloc(8000, torch.float32)
            for part in (1000, 2052, 4):
                bucket = bucket_buf[: world * part]
                acc = torch.full((part,), 0.5, device=dev)
                contrib = []
                for r in range(world):
                    g = torch.Generator(device="cuda").manual_seed(100 * r + part)
                    contrib.append(torch.randn(world * part, device=dev, generator=g))
                for _ in range(2):  # two reductions accumulate
                    bucket.copy_(contrib[rank])
                    assert coll.bucket_reduce_(bucket, acc, 0.5)
                torch.cuda.synchronize()
                assert torch.count_nonzero(bucket_buf) == 0, "the bucket is cleared on every rank"
                want = 0.5 + torch.stack(contrib).sum(0)[rank * part:(rank + 1) * part]  # 2 calls x 0.5
                torch.testing.assert_close(acc, want, rtol=1e-5, atol=1e-5, msg=f"mc={multicast} part={part}")
            assert not coll.bucket_reduce_(torch.zeros(16, device=dev), torch.zeros(8, device=dev), 1.0)

            # AdamW on an interleaved shard + all-gather of the valid part of every slice
            buckets = [(0, 1000), (1000, 3056)]  # flat ranges; slices of 504 and 1032 at W = 2
            params = coll.alloc(4096, torch.bfloat16)
            params.fill_(7.0)  # sentinel: nothing past the buckets is written
            rows, shard_off, parts = [], 0, []
            for lo, hi in buckets:
                part = -(-(hi - lo) // (8 * world)) * 8
                valid = max(0, min(part, (hi - lo) - rank * part))
                rows.append((shard_off // 8, part // 8, valid // 8, lo * 2))
                parts.append((lo, hi, part, shard_off))
                shard_off += part
            segs = torch.tensor(rows, dtype=torch.int64, device=dev)
            cfg = AdamWConfig(lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)

            def state(r):
                g = torch.Generator(device="cuda").manual_seed(7 + r)
                return (torch.randn(shard_off, device=dev, generator=g),
                        torch.randn(shard_off, device=dev, generator=g))

            master, grad = state(rank)
            m, v = torch.zeros_like(master), torch.zeros_like(master)
            scale = torch.tensor([0.25], device=dev)
            assert coll.adamw_allgather_segments(params, segs, master, m, v, grad, scale, cfg, 1)
            torch.cuda.synchronize()
            expect = torch.full((4096,), 7.0, device=dev)
            for r in range(world):
                w0, g0 = state(r)
                g0 = g0 * 0.25
                m0, v0 = 0.1 * g0, 0.05 * g0 * g0
                new = w0 * (1 - cfg.lr * cfg.weight_decay) - (cfg.lr / 0.1) * m0 / (v0.sqrt() / 0.05 ** 0.5 + cfg.eps)
                if r == rank:
                    torch.testing.assert_close(master, new, rtol=1e-5, atol=1e-6)
                for lo, hi, part, off in parts:
                    valid = max(0, min(part, (hi - lo) - r * part))
                    expect[lo + r * part:lo + r * part + valid] = new[off:off + valid]
            torch.testing.assert_close(params.float(), expect.to(torch.bfloat16).float(), rtol=0, atol=0)
            coll.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_bucket_reduce_and_segmented_adamw():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_bucket_worker, args=(2, find_free_port()), nprocs=2, join=True)


def _push_worker(rank: int, world: int, port: int) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200 import ops
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives

        ops.load_extension().reset_device_errors()
        os.environ["ZB_RS_MODE"] = "push"
        dev = torch.device("cuda", rank)
        for multicast in (True, False):
            coll = NvlinkCollectives(device=dev, use_multicast=multicast)
            assert coll.rs_push()
            coll.LANDING_MAX_BYTES = 4096 * 4 * world  # several pieces per call
            for n in (8 * world * 1000, 8 * world * 7):
                g = torch.Generator(device="cuda").manual_seed(rank + n)
                flat = torch.randn(n, device=dev, generator=g)  # ordinary (not symmetric) memory
                keep = flat.clone()
                part = n // world
                acc = torch.full((part,), 0.25, device=dev)
                coll.reduce_scatter_accumulate_(acc, flat, 0.5)
                ref = flat.clone()
                dist.all_reduce(ref)
                torch.testing.assert_close(acc, 0.25 + 0.5 * ref[rank * part:(rank + 1) * part], rtol=1e-5, atol=1e-5)
                assert torch.equal(flat, keep)  # the source is left as it was
            bucket = coll.alloc(world * 2000, torch.float32)
            g = torch.Generator(device="cuda").manual_seed(50 + rank)
            data = torch.randn(world * 2000, device=dev, generator=g)
            bucket.copy_(data)
            acc = torch.zeros(2000, device=dev)
            assert coll.bucket_reduce_(bucket, acc, 1.0)
            ref = data.clone()
            dist.all_reduce(ref)
            torch.testing.assert_close(acc, ref[rank * 2000:(rank + 1) * 2000], rtol=1e-5, atol=1e-5)
            torch.cuda.synchronize()
            assert torch.count_nonzero(bucket) == 0  # cleared by the push kernel
            coll.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_push_reduce_scatter():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_push_worker, args=(2, find_free_port()), nprocs=2, join=True)


def _engine_worker(rank: int, world: int, port: int, slots: str, rs_mode: str) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
        from cs244c_llama_zero_b200.parallel import TorchCollectives
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero import ZeROStage2Optimizer

        os.environ["ZB_STAGE2_RING_SLOTS"] = slots
        os.environ["ZB_RS_MODE"] = rs_mode
        os.environ["ZB_STAGE2_GRADS"] = "ring"  # "auto" keeps the full buffer for a model this small
        cfg = ModelConfig(name="t", vocab_size=1024, max_seq_len=256, dim=256, n_layers=3, n_heads=4, n_kv_heads=2,
                          ffn_dim=512)
        dev = torch.device("cuda", rank)
        models, engines = [], []
        for coll in (TorchCollectives(), NvlinkCollectives(device=dev)):
            torch.manual_seed(0)
            model = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
            model.set_backend("b200")
            models.append(model)
            engines.append(ZeROStage2Optimizer(model=model, lr=1e-3, collectives=coll))
        ring = engines[1]
        assert ring._ring and ring.space.grads is None and not engines[0]._ring
        assert len(ring._ring_slots) == int(slots)
        full_mb = ring.space.padded_numel * 4 / 2**20
        assert ring.debug_memory_components_mb()["live_flat_grad_buffer_mb"] < full_mb
        gens = torch.Generator(device="cuda").manual_seed(rank)
        batches = [torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len), device=dev, generator=gens)
                   for _ in range(4)]
        for step, micro in enumerate(([batches[0]], [batches[1], batches[2]], [batches[3]])):
            for model, engine in zip(models, engines):
                engine.zero_grad()
                for ids in micro:
                    engine.prepare_forward()
                    with torch.autocast("cuda", dtype=torch.bfloat16):
                        loss = model(input_ids=ids, labels=ids, return_logits=False).loss
                    engine.backward(loss / len(micro))
                engine.step(max_grad_norm=1.0 if step != 2 else 0.0)
        norms = []
        for shard in (engines[0].grad_shard, ring.grad_shard):  # contiguous vs interleaved shards
            sq = shard.float().pow(2).sum()
            dist.all_reduce(sq)
            norms.append(sq.sqrt().item())
        assert abs(norms[1] - norms[0]) <= 2e-2 * norms[0], norms  # the last step's averaged gradient
        for (n, a), (_, b) in zip(models[0].named_parameters(), models[1].named_parameters()):
            torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=2e-3, msg=n)
        ring.collectives.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("slots,rs_mode", [("2", "switch"), ("1", "switch"), ("2", "push")])
def test_ring_stage2_trains_like_nccl(slots, rs_mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_engine_worker, args=(2, find_free_port(), slots, rs_mode), nprocs=2, join=True)
