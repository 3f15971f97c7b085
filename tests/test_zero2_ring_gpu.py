"""ZeRO-2 gradient ring (the default stage-2 gradient path with the NVLink collectives).

* ``bucket_reduce_to_owners_``: one bucket of every rank's gradient, reduced into the owners' fp32
  shards (1/W of the bucket per rank, or each rank its own part), the bucket cleared afterwards, a
  bucket that straddles a shard boundary, accumulation over two calls; multicast and peer loads;
* the stage-2 engine in ring mode (no full gradient buffer) against the NCCL engine with its full
  buffer, with clipping and two micro-batches per step.

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

        ops.load_extension().reset_device_errors()
        dev = torch.device("cuda", rank)
        chunk = 8192
        for multicast in (True, False):
            coll = NvlinkCollectives(device=dev, use_multicast=multicast)
            shard = coll.alloc(chunk, torch.float32)
            bases = coll.shard_bases(shard)
            bucket_buf = coll.alloc(6000, torch.float32)
            for balanced in (True, False):
                for flat0, n in ((chunk - 1000, 4000), (64, 2052), (chunk + 16, 5000)):
                    shard.fill_(0.5)
                    bucket = bucket_buf[:n]
                    contrib = []
                    for r in range(world):
                        g = torch.Generator(device="cuda").manual_seed(100 * r + n)
                        contrib.append(torch.randn(n, device=dev, generator=g))
                    for _ in range(2):  # two reductions accumulate
                        bucket.copy_(contrib[rank])
                        assert coll.bucket_reduce_to_owners_(bucket, flat0, chunk, bases, 0.5, balanced)
                    torch.cuda.synchronize()
                    assert torch.count_nonzero(bucket_buf) == 0, "the bucket is cleared on every rank"
                    total = torch.stack(contrib).sum(0)  # every rank holds every contribution
                    flat = torch.full((chunk * world,), 0.5, device=dev)
                    flat[flat0:flat0 + n] += total  # 2 calls x scale 0.5
                    want = flat[rank * chunk:(rank + 1) * chunk]
                    torch.testing.assert_close(shard, want, rtol=1e-5, atol=1e-5,
                                               msg=f"mc={multicast} balanced={balanced} flat0={flat0}")
            # a bucket that is not in a symmetric buffer is declined
            assert not coll.bucket_reduce_to_owners_(torch.zeros(16, device=dev), 0, chunk, bases, 1.0)
            coll.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_bucket_reduce_to_owners():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_bucket_worker, args=(2, find_free_port()), nprocs=2, join=True)


def _engine_worker(rank: int, world: int, port: int, split: str) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
        from cs244c_llama_zero_b200.parallel import TorchCollectives
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero import ZeROStage2Optimizer

        os.environ["ZB_STAGE2_RING_SPLIT"] = split
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
        diff = (ring.grad_shard - engines[0].grad_shard).norm() / engines[0].grad_shard.norm()
        assert diff.item() < 2e-2, diff.item()  # the last step's averaged gradient shard
        for (n, a), (_, b) in zip(models[0].named_parameters(), models[1].named_parameters()):
            torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=2e-3, msg=n)
        ring.collectives.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("split", ["balanced", "owner"])
def test_ring_stage2_trains_like_nccl(split):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_engine_worker, args=(2, find_free_port(), split), nprocs=2, join=True)
