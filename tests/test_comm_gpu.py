"""NVLink/NVSwitch collective kernels vs NCCL on 2+ GPUs, and the bounded-wait error path on one GPU."""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from .dist_utils import find_free_port

pytestmark = pytest.mark.gpu


def _init(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _collectives_worker(rank: int, world: int, port: int, impl: str) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero.optim import AdamWConfig, adamw_update_

        coll = NvlinkCollectives(device=torch.device("cuda", rank), use_multicast=(impl == "nvls"))
        n = world * 4096 * 3
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        data = torch.randn(n, device="cuda", generator=g)
        chunk = n // world
        for dtype, tol in ((torch.float32, 1e-5), (torch.bfloat16, 2e-2)):
            buf = coll.alloc(n, dtype)
            src = data.to(dtype)
            ref = src.float().clone()
            dist.all_reduce(ref)
            # all-reduce with fused scale
            buf.copy_(src)
            coll.allreduce_scaled_(buf, 0.5)
            torch.testing.assert_close(buf.float(), ref * 0.5, rtol=tol, atol=tol)
            # reduce-scatter accumulated into a local fp32 shard
            buf.copy_(src)
            acc = torch.ones(chunk, device="cuda")
            coll.reduce_scatter_accumulate_(acc, buf, 0.25)
            torch.testing.assert_close(acc, 1.0 + 0.25 * ref[rank * chunk : (rank + 1) * chunk], rtol=tol, atol=tol)
        # all-gather bf16 shards in place
        pbuf = coll.alloc(n, torch.bfloat16)
        shard = (torch.arange(chunk, device="cuda", dtype=torch.float32) + 1000 * rank).to(torch.bfloat16)
        pbuf[rank * chunk : (rank + 1) * chunk].copy_(shard)
        coll.allgather_into(pbuf, pbuf[rank * chunk : (rank + 1) * chunk])
        parts = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(parts, shard)
        torch.testing.assert_close(pbuf, torch.cat(parts))
        # copy-engine pull gather: every rank's shard at the same offset of a symmetric store
        store = coll.alloc(chunk + 64, torch.bfloat16)
        store[64:].copy_(shard)
        coll.barrier()
        pulled = torch.full((n,), -1.0, device="cuda", dtype=torch.bfloat16)
        assert coll.pull_allgather_into(pulled, store[64:])
        torch.testing.assert_close(pulled, torch.cat(parts))
        coll.barrier()
        # fused AdamW + all-gather vs update + NCCL all-gather
        master = torch.randn(chunk, device="cuda", generator=g)
        m, v = torch.zeros(chunk, device="cuda"), torch.zeros(chunk, device="cuda")
        grad = torch.randn(chunk, device="cuda", generator=g)
        r_master, r_m, r_v = master.clone(), m.clone(), v.clone()
        cfg = AdamWConfig(lr=1e-3, weight_decay=0.1)
        scale = torch.tensor([0.5], device="cuda")
        assert coll.adamw_allgather(pbuf, master, m, v, grad, scale, cfg, 1)
        r_out = torch.empty(chunk, device="cuda", dtype=torch.bfloat16)
        adamw_update_(r_master, r_m, r_v, grad, cfg, 1, grad_scale=scale, param_out=r_out)
        torch.testing.assert_close(master, r_master, rtol=1e-5, atol=1e-6)
        parts = [torch.empty_like(r_out) for _ in range(world)]
        dist.all_gather(parts, r_out)
        torch.testing.assert_close(pbuf, torch.cat(parts))
        torch.cuda.synchronize()
        coll.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _need(n: int):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("impl", ["nvls", "p2p"])
def test_symmetric_collectives_match_nccl(impl):
    _need(2)
    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_collectives_worker, args=(world, find_free_port(), impl), nprocs=world, join=True)


def _engine_worker(rank: int, world: int, port: int, stage: int) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
        from cs244c_llama_zero_b200.parallel import TorchCollectives
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero import ENGINES

        cfg = ModelConfig(name="t", vocab_size=1024, max_seq_len=256, dim=256, n_layers=2, n_heads=4, n_kv_heads=2,
                          ffn_dim=512)
        models, engines = [], []
        for coll in (TorchCollectives(), NvlinkCollectives(device=torch.device("cuda", rank))):
            torch.manual_seed(0)
            model = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
            model.set_backend("b200")
            models.append(model)
            engines.append(ENGINES[stage](model=model, lr=1e-3, collectives=coll))
        ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len), device="cuda",
                            generator=torch.Generator(device="cuda").manual_seed(rank))
        for _ in range(3):
            for model, engine in zip(models, engines):
                engine.zero_grad()
                engine.prepare_forward()
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    loss = model(input_ids=ids, labels=ids, return_logits=False).loss
                engine.backward(loss)
                engine.step(max_grad_norm=1.0)
        ctx = [e.summon_full_params() if hasattr(e, "summon_full_params") else None for e in engines]
        for c in ctx:
            if c is not None:
                c.__enter__()
        for (n, a), (_, b) in zip(models[0].named_parameters(), models[1].named_parameters()):
            torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=2e-3, msg=n)
        for c in ctx:
            if c is not None:
                c.__exit__(None, None, None)
        engines[1].collectives.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_engines_with_nvlink_collectives_match_nccl(stage):
    _need(2)
    mp.spawn(_engine_worker, args=(2, find_free_port(), stage), nprocs=2, join=True)


def _timeout_worker(rank: int, world: int, port: int) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200 import ops
        from cs244c_llama_zero_b200.parallel.comm.nvlink import CommTimeoutError, NvlinkCollectives

        C = ops.load_extension()
        C.reset_device_errors()
        coll = NvlinkCollectives(device=torch.device("cuda", rank), use_multicast=False)
        buf = coll.alloc(1024, torch.float32)
        coll.buffers[0].ctx.wait_unsignalled(int(0.5e9))  # nobody signals: the wait must expire
        torch.cuda.synchronize()
        with pytest.raises(CommTimeoutError):
            coll.check_errors()
        # The context is still usable afterwards.
        C.reset_device_errors()
        buf.fill_(2.0)
        coll.allreduce_scaled_(buf, 1.0)
        torch.cuda.synchronize()
        assert float(buf[0]) == 2.0 * world
        coll.check_errors()
    finally:
        dist.destroy_process_group()


def test_bounded_wait_expires_and_reports():
    _need(1)
    mp.spawn(_timeout_worker, args=(1, find_free_port()), nprocs=1, join=True)


def _skip_signal_worker(rank: int, world: int, port: int) -> None:
    os.environ["ZB_COMM_TIMEOUT_S"] = "1"  # read when the communicator is built: expiries end within a second
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200 import ops
        from cs244c_llama_zero_b200.parallel.comm.nvlink import CommTimeoutError, NvlinkCollectives

        C = ops.load_extension()
        C.reset_device_errors()
        coll = NvlinkCollectives(device=torch.device("cuda", rank), use_multicast=False)  # plain peer loads
        buf = coll.alloc(4096, torch.float32)
        buf.fill_(1.0)
        coll.barrier()
        torch.cuda.synchronize()
        if rank == world - 1:
            coll.skip_next_collective()  # ZB_FAULT=skip_signal: this rank launches nothing, posts no signal
        coll.allreduce_scaled_(buf, 1.0)
        torch.cuda.synchronize()
        if rank == world - 1:
            coll.check_errors()  # it waited on nothing
        else:
            with pytest.raises(CommTimeoutError):
                coll.check_errors()
        C.reset_device_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_peer_that_skips_its_signal_is_detected():
    """A rank leaves its collective kernel out; the others' bounded barrier waits expire and report."""
    _need(2)
    mp.spawn(_skip_signal_worker, args=(2, find_free_port()), nprocs=2, join=True)
