"""The one-kernel unclipped ZeRO-1/2 step (``rs_adamw_allgather``): reduce-scatter of the flat fp32
gradients, squared norm, AdamW and bf16 all-gather in one launch.

* one GPU (a world of one rank, plain peer loads): the kernel against the step written out in
  fp32 PyTorch;
* two GPUs: the stage-1 and stage-2 engines with ``ZB_FUSED_STEP=1`` train like the NCCL engines.
"""

from __future__ import annotations

import math
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from .dist_utils import find_free_port

pytestmark = pytest.mark.gpu


def _need(n: int) -> None:
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _init(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _kernel_worker(rank: int, world: int, port: int) -> None:
    _init(rank, world, port)
    try:
        from cs244c_llama_zero_b200 import ops
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero.optim import AdamWConfig

        ops.load_extension().reset_device_errors()
        coll = NvlinkCollectives(device=torch.device("cuda", rank), use_multicast=False)
        chunk = 4096 + 8 * 37
        params = coll.alloc(chunk, torch.bfloat16)
        grads = coll.alloc(chunk, torch.float32)
        g = torch.Generator(device="cuda").manual_seed(7)
        grads.copy_(torch.randn(chunk, device="cuda", generator=g))
        master = torch.randn(chunk, device="cuda", generator=g)
        m = torch.randn(chunk, device="cuda", generator=g) * 0.1
        v = torch.rand(chunk, device="cuda", generator=g) * 0.01
        ref = [t.clone() for t in (master, m, v)]
        cfg = AdamWConfig(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
        sq = torch.full((1,), 123.0, device="cuda")  # the launcher zeroes it first
        step, scale = 4, 0.5
        assert coll.reduce_scatter_adamw_allgather(params, grads, master, m, v, scale, cfg, step, None, sq)
        torch.cuda.synchronize()
        gg = grads * scale
        pm, mm, vv = ref
        mm.mul_(0.9).add_(gg, alpha=0.1)
        vv.mul_(0.95).addcmul_(gg, gg, value=0.05)
        pm.mul_(1 - cfg.lr * cfg.weight_decay)
        pm.addcdiv_(mm, vv.sqrt() / math.sqrt(1 - 0.95 ** step) + cfg.eps, value=-cfg.lr / (1 - 0.9 ** step))
        torch.testing.assert_close(master, pm, atol=1e-6, rtol=1e-5)
        torch.testing.assert_close(m, mm, atol=1e-7, rtol=1e-6)
        torch.testing.assert_close(v, vv, atol=1e-7, rtol=1e-6)
        torch.testing.assert_close(params, pm.to(torch.bfloat16))
        torch.testing.assert_close(sq[0], gg.double().pow(2).sum().float(), rtol=1e-4, atol=1e-3)
        coll.check_errors()
    finally:
        dist.destroy_process_group()


def test_fused_step_kernel_matches_fp32_reference():
    _need(1)
    mp.spawn(_kernel_worker, args=(1, find_free_port()), nprocs=1, join=True)


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
        for fused, coll in ((False, TorchCollectives()),
                            (True, NvlinkCollectives(device=torch.device("cuda", rank), use_multicast=False))):
            os.environ["ZB_FUSED_STEP"] = "1" if fused else "0"
            torch.manual_seed(0)
            model = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
            model.set_backend("b200")
            models.append(model)
            engines.append(ENGINES[stage](model=model, lr=1e-3, collectives=coll))
        assert engines[1]._fused_step and not engines[0]._fused_step
        ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len), device="cuda",
                            generator=torch.Generator(device="cuda").manual_seed(rank))
        norms = [[], []]
        for _ in range(3):
            for k, (model, engine) in enumerate(zip(models, engines)):
                engine.zero_grad()
                engine.prepare_forward()
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    loss = model(input_ids=ids, labels=ids, return_logits=False).loss
                engine.backward(loss)
                norms[k].append(engine.step(max_grad_norm=0.0))
        for (n, a), (_, b) in zip(models[0].named_parameters(), models[1].named_parameters()):
            torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=2e-3, msg=n)
        torch.testing.assert_close(torch.tensor(norms[1]), torch.tensor(norms[0]), rtol=2e-2, atol=1e-4)
        engines[1].collectives.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("stage", [1, 2])
def test_fused_step_trains_like_nccl(stage):
    _need(2)
    mp.spawn(_engine_worker, args=(2, find_free_port(), stage), nprocs=2, join=True)
