"""Gradients routed to the ranks that own them (ZeRO-2 without a full gradient buffer).

* ``linear_wgrad_routed``: the weight-gradient GEMM with the reduce-scatter fused into its epilogue;
* ``routed_add``: the push of a finished gradient buffer into the owners' shards;
* ``embedding_bwd_routed``: the embedding backward adding its rows straight into the owners' shards;
* the B200 model's gradient sinks in routed mode against the engine's flat gradient buffer;
* on two GPUs, the routed stage-2 engine against the NCCL engine.

On one GPU the "ranks" are separate local buffers standing in for the peers' shards, which exercises
the whole routing (flat index, owner, offset inside the owner's shard, partial sums reducing in place).
"""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from .dist_utils import find_free_port

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from cs244c_llama_zero_b200 import ops

    ext = ops.load_extension()
    ext.reset_device_errors()
    yield ext
    assert list(ext.read_device_errors()) == [0, 0, 0, 0], "a kernel reported an error"


def _bf(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("T,out,inp,world,splits,bn", [(1024, 768, 512, 4, 0, 0), (520, 264, 136, 3, 2, 0),
                                                        (1024, 640, 512, 2, 1, 1128), (512, 384, 1024, 8, 0, 0)])
def test_routed_wgrad_lands_in_the_owners_shards(C, T, out, inp, world, splits, bn):
    dy, x = _bf(T, out, seed=1), _bf(T, inp, seed=2)
    flat0 = 44  # the weight starts inside the first shard, not at 0
    used = flat0 + out * inp
    chunk = ((used + 64 + world - 1) // world + 3) // 4 * 4
    shards = [torch.full((chunk,), 0.5, device="cuda") for _ in range(world)]  # earlier contents accumulate
    C.linear_wgrad_routed(dy, x, flat0, inp, chunk, [s.data_ptr() for s in shards], splits, bn)
    torch.cuda.synchronize()
    flat = torch.cat(shards) - 0.5
    got = flat[flat0:used].view(out, inp)
    ref = dy.float().t() @ x.float()
    err = (got - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err
    assert torch.count_nonzero(flat[:flat0]) == 0 and torch.count_nonzero(flat[used:]) == 0
    plain = torch.zeros(out, inp, device="cuda")
    C.linear_wgrad(dy, x, plain, splits, bn)
    torch.testing.assert_close(got, plain, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("T,out,inp,world", [(1024, 1280, 768, 4), (2048, 4096, 768, 2), (1000, 264, 392, 3)])
def test_grouped_dgrad_with_routed_wgrad(C, T, out, inp, world):
    dy, w, x = _bf(T, out, seed=5), _bf(out, inp, seed=6) * 0.05, _bf(T, inp, seed=7)
    flat0 = 64
    used = flat0 + out * inp
    chunk = ((used + world - 1) // world + 3) // 4 * 4
    shards = [torch.zeros(chunk, device="cuda") for _ in range(world)]
    dx = torch.empty(T, inp, device="cuda", dtype=torch.bfloat16)
    C.linear_dgrad_wgrad_routed(dy, w, x, dx, flat0, inp, chunk, [s.data_ptr() for s in shards])
    dx_ref = torch.empty_like(dx)
    dw_ref = torch.zeros(out, inp, device="cuda")
    C.linear_dgrad_wgrad(dy, w, x, dx_ref, dw_ref)
    torch.cuda.synchronize()
    assert torch.equal(dx, dx_ref)  # the data-gradient problem is untouched by the routing
    got = torch.cat(shards)[flat0:used].view(out, inp)
    torch.testing.assert_close(got, dw_ref, rtol=1e-4, atol=1e-3)
    assert torch.count_nonzero(torch.cat(shards)[:flat0]) == 0


def test_routed_wgrad_rejects_a_weight_outside_the_shards(C):
    dy, x = _bf(256, 128, seed=3), _bf(256, 64, seed=4)
    shard = torch.zeros(1024, device="cuda")
    with pytest.raises(RuntimeError, match="outside the sharded flat space"):
        C.linear_wgrad_routed(dy, x, 0, 64, 1024, [shard.data_ptr()], 0, 0)


def test_routed_add_pushes_into_owner_shards(C):
    world, chunk, flat0, n = 3, 4096, 1000, 9001  # a tail of 1 element after the 16-byte groups
    shards = [torch.full((chunk,), 1.0, device="cuda") for _ in range(world)]
    src = torch.randn(n, device="cuda")
    for _ in range(2):  # two pushes accumulate
        C.routed_add(src, flat0, chunk, [s.data_ptr() for s in shards])
    torch.cuda.synchronize()
    flat = torch.cat(shards) - 1.0
    torch.testing.assert_close(flat[flat0:flat0 + n], 2 * src)
    assert torch.count_nonzero(flat[:flat0]) == 0 and torch.count_nonzero(flat[flat0 + n:]) == 0
    with pytest.raises(RuntimeError, match="outside the sharded space"):
        C.routed_add(src, chunk * world - 4, chunk, [s.data_ptr() for s in shards])


def test_routed_embedding_backward(C):
    V, d, T, world = 1000, 256, 4096, 3
    ids = torch.randint(0, 50, (T,), device="cuda")  # many repeated rows: reductions must accumulate
    dy = _bf(T, d, seed=9)
    flat0 = 128
    chunk = ((flat0 + V * d + world - 1) // world + 3) // 4 * 4
    shards = [torch.zeros(chunk, device="cuda") for _ in range(world)]
    C.embedding_bwd_routed(ids, dy, V, flat0, chunk, [s.data_ptr() for s in shards])
    ref = torch.zeros(V, d, device="cuda")
    C.embedding_bwd(ids, dy, ref)
    torch.cuda.synchronize()
    got = torch.cat(shards)[flat0:flat0 + V * d].view(V, d)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-4)


def test_routed_sinks_match_the_flat_gradient_buffer(C):
    from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
    from cs244c_llama_zero_b200.parallel.zero import ZeROStage0DDP
    from cs244c_llama_zero_b200.parallel.zero.stage012 import _ShardRoute

    cfg = ModelConfig(name="t", vocab_size=1024, max_seq_len=256, dim=256, n_layers=2, n_heads=4, n_kv_heads=2,
                      ffn_dim=512)
    torch.manual_seed(0)
    ref = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
    routed = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
    routed.load_state_dict(ref.state_dict())
    for m in (ref, routed):
        m.set_backend("b200")
    engine = ZeROStage0DDP(model=ref, lr=1e-3)  # flat fp32 gradient buffer
    world = 4
    chunk = (engine.space.padded_numel + world - 1) // world
    chunk = (chunk + 3) // 4 * 4
    shards = [torch.zeros(chunk, device="cuda") for _ in range(world)]

    class LocalPeers:  # the shards are local buffers here
        def routed_push(self, src, flat0, chunk_, bases):
            C.routed_add(src, flat0, chunk_, bases)

    route = _ShardRoute(LocalPeers(), chunk, [s.data_ptr() for s in shards])
    for p, off in zip(routed.parameters(), engine.space.offsets):
        p.grad_route = (route, int(off))
    ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len), device="cuda")
    engine.zero_grad()
    for model in (ref, routed):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(input_ids=ids, labels=ids, return_logits=False).loss
        loss.backward()
    for p, off in zip(routed.parameters(), engine.space.offsets):  # any gradient autograd produced
        if p.grad is not None:
            route.push(p.grad.float().reshape(-1), int(off))
            p.grad = None
    torch.cuda.synchronize()
    got = torch.cat(shards)[: engine.space.padded_numel]
    want = engine.space.grads
    err = (got - want).abs().max().item()
    assert err <= 1e-3 * want.abs().max().item() + 1e-6, err


def _engine_worker(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig
        from cs244c_llama_zero_b200.parallel import TorchCollectives
        from cs244c_llama_zero_b200.parallel.comm.nvlink import NvlinkCollectives
        from cs244c_llama_zero_b200.parallel.zero import ZeROStage2Optimizer

        cfg = ModelConfig(name="t", vocab_size=1024, max_seq_len=256, dim=256, n_layers=2, n_heads=4, n_kv_heads=2,
                          ffn_dim=512)
        models, engines = [], []
        for routed, coll in ((False, TorchCollectives()),
                             (True, NvlinkCollectives(device=torch.device("cuda", rank), use_multicast=False))):
            os.environ["ZB_ROUTED_GRADS"] = "1" if routed else "0"
            torch.manual_seed(0)
            model = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
            model.set_backend("b200")
            models.append(model)
            engines.append(ZeROStage2Optimizer(model=model, lr=1e-3, collectives=coll))
        assert engines[1]._routed and not engines[0]._routed
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
        for (n, a), (_, b) in zip(models[0].named_parameters(), models[1].named_parameters()):
            torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=2e-3, msg=n)
        engines[1].collectives.check_errors()
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_routed_stage2_trains_like_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_engine_worker, args=(2, find_free_port()), nprocs=2, join=True)
