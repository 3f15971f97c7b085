"""Weight-gradient GEMM with the reduce-scatter fused into its epilogue (``linear_wgrad_routed``).

Each fp32 partial sum goes straight to the shard of the rank that owns that element of the flat
gradient space.  On one GPU the "ranks" are separate local buffers standing in for the peers' shards,
which exercises the whole routing (flat index, owner, offset inside the owner's shard, K-split partial
sums reducing in place) against the plain weight-gradient GEMM and an fp32 reference.
"""

from __future__ import annotations

import pytest
import torch

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


def test_routed_wgrad_rejects_a_weight_outside_the_shards(C):
    dy, x = _bf(256, 128, seed=3), _bf(256, 64, seed=4)
    shard = torch.zeros(1024, device="cuda")
    with pytest.raises(RuntimeError, match="outside the sharded flat space"):
        C.linear_wgrad_routed(dy, x, 0, 64, 1024, [shard.data_ptr()], 0, 0)
