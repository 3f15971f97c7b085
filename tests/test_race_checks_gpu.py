"""Race and bounds checks that need no sanitizer tool.

* Canary padding: each output is a view into a larger buffer whose other rows hold a sentinel; a
  kernel that writes outside its output (a tail tile that is not clipped, a wrong row stride) shows
  up as a changed sentinel.
* Deterministic replay: kernels whose reduction order is fixed (the GEMMs without K-split, attention
  forward, RMSNorm, embedding, the model's forward) must give bitwise-identical results when run
  twice on the same inputs; the ones that add partial results in hardware order (K-split weight
  gradients, the attention dQ reduction) must agree to rounding.  A data race shows up as a
  run-to-run difference.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

SENTINEL = 7.5
PAD = 3


@pytest.fixture(scope="module")
def C():
    from cs244c_llama_zero_b200 import ops

    ext = ops.load_extension()
    ext.reset_device_errors()
    yield ext
    assert list(ext.read_device_errors()) == [0, 0, 0, 0], "a kernel's bounded wait expired"


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


def _padded(rows, cols, dtype, fill=None):
    """A [rows, cols] contiguous view inside a buffer with PAD sentinel rows on each side."""
    big = torch.full((rows + 2 * PAD, cols), SENTINEL, device="cuda", dtype=dtype)
    view = big[PAD:PAD + rows]
    if fill is not None:
        view.fill_(fill)
    return big, view


def _canaries_intact(big):
    assert torch.all(big[:PAD] == SENTINEL), "a kernel wrote above its output"
    assert torch.all(big[-PAD:] == SENTINEL), "a kernel wrote below its output"


@pytest.mark.parametrize("M,N,K,bn", [(300, 264, 136, 128), (520, 776, 264, 192), (600, 392, 200, 1128),
                                      (1000, 768, 768, 0)])
def test_gemm_writes_stay_inside_their_outputs(C, M, N, K, bn):
    x, w = _bf(M, K, seed=1), _bf(N, K, scale=0.05, seed=2)
    big, out = _padded(M, N, torch.bfloat16)
    C.linear_fwd(x, w, out, _bf(M, N, seed=3), bn)
    _canaries_intact(big)
    dy = _bf(M, N, seed=4)
    big, dx = _padded(M, K, torch.bfloat16)
    C.linear_dgrad(dy, w, dx, 0)
    _canaries_intact(big)
    big, dw = _padded(N, K, torch.float32, fill=0.0)
    C.linear_wgrad(dy, x, dw, 0, 0)  # automatic tile and K-split: fp32 add-reductions into the view
    _canaries_intact(big)
    torch.testing.assert_close(dw, dy.float().t() @ x.float(), rtol=2e-2, atol=2e-2)


def test_norm_and_embedding_writes_stay_inside(C):
    T, d, V = 333, 768, 1000
    x, w = _bf(T, d, seed=5), _bf(d, seed=6)
    big, y = _padded(T, d, torch.bfloat16)
    C.rmsnorm_fwd(x, w, y, torch.empty(T, device="cuda"), 1e-5)
    _canaries_intact(big)
    table = _bf(V, d, seed=7)
    ids = torch.randint(0, V, (T,), device="cuda")
    big, out = _padded(T, d, torch.bfloat16)
    C.embedding_fwd(ids, table, out)
    _canaries_intact(big)
    assert torch.equal(out, table[ids])


def test_forward_kernels_replay_bitwise(C):
    from cs244c_llama_zero_b200.ops.functional import attention_forward

    M, N, K = 1000, 1280, 768
    x, w = _bf(M, K, seed=8), _bf(N, K, scale=0.05, seed=9)
    a, b = (torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    C.linear_fwd(x, w, a, None, 0)
    C.linear_fwd(x, w, b, None, 0)
    assert torch.equal(a, b)
    B, S, H, KV, hd = 4, 1024, 12, 4, 64
    qkv = _bf(B * S, (H + 2 * KV) * hd, seed=10)
    o1, l1 = attention_forward(qkv, B, S, H, KV, hd)
    o2, l2 = attention_forward(qkv, B, S, H, KV, hd)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_accumulating_kernels_replay_to_rounding(C):
    from cs244c_llama_zero_b200.ops.functional import attention_backward, attention_forward, rope_tables

    M, N, K = 4096, 768, 2048
    dy, x = _bf(M, N, seed=11), _bf(M, K, seed=12)
    runs = []
    for _ in range(2):
        dw = torch.zeros(N, K, device="cuda")
        C.linear_wgrad(dy, x, dw, 4, 0)
        runs.append(dw)
    torch.testing.assert_close(runs[0], runs[1], rtol=1e-5, atol=1e-4)
    B, S, H, KV, hd = 2, 1024, 12, 4, 64
    qkv = _bf(B * S, (H + 2 * KV) * hd, seed=13)
    out, lse = attention_forward(qkv, B, S, H, KV, hd)
    dout = _bf(B * S, H * hd, seed=14)
    cos, sin = rope_tables(S, hd, 10000.0, qkv.device)
    grads = []
    for _ in range(2):
        dqkv = torch.empty_like(qkv)
        attention_backward(qkv, out, dout, lse, B, S, H, KV, hd, dqkv, cos, sin)
        grads.append(dqkv.float())
    torch.testing.assert_close(grads[0], grads[1], rtol=2e-2, atol=2e-2)


def test_model_forward_replays_bitwise(C):
    from cs244c_llama_zero_b200.models import LlamaForCausalLM, ModelConfig

    cfg = ModelConfig(name="replay", vocab_size=1024, max_seq_len=256, dim=256, n_layers=2, n_heads=4,
                      n_kv_heads=2, ffn_dim=512, rope_theta=10000.0)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).cuda().to(torch.bfloat16)
    model.set_backend("b200")
    model.eval()
    ids = torch.randint(0, cfg.vocab_size, (2, cfg.max_seq_len), device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        a = model(input_ids=ids).logits
        b = model(input_ids=ids).logits
    assert torch.equal(a, b)
