"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op."""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


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


def _close(a, b, tol):
    """Max-abs error within ``tol`` of the reference's largest magnitude, and every row within 4 * tol
    of its own magnitude (floored at 1e-3 of the global scale), so a wrong tail row or a wrong block of
    columns in one row cannot hide under the global scale."""
    a32, b32 = a.float(), b.float()
    diff = (a32 - b32).abs()
    err = diff.max().item()
    ref = b32.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max abs err {err:.4g} vs ref scale {ref:.4g}"
    if b32.dim() >= 2 and b32.shape[-1] > 1:
        rows_ref = b32.reshape(-1, b32.shape[-1]).abs().amax(dim=1) + 1e-3 * ref
        rows_err = diff.reshape(-1, b32.shape[-1]).amax(dim=1)
        worst = (rows_err / rows_ref).max().item()
        assert worst <= 4 * tol, f"worst per-row relative error {worst:.4g} (row {(rows_err / rows_ref).argmax().item()})"


@pytest.mark.parametrize("M,N,K,bn", [(256, 512, 128, 256), (300, 264, 136, 128), (1024, 1280, 768, 256),
                                      (128, 768, 2048, 256), (520, 776, 264, 192), (1024, 768, 768, 0),
                                      (512, 512, 256, 1256), (600, 392, 200, 1128), (384, 776, 264, 1192)])
def test_linear_fwd(C, M, N, K, bn):
    """bn >= 1000 requests a CTA-pair (cta_group::2) tile of width bn - 1000; 0 = automatic choice."""
    x, w = _bf(M, K, seed=1), _bf(N, K, scale=0.05, seed=2)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.linear_fwd(x, w, out, None, bn)
    _close(out, x.float() @ w.float().t(), 2e-2)
    res = _bf(M, N, seed=3)
    C.linear_fwd(x, w, out, res, bn)
    _close(out, res.float() + x.float() @ w.float().t(), 2e-2)


@pytest.mark.parametrize("M,N,K,bn", [(256, 768, 512, 0), (200, 136, 264, 0), (1024, 768, 2048, 0),
                                      (384, 512, 776, 192), (256, 640, 384, 128), (600, 256, 392, 1128),
                                      (512, 384, 1024, 1256)])
def test_linear_dgrad(C, M, N, K, bn):
    dy, w = _bf(M, N, seed=4), _bf(N, K, scale=0.05, seed=5)
    dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    C.linear_dgrad(dy, w, dx, bn)
    _close(dx, dy.float() @ w.float(), 2e-2)


@pytest.mark.parametrize("M,N,K,splits,bn", [(512, 384, 256, 1, 0), (1024, 768, 1280, 4, 0), (300, 136, 200, 0, 0),
                                             (4096, 1280, 768, 0, 0), (1024, 384, 776, 3, 192),
                                             (1024, 640, 512, 2, 1128), (512, 384, 1024, 1, 1256)])
def test_linear_wgrad_accumulates(C, M, N, K, splits, bn):
    dy, x = _bf(M, N, seed=6), _bf(M, K, seed=7)
    dw = torch.ones(N, K, device="cuda", dtype=torch.float32)
    C.linear_wgrad(dy, x, dw, splits, bn)
    _close(dw, 1.0 + dy.float().t() @ x.float(), 1e-2)


@pytest.mark.parametrize("T,out,inp,splits", [(1024, 768, 768, 0), (4096, 4096, 768, 0), (1000, 264, 392, 0),
                                               (2048, 4000, 768, 3), (8192, 1280, 768, 0)])
def test_grouped_dgrad_wgrad(C, T, out, inp, splits):
    """One launch computing dx = dy @ w and dw += dy^T @ x (both problems' tiles dealt together)."""
    dy, w, x = _bf(T, out, seed=31), _bf(out, inp, scale=0.05, seed=32), _bf(T, inp, seed=33)
    dx = torch.full((T, inp), 7.0, device="cuda", dtype=torch.bfloat16)
    dw = torch.ones(out, inp, device="cuda", dtype=torch.float32)
    C.linear_dgrad_wgrad(dy, w, x, dx, dw, splits)
    _close(dx, dy.float() @ w.float(), 2e-2)
    _close(dw, 1.0 + dy.float().t() @ x.float(), 1e-2)


def _rope_ref(t, S, hd, theta):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device="cuda").float() / hd))
    ang = torch.outer(torch.arange(S, device="cuda").float(), inv)
    cos, sin = torch.cat([ang.cos()] * 2, -1), torch.cat([ang.sin()] * 2, -1)
    B = t.shape[0] // S
    tt = t.view(B, S, -1, hd)
    rot = torch.cat([-tt[..., hd // 2:], tt[..., : hd // 2]], -1)
    return (tt * cos[None, :, None] + rot * sin[None, :, None]).view_as(t)


@pytest.mark.parametrize("hd,H,KV", [(64, 4, 2), (128, 4, 2)])
def test_qkv_rope_epilogue(C, hd, H, KV):
    from cs244c_llama_zero_b200.ops.functional import rope_tables, rope_tables_t

    B, S, d = 2, 256, 256
    x, w = _bf(B * S, d, seed=8), _bf((H + 2 * KV) * hd, d, scale=0.05, seed=9)
    cos, sin = rope_tables(S, hd, 10000.0, x.device)
    cos_t, sin_t = rope_tables_t(S, hd, 10000.0, x.device)  # the epilogue's frequency-major layout
    out = torch.empty(B * S, (H + 2 * KV) * hd, device="cuda", dtype=torch.bfloat16)
    C.qkv_rope_fwd(x, w, out, cos_t, sin_t, S, hd, (H + KV) * hd)
    full = x.float() @ w.float().t()
    qk = full[:, : (H + KV) * hd]
    ref = torch.cat([_rope_ref(qk.contiguous(), S, hd, 10000.0), full[:, (H + KV) * hd:]], 1)
    _close(out, ref, 2e-2)
    # RoPE backward kernel = exact inverse rotation
    g = out.clone()
    C.rope_bwd(g, (H + KV) * hd, hd, S, cos, sin)
    _close(g, full, 3e-2)


def test_swiglu_forward_and_backward_epilogues(C):
    M, d, ffn = 384, 256, 512
    x, w_gu, w_down = _bf(M, d, seed=10), _bf(2 * ffn, d, scale=0.05, seed=11), _bf(d, ffn, scale=0.05, seed=12)
    h = torch.empty(M, ffn, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * ffn, device="cuda", dtype=torch.bfloat16)
    C.swiglu_fwd(x, w_gu, h, gu)
    g_ref = x.float() @ w_gu[:ffn].float().t()
    u_ref = x.float() @ w_gu[ffn:].float().t()
    _close(gu[:, :ffn], g_ref, 2e-2)
    _close(gu[:, ffn:], u_ref, 2e-2)
    _close(h, F.silu(g_ref) * u_ref, 3e-2)
    dy = _bf(M, d, seed=13)
    dgu = torch.empty_like(gu)
    C.swiglu_dgrad(dy, w_down, gu, dgu)
    g, u = gu[:, :ffn].float(), gu[:, ffn:].float()
    da = dy.float() @ w_down.float()
    sig = torch.sigmoid(g)
    _close(dgu[:, :ffn], da * u * sig * (1 + g * (1 - sig)), 3e-2)
    _close(dgu[:, ffn:], da * g * sig, 3e-2)


@pytest.mark.parametrize("d,with_res", [(256, True), (768, True), (2048, True), (3080, True), (4096, True),
                                        (4096, False)])
def test_rmsnorm(C, d, with_res):
    T = 333
    x, w = _bf(T, d, seed=14), (1 + 0.1 * _bf(d, seed=15).float()).to(torch.bfloat16)
    y = torch.empty_like(x)
    rstd = torch.empty(T, device="cuda")
    C.rmsnorm_fwd(x, w, y, rstd, 1e-5)
    xf = x.float().requires_grad_()
    wf = w.float().requires_grad_()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * wf
    _close(y, ref, 1e-2)
    dy, dres = _bf(T, d, seed=16), (_bf(T, d, seed=17) if with_res else None)
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dw = torch.zeros(d, device="cuda")
    C.rmsnorm_bwd(dy, x, w, rstd, dres, dx, dw)  # d > 2048: the wide-row kernel
    _close(dx, xf.grad + (dres.float() if with_res else 0.0), 2e-2)
    _close(dw, wf.grad, 1e-2)


def test_embedding(C):
    V, d, T = 1000, 256, 777
    table = _bf(V, d, seed=18)
    ids = torch.randint(0, V, (T,), device="cuda")
    out = torch.empty(T, d, device="cuda", dtype=torch.bfloat16)
    C.embedding_fwd(ids, table, out)
    assert torch.equal(out, table[ids])
    dy = _bf(T, d, seed=19)
    dt = torch.zeros(V, d, device="cuda")
    C.embedding_bwd(ids, dy, dt)
    ref = torch.zeros(V, d, device="cuda").index_add_(0, ids, dy.float())
    _close(dt, ref, 1e-5)


def test_embedding_out_of_range_id_is_recorded_not_read(C):
    from cs244c_llama_zero_b200 import ops

    V, d, T = 64, 128, 16
    table = _bf(V, d, seed=21)
    ids = torch.randint(0, V, (T,), device="cuda")
    ids[5] = V + 3  # a bad token id: the row is skipped (zeros) and the error record names it
    out = torch.full((T, d), 7.0, device="cuda", dtype=torch.bfloat16)
    C.reset_device_errors()
    C.embedding_fwd(ids, table, out)
    torch.cuda.synchronize()
    code, where, _, _ = C.read_device_errors()
    C.reset_device_errors()
    assert (code, where) == (6, 5)
    assert torch.equal(out[5], torch.zeros(d, device="cuda", dtype=torch.bfloat16))
    keep = torch.arange(T, device="cuda") != 5
    assert torch.equal(out[keep], table[ids[keep]])
    with pytest.raises(ops.DeviceWaitError, match="index out of range"):
        ops.raise_for_device_errors([code, where, 0, 1])


def test_adamw_matches_reference_math(C):
    n = 10_003
    g = torch.Generator(device="cuda").manual_seed(20)
    master = torch.randn(n, device="cuda", generator=g)
    m, v = torch.randn(n, device="cuda", generator=g) * 0.1, torch.rand(n, device="cuda", generator=g) * 0.01
    grad = torch.randn(n, device="cuda", generator=g)
    ref = [t.clone() for t in (master, m, v)]
    out = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    scale = torch.tensor([0.5], device="cuda")
    lr, b1, b2, eps, wd, step = 1e-3, 0.9, 0.95, 1e-8, 0.1, 3
    C.adamw(master, m, v, grad, out, scale, 1.0, lr, b1, b2, eps, wd, step)
    pm, mm, vv = ref
    gg = grad * 0.5
    mm.mul_(b1).add_(gg, alpha=1 - b1)
    vv.mul_(b2).addcmul_(gg, gg, value=1 - b2)
    pm.mul_(1 - lr * wd)
    denom = vv.sqrt() / math.sqrt(1 - b2 ** step) + eps
    pm.addcdiv_(mm, denom, value=-lr / (1 - b1 ** step))
    torch.testing.assert_close(master, pm, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(m, mm, atol=1e-7, rtol=1e-6)
    torch.testing.assert_close(v, vv, atol=1e-7, rtol=1e-6)
    torch.testing.assert_close(out.float(), pm, atol=1e-2, rtol=1e-2)


def test_adamw_device_step_matches_host_step(C):
    """The device step counter (CUDA-graph mode) gives the host step's bias corrections."""
    n = 4096
    g = torch.Generator(device="cuda").manual_seed(24)
    state = [torch.randn(n, device="cuda", generator=g) for _ in range(2)] + [torch.rand(n, device="cuda", generator=g)]
    grad = torch.randn(n, device="cuda", generator=g)
    a, b = [t.clone() for t in state], [t.clone() for t in state]
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.95, 1e-8, 0.1
    step_t = torch.tensor([4], dtype=torch.int32, device="cuda")
    sc = torch.zeros(2, device="cuda")
    C.adam_advance(step_t, sc, lr, b1, b2)
    assert int(step_t.item()) == 5
    torch.testing.assert_close(sc.cpu(), torch.tensor([lr / (1 - b1 ** 5), 1 / math.sqrt(1 - b2 ** 5)]), rtol=1e-5,
                               atol=0.0)
    C.adamw(*a, grad, None, None, 1.0, lr, b1, b2, eps, wd, 5)
    C.adamw(*b, grad, None, None, 1.0, lr, b1, b2, eps, wd, 999, sc)  # the host step is ignored
    for x, y in zip(a, b):  # same scalars to the bit (double, rounded once), so the same update bits
        assert torch.equal(x, y)


def test_sum_squares(C):
    x = torch.randn(1_000_001, device="cuda")
    out = torch.empty(1, device="cuda")
    C.sum_squares(x, out)
    torch.testing.assert_close(out[0], (x.double() ** 2).sum().float(), rtol=1e-4, atol=1e-3)


def test_cross_entropy(C):
    T, V = 300, 4000
    logits = _bf(T, V, scale=2.0, seed=21)
    targets = torch.randint(0, V, (T,), device="cuda")
    targets[::7] = -100
    lse = torch.empty(T, device="cuda")
    scratch = torch.empty(3, device="cuda")
    C.cross_entropy_fwd(logits, targets, lse, scratch[0:1], scratch[1:2], scratch[2:3])
    lf = logits.float().requires_grad_()
    ref = F.cross_entropy(lf, targets, ignore_index=-100)
    torch.testing.assert_close(scratch[2], ref.detach(), rtol=1e-4, atol=1e-4)
    ref.backward()
    g = torch.tensor([1.0], device="cuda")
    work = logits.clone()
    C.cross_entropy_bwd(work, targets, lse, g, scratch[1:2])
    _close(work, lf.grad, 1e-2)


def _lm_head_case(seed: int):
    B, S, d, V = 2, 512, 256, 1024
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(B, S, d, device="cuda", generator=g) * 0.5).to(torch.bfloat16).requires_grad_()
    w = torch.nn.Parameter((torch.randn(V, d, device="cuda", generator=g) * 0.05).to(torch.bfloat16))
    labels = torch.randint(0, V, (B, S), device="cuda", generator=g)
    labels[0, ::5] = -100
    return x, w, labels


def _lm_head_reference(x, w, labels, scale):
    xf = x.detach().float().requires_grad_()
    wf = w.detach().float().requires_grad_()
    logits = xf @ wf.t()
    loss = F.cross_entropy(logits[:, :-1].reshape(-1, w.shape[0]), labels[:, 1:].reshape(-1), ignore_index=-100)
    (loss * scale).backward()
    return loss.detach(), xf.grad, wf.grad


def test_lm_head_gradients_in_forward_match_fp32_and_the_logits_path(C, monkeypatch):
    """With the loss-gradient scale announced, the LM head + cross-entropy computes dx and dW during the
    forward pass in blocks of rows (no [T, V] logits tensor); loss and both gradients must match fp32
    PyTorch and the path that keeps the logits for backward."""
    from cs244c_llama_zero_b200.ops import functional as B

    monkeypatch.setenv("ZB_LM_BLOCK_MB", "1")  # 512-row blocks: two blocks for 1024 tokens
    scale = 0.5
    x, w, labels = _lm_head_case(31)
    loss_ref, dx_ref, dw_ref = _lm_head_reference(x, w, labels, scale)
    w.main_grad = torch.zeros(w.shape, dtype=torch.float32, device="cuda")  # the flat-buffer sink
    s_t = torch.full((), scale, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    before = torch.cuda.memory_allocated()
    with B.loss_gradient_scale(s_t):
        loss = B.lm_head_cross_entropy(x, w, labels)
    # one 512-row block of logits (1 MB) and dx (0.5 MB) live, never the 2 MB of [T, V] logits
    assert torch.cuda.max_memory_allocated() - before < 1024 * 1024 * 2
    (loss * scale).backward()
    torch.testing.assert_close(loss.detach(), loss_ref, rtol=2e-3, atol=2e-3)
    _close(x.grad, dx_ref, 2e-2)
    _close(w.main_grad, dw_ref, 2e-2)
    assert list(C.read_device_errors()) == [0, 0, 0, 0]
    # the logits-keeping path (no scale announced) gives the same gradients
    x2, w2, _ = _lm_head_case(31)
    w2.main_grad = torch.zeros(w2.shape, dtype=torch.float32, device="cuda")
    loss2 = B.lm_head_cross_entropy(x2, w2, labels)
    (loss2 * scale).backward()
    torch.testing.assert_close(loss2.detach(), loss.detach(), rtol=1e-4, atol=1e-4)
    _close(x.grad, x2.grad, 1e-2)
    _close(w.main_grad, w2.main_grad, 1e-2)


def test_lm_head_gradients_in_forward_flag_a_wrong_backward_scale(C, monkeypatch):
    from cs244c_llama_zero_b200.ops import functional as B

    monkeypatch.setenv("ZB_LM_BLOCK_MB", "1")
    x, w, labels = _lm_head_case(32)
    w.main_grad = torch.zeros(w.shape, dtype=torch.float32, device="cuda")
    with B.loss_gradient_scale(torch.full((), 0.5, dtype=torch.float32, device="cuda")):
        loss = B.lm_head_cross_entropy(x, w, labels)
    loss.backward()  # scale 1, not the announced 0.5
    torch.cuda.synchronize()
    assert C.read_device_errors()[0] == 8
    C.reset_device_errors()


def _attn_ref(qkv, B, S, H, KV, hd):
    q = qkv[:, : H * hd].view(B, S, H, hd).transpose(1, 2)
    k = qkv[:, H * hd : (H + KV) * hd].view(B, S, KV, hd).transpose(1, 2)
    v = qkv[:, (H + KV) * hd :].view(B, S, KV, hd).transpose(1, 2)
    rep = H // KV
    k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
    s = s.masked_fill(torch.ones(S, S, device=qkv.device, dtype=torch.bool).triu(1), float("-inf"))
    o = torch.softmax(s, -1) @ v
    return o.transpose(1, 2).reshape(B * S, H * hd)


@pytest.mark.parametrize("B,S,H,KV,hd", [(2, 256, 4, 2, 64), (1, 512, 4, 4, 128), (2, 384, 6, 2, 64),
                                         (1, 256, 4, 2, 128),
                                         # more work items than SMs: each persistent CTA walks several
                                         (4, 1024, 12, 4, 64), (2, 1024, 16, 8, 128)])
def test_attention_forward_and_backward(C, B, S, H, KV, hd):
    from cs244c_llama_zero_b200.ops.functional import attention_backward, attention_forward, rope_tables

    qkv = _bf(B * S, (H + 2 * KV) * hd, seed=22)
    out, lse = attention_forward(qkv, B, S, H, KV, hd)
    qf = qkv.float().requires_grad_()
    ref = _attn_ref(qf, B, S, H, KV, hd)
    _close(out, ref, 2e-2)
    # log-sum-exp per (batch, head, row) in base-2 units of the scaled scores
    q = qf.detach()[:, : H * hd].view(B, S, H, hd).transpose(1, 2)
    k = qf.detach()[:, H * hd : (H + KV) * hd].view(B, S, KV, hd).transpose(1, 2).repeat_interleave(H // KV, 1)
    sc = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
    sc = sc.masked_fill(torch.ones(S, S, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    lse_ref = torch.logsumexp(sc, -1) / math.log(2.0)
    torch.testing.assert_close(lse.view(B, H, S), lse_ref, atol=2e-2, rtol=1e-3)
    dout = _bf(B * S, H * hd, seed=23)
    ref.backward(dout.float())
    # The backward kernel also applies RoPE backward to dq/dk: compare through an identity rotation.
    cos = torch.ones(S, hd // 2, device="cuda")
    sin = torch.zeros(S, hd // 2, device="cuda")
    dqkv = torch.empty_like(qkv)
    attention_backward(qkv, out, dout, lse, B, S, H, KV, hd, dqkv, cos, sin)
    _close(dqkv[:, : H * hd], qf.grad[:, : H * hd], 3e-2)
    _close(dqkv[:, H * hd : (H + KV) * hd], qf.grad[:, H * hd : (H + KV) * hd], 3e-2)
    _close(dqkv[:, (H + KV) * hd :], qf.grad[:, (H + KV) * hd :], 3e-2)
    # With a real rotation the result equals R^T applied to the identity-rotation gradient.
    cos, sin = rope_tables(S, hd, 10000.0, qkv.device)
    dqkv_rot = torch.empty_like(qkv)
    attention_backward(qkv, out, dout, lse, B, S, H, KV, hd, dqkv_rot, cos, sin)
    expect = dqkv.clone()
    C.rope_bwd(expect, (H + KV) * hd, hd, S, cos, sin)
    _close(dqkv_rot[:, : (H + KV) * hd], expect[:, : (H + KV) * hd], 2e-2)
