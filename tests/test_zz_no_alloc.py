"""The allocation-free attention-backward entry point, called through its exported C symbol.

Some callers cannot let a library allocate GPU memory for them: an inference server or framework
whose device memory belongs to its own allocator, or plain C/C++ code that holds only raw device
pointers.  ``b200_attention_bwd_noalloc`` serves them from a fixed scratch array compiled into the
library.  This test calls it twice in a row (the second call reuses the scratch the first one left
behind), reads the kernels' error record after each call through
``b200_attention_bwd_noalloc_last_error``, and compares each result with the regular entry point,
which takes its scratch from the caller.  The file is named so that pytest collects it last; it
needs no state from the other tests and passes when run on its own.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, ERR_TOO_LARGE, ERR_INVALID = 0, -1, -2


def _lib():
    from cs244c_llama_zero_b200 import ops

    lib = ctypes.CDLL(ops.load_extension().__file__)
    fn = lib.b200_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn.argtypes = [p, i, i, i, p, p, i, p, p, p, p, i, i, i, i, i, f, p]
    last = lib.b200_attention_bwd_noalloc_last_error
    last.restype = ctypes.c_int
    last.argtypes = [ctypes.POINTER(ctypes.c_int)]
    return fn, last


def _call(fn, qkv, out, dout, lse, dqkv, cos, sin, B, S, H, KV, hd, ld_out=None):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(qkv.data_ptr(), qkv.stride(0), H * hd, (H + KV) * hd, out.data_ptr(), dout.data_ptr(),
              out.stride(0) if ld_out is None else ld_out, lse.data_ptr(), dqkv.data_ptr(), cos.data_ptr(),
              sin.data_ptr(), B, S, H, KV, hd, hd ** -0.5, stream)


def _record(last):
    rec = (ctypes.c_int * 4)()
    assert last(rec) == OK
    return list(rec)


def _close_rows(a, b, tol):
    """Max-abs error within ``tol`` of the largest magnitude, and every row within 4x that bound of
    its own scale (a wrong tail row cannot hide under the global scale)."""
    a, b = a.float(), b.float()
    err = (a - b).abs()
    ref = b.abs().max().item() + 1e-6
    assert err.max().item() <= tol * ref, f"max abs err {err.max().item():.4g} vs ref scale {ref:.4g}"
    row_ref = b.abs().amax(dim=1) + 1e-3 * ref
    worst = (err.amax(dim=1) / row_ref).max().item()
    assert worst <= 4 * tol, f"worst per-row relative error {worst:.4g}"


@pytest.mark.parametrize("B,S,H,KV,hd", [(2, 256, 4, 2, 64), (1, 384, 4, 2, 128)])
def test_noalloc_backward_matches_regular_entry_point_twice(B, S, H, KV, hd):
    from cs244c_llama_zero_b200.ops.functional import attention_backward, attention_forward, rope_tables

    fn, last = _lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = (torch.randn(B * S, (H + 2 * KV) * hd, device="cuda", generator=g)).to(torch.bfloat16)
    dout = (torch.randn(B * S, H * hd, device="cuda", generator=g)).to(torch.bfloat16)
    cos, sin = rope_tables(S, hd, 10000.0, qkv.device)
    out, lse = attention_forward(qkv, B, S, H, KV, hd)
    expected = torch.empty_like(qkv)
    attention_backward(qkv, out, dout, lse, B, S, H, KV, hd, expected, cos, sin)
    for _ in range(2):
        got = torch.full_like(qkv, float("nan"))
        assert _call(fn, qkv, out, dout, lse, got, cos, sin, B, S, H, KV, hd) == OK
        torch.cuda.synchronize()
        assert _record(last) == [0, 0, 0, 0]
        assert torch.isfinite(got.float()).all()
        _close_rows(got, expected, 1e-2)


def test_noalloc_backward_rejects_problems_larger_than_its_scratch():
    fn, _ = _lib()
    B, S, H, KV, hd = 8, 1024, 12, 4, 64  # needs ~25 MiB of dQ accumulator; the array holds 8 MiB
    qkv = torch.zeros(B * S, (H + 2 * KV) * hd, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(B * S, H * hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(B * H * S, device="cuda")
    cos = torch.ones(S, hd // 2, device="cuda")
    sin = torch.zeros(S, hd // 2, device="cuda")
    dqkv = torch.empty_like(qkv)
    assert _call(fn, qkv, out, out, lse, dqkv, cos, sin, B, S, H, KV, hd) == ERR_TOO_LARGE


def test_noalloc_backward_rejects_invalid_arguments():
    fn, _ = _lib()
    B, S, H, KV = 1, 256, 4, 2
    for hd, ld_out in ((96, None), (64, 64)):  # unsupported head_dim; output rows narrower than H*hd
        qkv = torch.zeros(B * S, (H + 2 * KV) * hd, device="cuda", dtype=torch.bfloat16)
        out = torch.zeros(B * S, H * hd, device="cuda", dtype=torch.bfloat16)
        lse = torch.zeros(B * H * S, device="cuda")
        cos = torch.ones(S, hd // 2, device="cuda")
        sin = torch.zeros(S, hd // 2, device="cuda")
        dqkv = torch.empty_like(qkv)
        assert _call(fn, qkv, out, out, lse, dqkv, cos, sin, B, S, H, KV, hd, ld_out=ld_out) == ERR_INVALID
