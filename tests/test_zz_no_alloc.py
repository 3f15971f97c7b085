"""The allocation-free attention-backward entry point, called through its exported C symbol.

Callers such as inference servers or C/C++ hosts that own all device memory cannot let a library
allocate scratch for them; ``b200_attention_bwd_noalloc`` serves them from a fixed array compiled
into the library.  This test calls it twice in a row (the second call reuses the scratch the first
one left behind) and compares each result with the regular entry point, which takes its scratch
from the caller.  It lives in its own file, collected last, and works in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, ERR_TOO_LARGE = 0, -1


def _lib():
    from cs244c_llama_zero_b200 import ops

    lib = ctypes.CDLL(ops.load_extension().__file__)
    fn = lib.b200_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn.argtypes = [p, i, i, i, p, p, i, p, p, p, p, i, i, i, i, i, f, p]
    return fn


def _call(fn, qkv, out, dout, lse, dqkv, cos, sin, B, S, H, KV, hd):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(qkv.data_ptr(), qkv.stride(0), H * hd, (H + KV) * hd, out.data_ptr(), dout.data_ptr(), out.stride(0),
              lse.data_ptr(), dqkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), B, S, H, KV, hd, hd ** -0.5, stream)


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    ref = b.float().abs().max().item() + 1e-6
    assert err <= tol * ref, f"max abs err {err:.4g} vs ref scale {ref:.4g}"


@pytest.mark.parametrize("B,S,H,KV,hd", [(2, 256, 4, 2, 64), (1, 384, 4, 2, 128)])
def test_noalloc_backward_matches_regular_entry_point_twice(B, S, H, KV, hd):
    from cs244c_llama_zero_b200.ops.functional import attention_backward, attention_forward, rope_tables

    fn = _lib()
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
        assert torch.isfinite(got.float()).all()
        _close(got, expected, 1e-2)


def test_noalloc_backward_rejects_problems_larger_than_its_scratch():
    fn = _lib()
    B, S, H, KV, hd = 8, 1024, 12, 4, 64  # needs ~25 MiB of dQ accumulator; the array holds 8 MiB
    qkv = torch.zeros(B * S, (H + 2 * KV) * hd, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(B * S, H * hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(B * H * S, device="cuda")
    cos = torch.ones(S, hd // 2, device="cuda")
    sin = torch.zeros(S, hd // 2, device="cuda")
    dqkv = torch.empty_like(qkv)
    assert _call(fn, qkv, out, out, lse, dqkv, cos, sin, B, S, H, KV, hd) == ERR_TOO_LARGE
