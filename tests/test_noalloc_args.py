"""Argument checks of the allocation-free attention-backward C entry point, on the CPU.

The checks run before the entry point touches the GPU, so a layout that does not fit, or an
unsupported head size, is rejected here with ERR_INVALID without a device (the pointers are fake,
16-byte aligned and never dereferenced).
"""

from __future__ import annotations

import ctypes

import pytest

ERR_INVALID = -2


def _fn():
    from cs244c_llama_zero_b200 import ops

    try:
        lib = ctypes.CDLL(ops.load_extension().__file__)
    except ImportError:
        pytest.skip("extension not built")
    fn = lib.b200_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn.argtypes = [p, i, i, i, p, p, i, p, p, p, p, i, i, i, i, i, f, p]
    return fn


def _call(fn, *, ld, k_col, v_col, ld_out, H=4, KV=2, hd=64, S=256):
    fake = 1 << 20  # aligned, never dereferenced
    return fn(fake, ld, k_col, v_col, fake, fake, ld_out, fake, fake, fake, fake, 1, S, H, KV, hd, 0.125, None)


@pytest.mark.parametrize("kw", [
    dict(ld=512, k_col=256, v_col=384, ld_out=128),   # output rows narrower than heads*head_dim
    dict(ld=448, k_col=256, v_col=384, ld_out=256),   # v block runs past the row
    dict(ld=512, k_col=192, v_col=384, ld_out=256),   # q block overlaps k
    dict(ld=512, k_col=256, v_col=320, ld_out=256),   # k block overlaps v
    dict(ld=768, k_col=384, v_col=576, ld_out=384, hd=96),  # unsupported head_dim
])
def test_layouts_that_do_not_fit_are_rejected_before_any_cuda_call(kw):
    assert _call(_fn(), **kw) == ERR_INVALID
