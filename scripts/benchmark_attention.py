"""Attention micro-benchmark for the tcgen05 flash-attention kernels (causal GQA, forward and backward).

For each shape ``B x S x H x KV x hd`` it times the forward and the backward (delta pre-pass, main
kernel and dQ conversion) with CUDA events: three warm-up calls, then the median of ``--iters`` calls,
each preceded by a write of a 256 MB buffer so that L2 (126 MB) holds nothing of the operands.  FLOPs
count the causal half of the score matrix once: forward 2 * 2 * B*H*S^2*hd / 2, backward 2.5x that
(five matrix products instead of two).  Each line reports TFLOP/s and the fraction of the measured
bf16 peak (``MEASURED_PEAKS.json``).

    python scripts/benchmark_attention.py --shapes 8x1024x12x4x64 4x2048x16x8x128

``--trace out.json`` also records the forward kernel's phase clocks for CTA 0 (built-in debug
tracing, enabled through ``ZB_ATTN_TRACE=1``, which this flag sets): per softmax tile the cycles
spent waiting for the scores, reading them and taking the row maximum, exponentiating, and handing P
back, and for the MMA thread the wait for each tile's P.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _peak() -> float:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def _parse(shape: str):
    b, s, h, kv, hd = (int(x) for x in shape.lower().split("x"))
    return b, s, h, kv, hd


def phase_summary(trace) -> dict:
    """Median cycles per phase from the (event, clock) pairs of each traced role."""
    names = {1: "score_wait", 2: "load_and_max", 3: "exp", 4: "p_handoff"}
    out = {}
    for role, label in ((1, "tile_a"), (2, "tile_b")):
        ev = trace[role]
        dur = {k: [] for k in names}
        for (e0, c0), (e1, c1) in zip(ev, ev[1:]):
            if e0 in names and e1 == e0 + 1:
                dur[e0].append(c1 - c0)
        starts = [c for e, c in ev if e == 1]
        cycles = [b - a for a, b in zip(starts, starts[1:])]
        out[label] = {names[k]: (statistics.median(v) if v else None) for k, v in dur.items()}
        out[label]["block_cycle"] = statistics.median(cycles) if cycles else None
    waits = [c1 - c0 for (e0, c0), (e1, c1) in zip(trace[0], trace[0][1:]) if e0 in (10, 11) and e1 == e0 + 10]
    out["mma_p_wait"] = statistics.median(waits) if waits else None
    return out


def bench(shape, iters: int, peak: float, trace_path: str = "") -> dict:
    import torch

    from cs244c_llama_zero_b200 import ops
    from cs244c_llama_zero_b200.ops.functional import attention_backward, attention_forward, rope_tables

    B, S, H, KV, hd = shape
    g = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(B * S, (H + 2 * KV) * hd, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(B * S, H * hd, device="cuda", generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(S, hd, 10000.0, qkv.device)
    out, lse = attention_forward(qkv, B, S, H, KV, hd)
    dqkv = torch.empty_like(qkv)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def timeit(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    fwd_ms = timeit(lambda: attention_forward(qkv, B, S, H, KV, hd, out=out))
    bwd_ms = timeit(lambda: attention_backward(qkv, out, dout, lse, B, S, H, KV, hd, dqkv, cos, sin))
    flops = 4.0 * B * H * S * S * hd / 2
    rec = {"shape": f"{B}x{S}x{H}x{KV}x{hd}", "fwd_us": fwd_ms * 1e3, "fwd_tflops": flops / fwd_ms / 1e9,
           "bwd_us": bwd_ms * 1e3, "bwd_tflops": 2.5 * flops / bwd_ms / 1e9}
    rec["fwd_frac_of_measured_peak"] = rec["fwd_tflops"] / peak
    rec["bwd_frac_of_measured_peak"] = rec["bwd_tflops"] / peak
    if trace_path:
        attention_forward(qkv, B, S, H, KV, hd, out=out)
        torch.cuda.synchronize()
        raw = ops.load_extension().attention_trace()
        trace = {}
        for role in range(3):
            row = raw[role].tolist()
            trace[role] = [(row[2 * i], row[2 * i + 1]) for i in range(len(row) // 2) if row[2 * i + 1] != 0]
        rec["phases_cycles"] = phase_summary(trace)
        with open(trace_path, "w") as fh:
            json.dump({"shape": rec["shape"], "trace": trace}, fh)
    return rec


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--shapes", nargs="+", default=["8x1024x12x4x64", "4x2048x16x8x128"])
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--trace", type=str, default="", help="write the forward's phase clocks (first shape) here")
    args = p.parse_args(argv)
    if args.trace:
        os.environ["ZB_ATTN_TRACE"] = "1"  # read once by the extension, before its first forward
    peak = _peak()
    for i, shape in enumerate(args.shapes):
        rec = bench(_parse(shape), args.iters, peak, args.trace if i == 0 else "")
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
