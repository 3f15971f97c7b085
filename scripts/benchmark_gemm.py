"""GEMM micro-benchmark for the tcgen05 kernels: every tile width / CTA-group variant vs the automatic choice.

For each shape (M x N x K and the operand layout of a linear layer's forward, data-gradient or
weight-gradient GEMM) it times each variant with CUDA events: warm-up launches first, then the median
of `--iters` launches, each preceded by a write of a 256 MB buffer so that L2 (126 MB) holds nothing
of the operands.  It prints TFLOP/s per variant and the fraction of the measured bf16 peak
(`MEASURED_PEAKS.json`), with torch.matmul (cuBLAS) on the same shape for reference.  Weight-gradient
variants keep the automatic K-split for their tile.

    python scripts/benchmark_gemm.py --shapes 8192x768x4096:dgrad 8192x2048x768:fwd 1280x768x8192:wgrad
    python scripts/benchmark_gemm.py --shapes 8192x1280x768:rope64-1024 8192x4096x768:swiglu 8192x768x768:res

(`rope<hd>-<cols>`: the fused q|k|v projection with RoPE on its first `cols` columns (the q and k
heads); `swiglu`: gate|up with the SwiGLU epilogue, N = 2 * ffn; `res`: forward with the
residual-add epilogue.)

`T x out x in:pair` shapes time a linear layer's backward pair (dx = dy @ w and dw += dy^T @ x):
the two automatic launches one after the other vs the grouped launch that deals both problems'
tiles together (`linear_dgrad_wgrad`).

    python scripts/benchmark_gemm.py --shapes 8192x4096x768:pair 8192x768x768:pair 8192x1280x768:pair
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

# name -> bn argument of the bindings (0 = automatic; >= 1000 = CTA pair of width bn - 1000)
VARIANTS = [("auto", 0), ("cg1-256", 256), ("cg1-192", 192), ("cg1-128", 128), ("cg2-256", 1256), ("cg2-192", 1192),
            ("cg2-128", 1128)]


def _peak() -> float:
    try:
        return float(json.loads((Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def _time(fn, iters: int, flush: torch.Tensor) -> float:
    for _ in range(3):
        fn()
    times = []
    for _ in range(iters):
        flush.add_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--shapes", nargs="+", default=["8192x768x4096:dgrad", "8192x2048x768:fwd", "8192x768x2048:fwd",
                                                   "4096x768x8192:wgrad", "1280x768x8192:wgrad", "8192x32000x768:fwd"])
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--output-json", default="")
    a = p.parse_args(argv)
    from cs244c_llama_zero_b200 import ops

    C = ops.load_extension()
    peak = _peak()
    flush = torch.empty(64 * 2**20, device="cuda", dtype=torch.float32)
    rows = []
    for spec in a.shapes:
        dims, kind = spec.split(":")
        M, N, K = (int(x) for x in dims.split("x"))
        g = torch.Generator(device="cuda").manual_seed(0)
        rnd = lambda *s: (torch.randn(*s, device="cuda", generator=g) * 0.05).to(torch.bfloat16)  # noqa: E731
        flops = 2.0 * M * N * K
        if kind in ("fwd", "res"):  # y[M,N] = x[M,K] w[N,K]^T (+ residual r[M,N] for "res")
            x, w, y = rnd(M, K), rnd(N, K), torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            r = rnd(M, N) if kind == "res" else None
            run = lambda bn: C.linear_fwd(x, w, y, r, bn)  # noqa: E731
            ref = lambda: torch.matmul(x, w.t())  # noqa: E731
        elif kind.startswith("rope"):  # fused q|k|v projection, RoPE on the first columns: "rope64-1024"
            hd_s, _, cols_s = kind[4:].partition("-")
            hd = int(hd_s or 64)
            rope_cols = int(cols_s) if cols_s else N
            from cs244c_llama_zero_b200.ops.functional import rope_tables_t

            seq = 1024 if M % 1024 == 0 else M
            cos, sin = rope_tables_t(seq, hd, 10000.0, torch.device("cuda"))
            x, w, y = rnd(M, K), rnd(N, K), torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            run = lambda bn: C.qkv_rope_fwd(x, w, y, cos, sin, seq, hd, rope_cols, bn)  # noqa: E731
            ref = lambda: torch.matmul(x, w.t())  # noqa: E731
        elif kind == "swiglu":  # h[M,N/2] = silu(x Wg^T) * (x Wu^T), N = 2 * ffn
            x, w = rnd(M, K), rnd(N, K)
            h = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
            gu = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            run = lambda bn: C.swiglu_fwd(x, w, h, gu, bn)  # noqa: E731
            ref = lambda: torch.matmul(x, w.t())  # noqa: E731
        elif kind == "dgrad":  # dx[M,N] = dy[M,K] w[K,N]
            dy, w, dx = rnd(M, K), rnd(K, N), torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            run = lambda bn: C.linear_dgrad(dy, w, dx, bn)  # noqa: E731
            ref = lambda: torch.matmul(dy, w)  # noqa: E731
        else:  # wgrad: dw[M,N] += dy[K,M]^T x[K,N]
            dy, x, dw = rnd(K, M), rnd(K, N), torch.zeros(M, N, device="cuda", dtype=torch.float32)
            run = lambda bn: C.linear_wgrad(dy, x, dw, 0, bn)  # noqa: E731
            ref = lambda: torch.matmul(dy.t(), x)  # noqa: E731
        if kind == "pair":  # T x out x in: dx[T,in] = dy[T,out] w[out,in]; dw[out,in] += dy^T x[T,in]
            T, out, inp = M, N, K
            dy, w, x = rnd(T, out), rnd(out, inp), rnd(T, inp)
            dx = torch.empty(T, inp, device="cuda", dtype=torch.bfloat16)
            dw = torch.zeros(out, inp, device="cuda", dtype=torch.float32)
            flops = 4.0 * T * out * inp
            row = {"shape": spec, "gflop": flops / 1e9}
            for name, fn in (("separate", lambda: (C.linear_dgrad(dy, w, dx, 0), C.linear_wgrad(dy, x, dw, 0, 0))),
                             ("grouped", lambda: C.linear_dgrad_wgrad(dy, w, x, dx, dw, 0)),
                             ("cublas", lambda: (torch.matmul(dy, w), torch.matmul(dy.t(), x)))):
                ms = _time(fn, a.iters, flush)
                row[name] = {"ms": ms, "tflops": flops / ms / 1e9, "frac_of_measured": flops / ms / 1e9 / peak}
            rows.append(row)
            print(f"{spec:22s} " + " ".join(f"{k}={v['tflops']:.0f}" for k, v in row.items() if isinstance(v, dict)),
                  flush=True)
            continue
        row = {"shape": spec, "gflop": flops / 1e9}
        for name, bn in VARIANTS:
            try:
                ms = _time(lambda: run(bn), a.iters, flush)
                row[name] = {"ms": ms, "tflops": flops / ms / 1e9, "frac_of_measured": flops / ms / 1e9 / peak}
            except RuntimeError as exc:  # variant not available for this epilogue / operand layout
                row[name] = {"error": str(exc).splitlines()[0][:100]}
        ms = _time(ref, a.iters, flush)
        row["cublas"] = {"ms": ms, "tflops": flops / ms / 1e9, "frac_of_measured": flops / ms / 1e9 / peak}
        rows.append(row)
        print(f"{spec:22s} " + " ".join(f"{k}={v['tflops']:.0f}" if "tflops" in v else f"{k}=n/a"
                                        for k, v in row.items() if isinstance(v, dict)), flush=True)
    result = {"peak_bf16_tflops_measured": peak, "rows": rows}
    print(json.dumps(result))
    if a.output_json:
        Path(a.output_json).write_text(json.dumps(result, indent=2))


if __name__ == "__main__":
    main()
