"""The ZeRO paper's model-state memory diagram for one of this repository's models (SVG).

Per device, with Psi parameters, N_d data-parallel ranks and K bytes of optimizer state per
parameter (mixed-precision Adam: fp32 master, m, v -> K = 12), parameters and gradients 2 bytes each:

    baseline (stage 0)        (2 + 2 + K) * Psi
    P_os     (stage 1)        (2 + 2) * Psi + K * Psi / N_d
    P_os+g   (stage 2)        2 * Psi + (2 + K) * Psi / N_d
    P_os+g+p (stage 3)        (2 + 2 + K) * Psi / N_d

Each row draws the N_d devices' bars split into parameters / gradients / optimizer state, with the
sharded parts shrunk to 1 / N_d, and labels the per-device total.
"""

from __future__ import annotations

import argparse
from html import escape
from pathlib import Path
from typing import Dict, List, Tuple

from cs244c_llama_zero_b200.models import build_config, estimate_num_parameters

PARAM_BYTES, GRAD_BYTES = 2, 2
COLORS = {"params": "#315A9A", "grads": "#4E8A3A", "optimizer": "#C56B1A"}


def per_device_bytes(psi: int, n_d: int, k: int = 12) -> Dict[str, Dict[str, float]]:
    """{stage label: {params, grads, optimizer, total}} bytes per device."""
    rows = {
        "Baseline": (PARAM_BYTES * psi, GRAD_BYTES * psi, k * psi),
        "P_os": (PARAM_BYTES * psi, GRAD_BYTES * psi, k * psi / n_d),
        "P_os+g": (PARAM_BYTES * psi, GRAD_BYTES * psi / n_d, k * psi / n_d),
        "P_os+g+p": (PARAM_BYTES * psi / n_d, GRAD_BYTES * psi / n_d, k * psi / n_d),
    }
    return {name: {"params": p, "grads": g, "optimizer": o, "total": p + g + o} for name, (p, g, o) in rows.items()}


def _gb(x: float) -> str:
    v = x / 1e9
    return f"{v:.1f}GB" if v < 100 else f"{v:.0f}GB"


def render_svg(psi: int, n_d: int, k: int, title: str) -> str:
    rows = per_device_bytes(psi, n_d, k)
    full = rows["Baseline"]["total"]
    shown = min(n_d, 8)
    W, row_h, bar_w, gap = 980, 110, 90, 12
    scale = (row_h - 30) / full
    parts: List[str] = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{80 + 4 * row_h}" '
                        'font-family="sans-serif" font-size="12">', '<rect width="100%" height="100%" fill="white"/>',
                        f'<text x="{W / 2}" y="28" text-anchor="middle" font-size="16">{escape(title)}</text>']
    for i, (name, b) in enumerate(rows.items()):
        y0 = 60 + i * row_h + row_h - 10
        parts.append(f'<text x="10" y="{y0 - 30}" font-size="13">{escape(name)}</text>')
        parts.append(f'<text x="10" y="{y0 - 12}">{_gb(b["total"])} / device</text>')
        for d in range(shown):
            x = 150 + d * (bar_w + gap)
            y = y0
            for part in ("params", "grads", "optimizer"):
                h = b[part] * scale
                y -= h
                parts.append(f'<rect x="{x}" y="{y:.1f}" width="{bar_w}" height="{max(h, 0.5):.1f}" '
                             f'fill="{COLORS[part]}"/>')
            parts.append(f'<text x="{x + bar_w / 2}" y="{y0 + 12}" text-anchor="middle" font-size="10">GPU {d}</text>')
        if n_d > shown:
            parts.append(f'<text x="{150 + shown * (bar_w + gap)}" y="{y0 - 20}">... x{n_d}</text>')
    for j, (part, color) in enumerate(COLORS.items()):
        parts.append(f'<rect x="{W - 170}" y="{50 + 18 * j}" width="12" height="12" fill="{color}"/>')
        parts.append(f'<text x="{W - 152}" y="{60 + 18 * j}">{part}</text>')
    return "\n".join(parts + ["</svg>"]) + "\n"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="ZeRO model-state memory per device, per stage (SVG diagram)")
    p.add_argument("--model-size", default="baseline-7b")
    p.add_argument("--vocab-size", type=int, default=32000)
    p.add_argument("--num-gpus", type=int, default=8)
    p.add_argument("--optimizer-bytes", type=int, default=12, help="K: optimizer bytes per parameter")
    p.add_argument("--output", default="analysis/figures/memory_parallelism.svg")
    a = p.parse_args(argv)
    psi = estimate_num_parameters(build_config(a.model_size, vocab_size=a.vocab_size))
    out = Path(a.output).with_suffix(".svg")
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(render_svg(psi, a.num_gpus, a.optimizer_bytes,
                              f"{a.model_size}: Psi = {psi / 1e6:.0f}M, N_d = {a.num_gpus}, K = {a.optimizer_bytes}"))
    for name, b in per_device_bytes(psi, a.num_gpus, a.optimizer_bytes).items():
        print(f"{name:10s} {_gb(b['total'])} per device")
    print(f"[memory-diagram] wrote {out}")


if __name__ == "__main__":
    main()
