"""Dependency-free SVG charts (line, grouped bar, stacked bar) for the analysis reports.

The image has no plotting library, so figures are written as standalone SVG documents: axes with
"nice" ticks, an optional log-scale x axis, a legend, and a fixed colour cycle.
"""

from __future__ import annotations

import math
from html import escape
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple

PALETTE = ["#1f77b4", "#ff7f0e", "#2ca02c", "#d62728", "#9467bd", "#8c564b", "#e377c2", "#7f7f7f",
           "#bcbd22", "#17becf"]
W, H = 760, 460
ML, MR, MT, MB = 80, 170, 50, 70  # margins: left, right (legend), top, bottom


def nice_ticks(lo: float, hi: float, n: int = 5) -> List[float]:
    """Round tick values covering [lo, hi] (1/2/5 x 10^k steps)."""
    if not math.isfinite(lo) or not math.isfinite(hi):
        return [0.0, 1.0]
    if hi <= lo:
        hi = lo + (abs(lo) if lo else 1.0)
    raw = (hi - lo) / max(1, n)
    mag = 10 ** math.floor(math.log10(raw))
    step = next(m * mag for m in (1, 2, 5, 10) if m * mag >= raw)
    start = math.floor(lo / step) * step
    ticks = []
    t = start
    while t <= hi + step * 0.5:
        ticks.append(round(t, 12))
        t += step
    return ticks


def _fmt(v: float) -> str:
    if v == 0:
        return "0"
    a = abs(v)
    if a >= 1e6 or a < 1e-3:
        return f"{v:.2e}"
    return f"{v:,.0f}" if a >= 100 else f"{v:g}"


class _Canvas:
    def __init__(self, title: str, xlabel: str, ylabel: str):
        self.parts: List[str] = [
            f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" viewBox="0 0 {W} {H}" '
            'font-family="sans-serif" font-size="12">',
            f'<rect width="{W}" height="{H}" fill="white"/>',
            f'<text x="{(ML + W - MR) / 2}" y="28" text-anchor="middle" font-size="16">{escape(title)}</text>',
            f'<text x="{(ML + W - MR) / 2}" y="{H - 18}" text-anchor="middle">{escape(xlabel)}</text>',
            f'<text x="18" y="{(MT + H - MB) / 2}" text-anchor="middle" '
            f'transform="rotate(-90 18 {(MT + H - MB) / 2})">{escape(ylabel)}</text>',
        ]
        self.legend_rows = 0

    def y_axis(self, ticks: Sequence[float]) -> Tuple[float, float]:
        lo, hi = ticks[0], ticks[-1]
        for t in ticks:
            y = self.ymap(t, lo, hi)
            self.parts.append(f'<line x1="{ML}" x2="{W - MR}" y1="{y:.1f}" y2="{y:.1f}" stroke="#ddd"/>')
            self.parts.append(f'<text x="{ML - 6}" y="{y + 4:.1f}" text-anchor="end">{_fmt(t)}</text>')
        self.parts.append(f'<line x1="{ML}" x2="{ML}" y1="{MT}" y2="{H - MB}" stroke="black"/>')
        self.parts.append(f'<line x1="{ML}" x2="{W - MR}" y1="{H - MB}" y2="{H - MB}" stroke="black"/>')
        return lo, hi

    @staticmethod
    def ymap(v: float, lo: float, hi: float) -> float:
        return H - MB - (v - lo) / (hi - lo or 1.0) * (H - MB - MT)

    def legend(self, label: str, color: str) -> None:
        y = MT + 18 * self.legend_rows
        self.parts.append(f'<rect x="{W - MR + 14}" y="{y}" width="12" height="12" fill="{color}"/>')
        self.parts.append(f'<text x="{W - MR + 32}" y="{y + 10}">{escape(label)}</text>')
        self.legend_rows += 1

    def save(self, output: Path) -> Path:
        output = Path(output)
        if output.suffix.lower() != ".svg":
            output = output.with_suffix(".svg")
        output.parent.mkdir(parents=True, exist_ok=True)
        output.write_text("\n".join(self.parts + ["</svg>"]) + "\n")
        return output


def line_chart(series: Dict[str, List[Tuple[float, float]]], output: Path, *, title: str, xlabel: str, ylabel: str,
               log_x: bool = False, x_tick_labels: Optional[Dict[float, str]] = None) -> Path:
    """One polyline with markers per series; ``x_tick_labels`` overrides the x tick text."""
    c = _Canvas(title, xlabel, ylabel)
    pts = [p for s in series.values() for p in s if p[1] is not None and math.isfinite(p[1])]
    if not pts:
        return c.save(output)
    xs = sorted({p[0] for p in pts})
    ys = [p[1] for p in pts]
    lo, hi = c.y_axis(nice_ticks(min(0.0, min(ys)), max(ys)))

    def xmap(x: float) -> float:
        if len(xs) == 1:
            return (ML + W - MR) / 2
        if log_x:
            a, b, v = math.log(xs[0]), math.log(xs[-1]), math.log(x)
        else:
            a, b, v = xs[0], xs[-1], x
        return ML + 20 + (v - a) / (b - a or 1.0) * (W - MR - ML - 40)

    for x in xs:
        label = (x_tick_labels or {}).get(x, _fmt(x))
        c.parts.append(f'<text x="{xmap(x):.1f}" y="{H - MB + 18}" text-anchor="middle">{escape(label)}</text>')
    for i, (name, s) in enumerate(series.items()):
        color = PALETTE[i % len(PALETTE)]
        s = sorted((p for p in s if p[1] is not None), key=lambda p: p[0])
        path = " ".join(f"{xmap(x):.1f},{c.ymap(y, lo, hi):.1f}" for x, y in s)
        c.parts.append(f'<polyline points="{path}" fill="none" stroke="{color}" stroke-width="2"/>')
        for x, y in s:
            c.parts.append(f'<circle cx="{xmap(x):.1f}" cy="{c.ymap(y, lo, hi):.1f}" r="3.5" fill="{color}"/>')
        c.legend(name, color)
    return c.save(output)


def bar_chart(categories: List[str], groups: Dict[str, List[Optional[float]]], output: Path, *, title: str,
              xlabel: str, ylabel: str, stacked: bool = False, annotate: bool = False) -> Path:
    """Grouped (or stacked) bars: ``groups[name][i]`` is the bar of ``name`` in ``categories[i]``."""
    c = _Canvas(title, xlabel, ylabel)
    n = max(1, len(categories))
    if stacked:
        tops = [sum((g[i] or 0.0) for g in groups.values()) for i in range(len(categories))]
    else:
        tops = [v for g in groups.values() for v in g if v is not None]
    lo, hi = c.y_axis(nice_ticks(0.0, max(tops) if tops else 1.0))
    slot = (W - MR - ML) / n
    k = 1 if stacked else max(1, len(groups))
    bw = slot * 0.8 / k
    for i, cat in enumerate(categories):
        c.parts.append(f'<text x="{ML + slot * (i + 0.5):.1f}" y="{H - MB + 18}" text-anchor="middle">'
                       f'{escape(cat)}</text>')
    base = [0.0] * len(categories)
    for j, (name, vals) in enumerate(groups.items()):
        color = PALETTE[j % len(PALETTE)]
        for i, v in enumerate(vals):
            if v is None:
                continue
            x = ML + slot * i + slot * 0.1 + (0 if stacked else j * bw)
            y0 = base[i] if stacked else 0.0
            top, bottom = c.ymap(y0 + v, lo, hi), c.ymap(y0, lo, hi)
            c.parts.append(f'<rect x="{x:.1f}" y="{top:.1f}" width="{bw:.1f}" height="{max(0.0, bottom - top):.1f}" '
                           f'fill="{color}"/>')
            if annotate:
                c.parts.append(f'<text x="{x + bw / 2:.1f}" y="{top - 4:.1f}" text-anchor="middle" font-size="10">'
                               f'{_fmt(v)}</text>')
            if stacked:
                base[i] += v
        c.legend(name, color)
    return c.save(output)
