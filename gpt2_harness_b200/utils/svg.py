"""Dependency-free SVG charts (the image has no plotting library).

Three chart kinds cover every figure of the framework: ``LineChart`` (lines
and scatter, linear or log axes, legend), ``BarChart`` (horizontal bars with
optional error bars) and ``Heatmap`` (a labelled grid). Output is a plain SVG
string / file that any browser renders.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence
from xml.sax.saxutils import escape

__all__ = ["PALETTE", "LineChart", "BarChart", "Heatmap", "nice_ticks"]

PALETTE = ["#1f77b4", "#d62728", "#2ca02c", "#ff7f0e", "#9467bd", "#8c564b", "#e377c2", "#17becf", "#7f7f7f"]


def nice_ticks(lo: float, hi: float, n: int = 5, log: bool = False) -> list[float]:
    if log:
        a, b = math.floor(math.log10(lo)), math.ceil(math.log10(hi))
        return [10.0 ** e for e in range(a, b + 1)]
    if hi <= lo:
        hi = lo + 1.0
    raw = (hi - lo) / max(1, n)
    mag = 10 ** math.floor(math.log10(raw))
    step = min((m * mag for m in (1, 2, 2.5, 5, 10) if m * mag >= raw), default=raw)
    start = math.floor(lo / step) * step
    out, v = [], start
    while v <= hi + 1e-9 * step:
        out.append(round(v, 12))
        v += step
    return out


def _fmt(v: float) -> str:
    if v == 0:
        return "0"
    a = abs(v)
    if a >= 1e4 or a < 1e-2:
        e = int(math.floor(math.log10(a)))
        m = v / 10 ** e
        return f"{m:g}e{e}" if abs(m - round(m)) > 1e-9 else f"1e{e}" if round(m) == 1 else f"{round(m)}e{e}"
    return f"{v:g}"


class _Canvas:
    def __init__(self, w: int, h: int) -> None:
        self.w, self.h = w, h
        self.parts: list[str] = []

    def add(self, s: str) -> None:
        self.parts.append(s)

    def text(self, x, y, s, size=12, anchor="middle", rotate: Optional[float] = None, color="#222", weight="normal"):
        tr = f' transform="rotate({rotate} {x:.1f} {y:.1f})"' if rotate else ""
        self.add(f'<text x="{x:.1f}" y="{y:.1f}" font-size="{size}" text-anchor="{anchor}" fill="{color}" '
                 f'font-family="sans-serif" font-weight="{weight}"{tr}>{escape(str(s))}</text>')

    def svg(self) -> str:
        return (f'<svg xmlns="http://www.w3.org/2000/svg" width="{self.w}" height="{self.h}" '
                f'viewBox="0 0 {self.w} {self.h}"><rect width="100%" height="100%" fill="white"/>'
                + "".join(self.parts) + "</svg>")


@dataclass
class LineChart:
    title: str = ""
    xlabel: str = ""
    ylabel: str = ""
    xlog: bool = False
    ylog: bool = False
    width: int = 720
    height: int = 440
    series: list = field(default_factory=list)    # (label, xs, ys, color, dashed, markers_only)
    hlines: list = field(default_factory=list)    # (y, label, color)
    annotations: list = field(default_factory=list)  # (x, y, text)

    def line(self, xs: Sequence[float], ys: Sequence[float], label: str = "", color: Optional[str] = None,
             dashed: bool = False, markers_only: bool = False) -> "LineChart":
        self.series.append((label, list(xs), list(ys), color or PALETTE[len(self.series) % len(PALETTE)], dashed,
                            markers_only))
        return self

    def hline(self, y: float, label: str = "", color: str = "#888") -> "LineChart":
        self.hlines.append((y, label, color))
        return self

    def annotate(self, x: float, y: float, text: str) -> "LineChart":
        self.annotations.append((x, y, text))
        return self

    def _range(self, vals, log):
        v = [x for x in vals if x is not None and math.isfinite(x) and (not log or x > 0)]
        if not v:
            return (1.0, 10.0) if log else (0.0, 1.0)
        lo, hi = min(v), max(v)
        if lo == hi:
            lo, hi = (lo / 2, hi * 2) if log else (lo - 1, hi + 1)
        return lo, hi

    def render(self) -> str:
        c = _Canvas(self.width, self.height)
        L, R, T, B = 80, 20, 40, 60
        pw, ph = self.width - L - R, self.height - T - B
        xs = [x for s in self.series for x in s[1]]
        ys = [y for s in self.series for y in s[2]] + [h[0] for h in self.hlines]
        x0, x1 = self._range(xs, self.xlog)
        y0, y1 = self._range(ys, self.ylog)
        xt, yt = nice_ticks(x0, x1, 6, self.xlog), nice_ticks(y0, y1, 5, self.ylog)
        x0, x1 = min(x0, xt[0]), max(x1, xt[-1])
        y0, y1 = min(y0, yt[0]), max(y1, yt[-1])
        f = (lambda v, lo, hi, lg: (math.log10(v) - math.log10(lo)) / (math.log10(hi) - math.log10(lo)) if lg
             else (v - lo) / (hi - lo))
        X = lambda v: L + pw * f(v, x0, x1, self.xlog)  # noqa: E731
        Y = lambda v: T + ph * (1 - f(v, y0, y1, self.ylog))  # noqa: E731
        for t in yt:
            c.add(f'<line x1="{L}" x2="{L + pw}" y1="{Y(t):.1f}" y2="{Y(t):.1f}" stroke="#eee"/>')
            c.text(L - 6, Y(t) + 4, _fmt(t), 11, "end")
        for t in xt:
            c.add(f'<line x1="{X(t):.1f}" x2="{X(t):.1f}" y1="{T}" y2="{T + ph}" stroke="#f4f4f4"/>')
            c.text(X(t), T + ph + 16, _fmt(t), 11)
        c.add(f'<rect x="{L}" y="{T}" width="{pw}" height="{ph}" fill="none" stroke="#444"/>')
        for y, lab, col in self.hlines:
            c.add(f'<line x1="{L}" x2="{L + pw}" y1="{Y(y):.1f}" y2="{Y(y):.1f}" stroke="{col}" '
                  f'stroke-dasharray="4,3"/>')
            if lab:
                c.text(L + pw - 4, Y(y) - 4, lab, 10, "end", color=col)
        for lab, sx, sy, col, dashed, mo in self.series:
            pts = [(X(a), Y(b)) for a, b in zip(sx, sy)
                   if a is not None and b is not None and math.isfinite(a) and math.isfinite(b)
                   and (not self.xlog or a > 0) and (not self.ylog or b > 0)]
            if not mo and len(pts) > 1:
                d = " ".join(f"{x:.1f},{y:.1f}" for x, y in pts)
                c.add(f'<polyline points="{d}" fill="none" stroke="{col}" stroke-width="2"'
                      + (' stroke-dasharray="6,4"' if dashed else "") + "/>")
            for x, y in pts:
                c.add(f'<circle cx="{x:.1f}" cy="{y:.1f}" r="3" fill="{col}"/>')
        for ax, ay, txt in self.annotations:
            c.text(X(ax) + 5, Y(ay) - 5, txt, 10, "start")
        leg = [(s[0], s[3]) for s in self.series if s[0]]
        for i, (lab, col) in enumerate(leg):
            yy = T + 14 + 16 * i
            c.add(f'<rect x="{L + 10}" y="{yy - 9}" width="12" height="10" fill="{col}"/>')
            c.text(L + 28, yy, lab, 11, "start")
        c.text(self.width / 2, 24, self.title, 15, weight="bold")
        c.text(L + pw / 2, self.height - 16, self.xlabel, 12)
        c.text(20, T + ph / 2, self.ylabel, 12, rotate=-90)
        return c.svg()

    def save(self, path) -> Path:
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(self.render(), encoding="utf-8")
        return p


@dataclass
class BarChart:
    title: str = ""
    xlabel: str = ""
    labels: list = field(default_factory=list)
    values: list = field(default_factory=list)
    errors: Optional[list] = None
    colors: Optional[list] = None
    reference: Optional[float] = None
    width: int = 720

    def render(self) -> str:
        n = len(self.labels)
        h = 70 + 26 * max(1, n)
        c = _Canvas(self.width, h)
        L, R, T = 230, 30, 40
        pw = self.width - L - R
        vals = [v for v in self.values if math.isfinite(v)] + ([self.reference] if self.reference is not None else [])
        lo = min(0.0, min(vals, default=0.0))
        hi = max(vals, default=1.0)
        if self.errors:
            hi = max(hi, max((v + e for v, e in zip(self.values, self.errors) if math.isfinite(v)), default=hi))
        hi = hi if hi > lo else lo + 1.0
        X = lambda v: L + pw * (v - lo) / (hi - lo)  # noqa: E731
        for t in nice_ticks(lo, hi, 5):
            if lo <= t <= hi:
                c.add(f'<line x1="{X(t):.1f}" x2="{X(t):.1f}" y1="{T}" y2="{T + 26 * n}" stroke="#eee"/>')
                c.text(X(t), T + 26 * n + 14, _fmt(t), 10)
        for i, (lab, v) in enumerate(zip(self.labels, self.values)):
            y = T + 26 * i
            col = (self.colors[i] if self.colors else PALETTE[0])
            if math.isfinite(v):
                x0, x1 = sorted((X(0.0), X(v)))
                c.add(f'<rect x="{x0:.1f}" y="{y + 4}" width="{max(1.0, x1 - x0):.1f}" height="18" fill="{col}"/>')
                c.text(x1 + 4, y + 17, _fmt(v), 10, "start")
                if self.errors:
                    e = self.errors[i]
                    c.add(f'<line x1="{X(v - e):.1f}" x2="{X(v + e):.1f}" y1="{y + 13}" y2="{y + 13}" '
                          f'stroke="#222"/>')
            c.text(L - 6, y + 17, lab, 11, "end")
        if self.reference is not None:
            c.add(f'<line x1="{X(self.reference):.1f}" x2="{X(self.reference):.1f}" y1="{T}" y2="{T + 26 * n}" '
                  f'stroke="#d62728" stroke-dasharray="4,3"/>')
        c.text(self.width / 2, 24, self.title, 15, weight="bold")
        c.text(L + pw / 2, h - 8, self.xlabel, 12)
        return c.svg()

    def save(self, path) -> Path:
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(self.render(), encoding="utf-8")
        return p


@dataclass
class Heatmap:
    title: str = ""
    grid: list = field(default_factory=list)  # rows of floats
    row_labels: Optional[list] = None
    col_labels: Optional[list] = None
    cell: int = 34

    def render(self) -> str:
        nr = len(self.grid)
        nc = len(self.grid[0]) if nr else 0
        L, T = 60, 50
        w, h = L + nc * self.cell + 90, T + nr * self.cell + 40
        c = _Canvas(w, h)
        flat = [v for r in self.grid for v in r if math.isfinite(v)]
        lo, hi = (min(flat), max(flat)) if flat else (0.0, 1.0)
        span = hi - lo if hi > lo else 1.0
        for i, row in enumerate(self.grid):
            for j, v in enumerate(row):
                t = (v - lo) / span if math.isfinite(v) else 0.0
                r_, g_, b_ = int(255 - 200 * t), int(255 - 120 * t), int(255 - 40 * t)
                x, y = L + j * self.cell, T + i * self.cell
                c.add(f'<rect x="{x}" y="{y}" width="{self.cell}" height="{self.cell}" fill="rgb({r_},{g_},{b_})" '
                      f'stroke="white"/>')
                c.text(x + self.cell / 2, y + self.cell / 2 + 4, f"{v:.2f}" if math.isfinite(v) else "-", 9,
                       color="white" if t > 0.6 else "#222")
            c.text(L - 6, T + i * self.cell + self.cell / 2 + 4,
                   self.row_labels[i] if self.row_labels else f"L{i}", 10, "end")
        for j in range(nc):
            c.text(L + j * self.cell + self.cell / 2, T - 6, self.col_labels[j] if self.col_labels else f"H{j}", 10)
        c.text(w / 2, 22, self.title, 14, weight="bold")
        c.text(L + nc * self.cell + 10, T + 12, f"max {_fmt(hi)}", 10, "start")
        c.text(L + nc * self.cell + 10, T + 28, f"min {_fmt(lo)}", 10, "start")
        return c.svg()

    def save(self, path) -> Path:
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(self.render(), encoding="utf-8")
        return p
