"""Performance figures (SVG): the roofline and the step breakdown.

Reference: src/transformer_internals/perf/plots.py:38-237 (operators placed
on the measured roofline; stacked step-time shares per configuration). Drawn
here with the dependency-free chart helper, so figures render on the GPU
image too.
"""

from __future__ import annotations

import math
from pathlib import Path
from typing import Any

from ..utils.svg import PALETTE, BarChart, LineChart

__all__ = ["fig_roofline", "fig_step_breakdown"]


def fig_roofline(payload: dict[str, Any], path) -> Path:
    """Roofline from a :func:`~gpt2_harness_b200.perf.roofline.roofline_payload`:
    the bound min(peak, I * bandwidth) and every operator of both dataflows
    at its intensity and roofline-attainable rate; measured rates, when
    present, as separate points."""
    pk = payload["peak"]
    P, BW = pk["peak_flops_per_s"], pk["peak_bytes_per_s"]
    rows = payload["eager"] + payload["native"]
    its = [r["intensity"] for r in rows]
    lo, hi = max(1e-2, min(its) / 3), max(its) * 3
    xs = [lo * (hi / lo) ** (i / 60) for i in range(61)]
    ch = LineChart(title=f"Roofline ({pk.get('device', '')}, {pk.get('dtype', '')})",
                   xlabel="arithmetic intensity (FLOP/byte)", ylabel="FLOP/s", xlog=True, ylog=True)
    ch.line(xs, [min(P, x * BW) for x in xs], "roofline", "#222")
    ch.line([r["intensity"] for r in payload["eager"]], [r["attainable_flops_per_s"] for r in payload["eager"]],
            "eager ops (bound)", PALETTE[1], markers_only=True)
    ch.line([r["intensity"] for r in payload["native"]], [r["attainable_flops_per_s"] for r in payload["native"]],
            "native fused ops (bound)", PALETTE[2], markers_only=True)
    for r in payload["native"]:
        ch.annotate(r["intensity"], r["attainable_flops_per_s"], r["name"].split(" (")[0])
    ch.hline(P, f"peak {P / 1e12:.0f} TFLOP/s")
    return ch.save(path)


def fig_step_breakdown(reports: list[dict[str, Any]], path) -> Path:
    """One bar per (configuration, category) share of step time, from
    profiler reports (``ProfileReport.as_dict()``) labelled by ``label``."""
    labels, vals, cols = [], [], []
    cats = sorted({c for r in reports for c in r.get("categories", {})})
    for ri, r in enumerate(reports):
        for ci, c in enumerate(cats):
            v = r.get("categories", {}).get(c, 0.0)
            if v > 0:
                labels.append(f"{r.get('label', f'run {ri}')}: {c}")
                vals.append(100.0 * v)
                cols.append(PALETTE[ci % len(PALETTE)])
    return BarChart(title="Step time by operator category", xlabel="% of device time", labels=labels,
                    values=vals, colors=cols).save(path)
