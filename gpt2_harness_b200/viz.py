"""Figures from committed result JSON (SVG, no plotting library needed).

Reference: src/transformer_internals/viz.py:129-735 (verification,
induction heatmap, ablations, KV-cache latency and memory, quantization,
pruning Pareto, distillation, quality/size Pareto, pipeline bubble). Every
function takes the JSON payload the matching module writes and a path;
:func:`make_all` redraws whatever payloads exist in a results directory, and
adds the B200 throughput-scaling figure from ``bench.py`` lines.

    python -m gpt2_harness_b200.viz results/ figures/
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path
from typing import Any

from .utils.svg import PALETTE, BarChart, Heatmap, LineChart

__all__ = ["fig_verification", "fig_induction_heatmap", "fig_ablations", "fig_kv_latency", "fig_kv_memory",
           "fig_quantization", "fig_pruning_pareto", "fig_distillation", "fig_pareto", "fig_parallel_bubble",
           "fig_scaling", "make_all"]


def fig_verification(report: dict[str, Any], path) -> Path:
    """Per-activation max |delta| against HF (log scale) with the tolerance."""
    rows = report["layers"]
    ch = LineChart(title="Activation agreement with HuggingFace GPT-2", xlabel="activation (depth order)",
                   ylabel="max |ours - HF|", ylog=True)
    ch.line(list(range(len(rows))), [max(r["max_abs"], 1e-12) for r in rows], "max |delta|")
    ch.hline(report.get("logit_tolerance", 1e-3), "logit tolerance")
    return ch.save(path)


def fig_induction_heatmap(scores: dict[str, Any], path, key: str = "prefix_matching") -> Path:
    g = scores[key]
    return Heatmap(title=f"Induction probe: {key.replace('_', ' ')} per head", grid=g,
                   row_labels=[f"L{i}" for i in range(len(g))]).save(path)


def fig_ablations(summary: dict[str, Any], path) -> Path:
    rows = summary["rows"]
    col = {"reference": "#7f7f7f", "indistinguishable": PALETTE[0], "worse": PALETTE[1], "better": PALETTE[2]}
    return BarChart(title="Ablations: final validation loss (mean +- std over seeds)", xlabel="val loss",
                    labels=[f"{r['label']} [{r['verdict']}]" for r in rows], values=[r["val_loss_mean"] for r in rows],
                    errors=[r["val_loss_std"] for r in rows], colors=[col.get(r["verdict"], PALETTE[0]) for r in rows],
                    reference=rows[0]["val_loss_mean"] if rows else None).save(path)


def fig_kv_latency(bench: dict[str, Any], path) -> Path:
    """ms/token vs prompt length per arm (cached / uncached / native)."""
    ch = LineChart(title="Decode latency vs prompt length", xlabel="prompt length (tokens)", ylabel="ms / token")
    for i, arm in enumerate(("cached", "uncached", "native")):
        pts = sorted((r["prompt_len"], r["ms_per_token"]) for r in bench["rows"] if r.get("arm") == arm)
        if pts:
            ch.line([p[0] for p in pts], [p[1] for p in pts], arm, PALETTE[i])
    return ch.save(path)


def fig_kv_memory(bench: dict[str, Any], path) -> Path:
    ch = LineChart(title="KV-cache size vs context", xlabel="context (tokens)", ylabel="MB", ylog=True)
    by_bs: dict = {}
    for r in bench["kv_cache"]:
        by_bs.setdefault(r["batch_size"], []).append((r["seq_len"], r["cache_mb"]))
    for i, (bs, pts) in enumerate(sorted(by_bs.items())):
        pts.sort()
        ch.line([p[0] for p in pts], [p[1] for p in pts], f"batch {bs}", PALETTE[i % len(PALETTE)])
    mb = next((r["model_bytes"] for r in bench["kv_cache"] if r.get("model_bytes")), None)
    if mb:
        ch.hline(mb / 1e6, "model weights")
    return ch.save(path)


def fig_quantization(quant: dict[str, Any], path) -> Path:
    rows = quant["rows"]
    return BarChart(title="Quantization: held-out perplexity (mean +- std over chunks)", xlabel="perplexity",
                    labels=[f"{r['label']} ({r['compression_ratio']:.1f}x)" for r in rows],
                    values=[r["ppl_mean"] for r in rows], errors=[r["ppl_std"] for r in rows],
                    reference=rows[0]["ppl_mean"] if rows else None).save(path)


def fig_pruning_pareto(prune: dict[str, Any], path) -> Path:
    ch = LineChart(title="Structured pruning: loss vs parameters removed", xlabel="fraction of parameters removed",
                   ylabel="val loss")
    for i, kind in enumerate(("heads", "neurons")):
        pts = sorted((r["fraction_removed"], r["val_loss"]) for r in prune["rows"] if r["kind"] == kind)
        if pts:
            ch.line([p[0] for p in pts], [p[1] for p in pts], kind, PALETTE[i])
    return ch.save(path)


def fig_distillation(dist: dict[str, Any], path) -> Path:
    ch = LineChart(title="Distillation: student validation loss", xlabel="step", ylabel="val loss")
    for i, run in enumerate(dist["runs"]):
        h = run["history"]
        ch.line([r["step"] for r in h], [r["val_loss"] for r in h], f"{run['label']} (alpha={run['alpha']})",
                PALETTE[i % len(PALETTE)])
    return ch.save(path)


def fig_pareto(pareto: dict[str, Any], path) -> Path:
    """Quality vs size across compression methods (points: size_mb, ppl)."""
    ch = LineChart(title="Quality / size Pareto", xlabel="model size (MB)", ylabel="perplexity", xlog=True)
    by: dict = {}
    for p in pareto["points"]:
        by.setdefault(p["method"], []).append((p["size_mb"], p["ppl"]))
    for i, (m, pts) in enumerate(sorted(by.items())):
        pts.sort()
        ch.line([a for a, _ in pts], [b for _, b in pts], m, PALETTE[i % len(PALETTE)])
    return ch.save(path)


def fig_parallel_bubble(payload: dict[str, Any], path) -> Path:
    """Measured pipeline bubble vs micro-batches, with (p-1)/(m+p-1)."""
    rows = payload["rows"]
    ch = LineChart(title="Pipeline bubble", xlabel="micro-batches m", ylabel="bubble fraction")
    for i, sched in enumerate(sorted({r["schedule"] for r in rows})):
        pts = sorted((r["micro_batches"], r["measured_bubble"]) for r in rows if r["schedule"] == sched)
        ch.line([a for a, _ in pts], [b for _, b in pts], f"{sched} measured", PALETTE[i])
    ms = sorted({r["micro_batches"] for r in rows})
    p = rows[0]["stages"]
    ch.line(ms, [(p - 1) / (m + p - 1) for m in ms], "(p-1)/(m+p-1)", "#222", dashed=True)
    return ch.save(path)


def fig_scaling(lines: list[dict[str, Any]], path) -> Path:
    """Tokens/s vs GPUs from ``bench.py`` JSON lines, with linear scaling."""
    pts = sorted((l["n_gpus"], l["value"]) for l in lines if "value" in l and "n_gpus" in l)
    ch = LineChart(title="Training throughput vs GPUs (B200)", xlabel="GPUs", ylabel="tokens/s")
    if pts:
        ch.line([a for a, _ in pts], [b for _, b in pts], "measured", PALETTE[0])
        ch.line([a for a, _ in pts], [pts[0][1] * a / pts[0][0] for a, _ in pts], "linear", "#888", dashed=True)
    return ch.save(path)


_MAKERS = {"verification.json": fig_verification, "induction.json": fig_induction_heatmap,
           "ablations.json": fig_ablations, "kv_cache.json": fig_kv_latency, "quantization.json": fig_quantization,
           "pruning.json": fig_pruning_pareto, "distillation.json": fig_distillation, "pareto.json": fig_pareto,
           "pipeline_bubble.json": fig_parallel_bubble}


def make_all(results_dir, out_dir) -> list[Path]:
    """Redraw every figure whose payload exists under ``results_dir``."""
    rd, od = Path(results_dir), Path(out_dir)
    out = []
    for name, fn in _MAKERS.items():
        f = rd / name
        if f.exists():
            payload = json.loads(f.read_text())
            out.append(fn(payload, od / name.replace(".json", ".svg")))
            if name == "kv_cache.json" and "kv_cache" in payload:
                out.append(fig_kv_memory(payload, od / "kv_memory.svg"))
    scale = rd / "scaling.jsonl"
    if scale.exists():
        lines = [json.loads(l) for l in scale.read_text().splitlines() if l.strip()]
        out.append(fig_scaling(lines, od / "scaling.svg"))
    return out


if __name__ == "__main__":
    for p in make_all(sys.argv[1] if len(sys.argv) > 1 else "results", sys.argv[2] if len(sys.argv) > 2 else "figures"):
        print(p)
