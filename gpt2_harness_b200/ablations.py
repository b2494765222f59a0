"""Architecture ablations: nine arms x several seeds, one verdict rule.

Reference: src/transformer_internals/ablations.py:50-300. Each arm changes
one ``GPTConfig`` switch from a shared small baseline (6 layers, 8x32 heads,
4096-token compact vocabulary, 250 steps); every arm trains on identical
batches (seeded generators). Verdict: an arm is *distinguishable* only when
|mean delta| exceeds the pooled std of the two arms (with three seeds a
significance test has no power, so effect and noise are reported together).

``run_grid(..., backend="native")`` trains arms whose architecture the B200
engine supports (pre-LN, tied, learned positions, GELU-tanh, head_dim 64) on
the native kernels; the others fall back to the oracle and say so in meta.
"""

from __future__ import annotations

import json
import statistics
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Optional

from .config import GPTConfig, TrainConfig
from .train import TrainResult, train

__all__ = ["BASELINE_MODEL", "BASELINE_TRAIN", "Arm", "build_arms", "run_arm", "run_grid", "summarize",
           "save_results"]

BASELINE_MODEL = GPTConfig(vocab_size=4096, n_positions=128, n_layer=6, n_head=8, n_embd=256, dropout=0.0)
BASELINE_TRAIN = TrainConfig(steps=250, batch_size=24, block_size=96, lr=3e-4, warmup_steps=50, eval_interval=50,
                             eval_batches=10)


@dataclass
class Arm:
    key: str
    label: str
    group: str
    overrides: dict = field(default_factory=dict)
    is_baseline: bool = False
    note: str = ""

    def config(self, base: GPTConfig = BASELINE_MODEL) -> GPTConfig:
        return GPTConfig(**{**base.to_dict(), **self.overrides})


def build_arms() -> list[Arm]:
    """Baseline first; six questions, nine configurations."""
    return [
        Arm("baseline", "GPT-2 defaults", "baseline", {}, True,
            "pre-LN, tied embeddings, learned positions, 8 heads of 32, scaled residual init, GELU-tanh"),
        Arm("post_ln", "post-LN", "norm_position", {"norm_position": "post"}, note="LayerNorm after the residual add"),
        Arm("untied", "untied embeddings", "tie_weights", {"tie_weights": False},
            note="separate output head (+vocab x n_embd parameters)"),
        Arm("sinusoidal", "sinusoidal positions", "pos_embedding", {"pos_embedding": "sinusoidal"},
            note="fixed sin/cos position table"),
        Arm("heads_16x16", "16 heads x 16 dim", "n_head", {"n_head": 16}, note="same width, narrower heads"),
        Arm("heads_4x64", "4 heads x 64 dim", "n_head", {"n_head": 4}, note="same width, wider heads"),
        Arm("heads_2x128", "2 heads x 128 dim", "n_head", {"n_head": 2}, note="same width, very wide heads"),
        Arm("no_resid_init", "no residual-scaled init", "residual_scaled_init", {"residual_scaled_init": False},
            note="residual projections at 0.02 instead of 0.02/sqrt(2L)"),
        Arm("relu", "ReLU", "activation", {"activation": "relu"}, note="ReLU MLP instead of GELU-tanh"),
    ]


def _native_ok(cfg: GPTConfig) -> bool:
    return (cfg.norm_position == "pre" and cfg.tie_weights and cfg.pos_embedding == "learned"
            and cfg.activation == "gelu_tanh" and cfg.n_embd // cfg.n_head == 64 and cfg.n_kv_head in (None, cfg.n_head))


def run_arm(arm: Arm, dataset, seed: int, base_model: GPTConfig = BASELINE_MODEL,
            base_train: TrainConfig = BASELINE_TRAIN, device=None, progress: bool = False,
            backend: str = "oracle") -> TrainResult:
    mcfg = arm.config(base_model)
    tcfg = TrainConfig(**{**base_train.to_dict(), "seed": seed})
    be = backend if backend == "oracle" or _native_ok(mcfg) else "oracle"
    _, res = train(mcfg, tcfg, dataset, device=device, progress=progress, backend=be)
    res.meta.update({"arm": arm.key, "label": arm.label, "group": arm.group, "note": arm.note, "seed": seed,
                     "backend_requested": backend, "backend_used": be})
    return res


def run_grid(dataset, seeds=(0, 1, 2), arms: Optional[list[Arm]] = None, **kw) -> dict[str, list[TrainResult]]:
    arms = arms or build_arms()
    return {a.key: [run_arm(a, dataset, s, **kw) for s in seeds] for a in arms}


def summarize(results: dict, arms: list[Arm]) -> dict[str, Any]:
    """One row per arm: mean/std final val loss, delta vs baseline, verdict,
    wall-clock ratio, divergence count and gradient-norm statistics."""
    def stats(key):
        losses = [r.final_val_loss for r in results[key]]
        walls = [r.wall_clock_s for r in results[key]]
        return (statistics.fmean(losses), statistics.stdev(losses) if len(losses) > 1 else 0.0,
                statistics.fmean(walls), losses)

    ref = "baseline" if results.get("baseline") else next(iter(results))
    bm, bs, bw, _ = stats(ref)
    rows = []
    for arm in arms:
        if not results.get(arm.key):
            continue
        m, s, w, losses = stats(arm.key)
        d = m - bm
        pooled = (s * s + bs * bs) ** 0.5
        verdict = ("reference" if arm.key == ref else "indistinguishable" if abs(d) <= pooled
                   else "worse" if d > 0 else "better")
        gn = [g for r in results[arm.key] for g in r.grad_norms]
        rows.append({"arm": arm.key, "label": arm.label, "group": arm.group, "note": arm.note,
                     "n_seeds": len(losses), "n_params": results[arm.key][0].n_params, "val_loss_mean": m,
                     "val_loss_std": s, "val_losses": losses, "delta_vs_baseline": d, "pooled_std": pooled,
                     "verdict": verdict, "wall_clock_s_mean": w, "wall_clock_ratio": w / bw if bw else float("nan"),
                     "diverged_seeds": sum(r.diverged for r in results[arm.key]),
                     "max_grad_norm": max(gn) if gn else 0.0, "mean_grad_norm": statistics.fmean(gn) if gn else 0.0})
    return {"reference_arm": ref, "rows": rows,
            "verdict_rule": "distinguishable only if |delta| > pooled std of the two arms"}


def save_results(path, payload: dict) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_suffix(p.suffix + ".tmp")
    tmp.write_text(json.dumps(payload, indent=1, default=lambda o: o.to_dict() if hasattr(o, "to_dict") else str(o)))
    tmp.replace(p)
