"""Model FLOPs utilisation.

The numerator follows the reference's operator-by-operator count
(src/transformer_internals/perf/mfu.py:111-171) so MFU figures of the two
frameworks are comparable: per token per layer the forward projections cost
2C(C+2kv) + 2C^2 + 2*(2*4C^2), the attention quadratic term 2*(2TC) (halved
only when ``causal_aware``), the tied head 2CV; training is 3x forward. The
denominator is a measured peak (MEASURED_PEAKS.json's cuBLAS bf16 figure on
this pool) or a published accelerator peak.
"""

from __future__ import annotations

import json
import os
import time
from dataclasses import asdict, dataclass
from typing import Callable, Optional

from gpt2_harness_b200.config import GPTConfig

__all__ = [
    "PUBLISHED_ACCELERATORS",
    "flops_6nd",
    "flops_per_token_exact",
    "param_count",
    "MFUReport",
    "measured_peak_tflops",
    "mfu_on_published_gpu",
    "measure_step_mfu",
]

#: Dense (no 2:4 sparsity) peak TFLOP/s by dtype, from vendor datasheets.
PUBLISHED_ACCELERATORS: dict[str, dict[str, float]] = {
    "A100-SXM": {"bf16": 312.0, "fp16": 312.0, "tf32": 156.0, "fp32": 19.5},
    "H100-SXM": {"bf16": 989.0, "fp16": 989.0, "tf32": 494.0, "fp32": 67.0},
    "H200-SXM": {"bf16": 989.0, "fp16": 989.0, "tf32": 494.0, "fp32": 67.0},
    "B200": {"bf16": 2250.0, "fp16": 2250.0, "fp8": 4500.0, "fp4": 9000.0, "tf32": 1100.0},
}


def flops_6nd(n_params: int, n_tokens: int) -> float:
    """The 6ND estimate of training FLOPs."""
    return 6.0 * n_params * n_tokens


def param_count(cfg: GPTConfig, non_embedding: bool = False) -> int:
    """Analytic parameter count (tied head counted once)."""
    c, v, p, L = cfg.n_embd, cfg.vocab_size, cfg.n_positions, cfg.n_layer
    kv = cfg.kv_heads * cfg.head_dim
    per = c * (c + 2 * kv) + ((c + 2 * kv) if cfg.attn_bias else 0)
    per += c * c + (c if cfg.attn_bias else 0)
    per += 4 * c * c + (4 * c if cfg.mlp_bias else 0)
    per += 4 * c * c + (c if cfg.mlp_bias else 0)
    per += 4 * c
    total = L * per + 2 * c + v * c
    if cfg.pos_embedding == "learned":
        total += p * c
    if not cfg.tie_weights:
        total += v * c
    if non_embedding:
        total -= v * c
        if cfg.pos_embedding == "learned":
            total -= p * c
    return total


def flops_per_token_exact(cfg: GPTConfig, seq_len: int, causal_aware: bool = False) -> dict:
    """Per-token training FLOPs by operator (see module docstring)."""
    c = float(cfg.n_embd)
    t = float(seq_len)
    kv = float(cfg.kv_heads * cfg.head_dim)
    proj = 2 * c * (c + 2 * kv) + 2 * c * c + 2 * (4 * c * c) * 2
    quad = 2 * (2 * t * c)
    if causal_aware:
        quad /= 2
    L = float(cfg.n_layer)
    head = 2 * c * float(cfg.vocab_size)
    fwd_params = L * proj + head
    fwd_attn = L * quad
    fwd = fwd_params + fwd_attn
    n_total = param_count(cfg)
    n_ne = param_count(cfg, non_embedding=True)
    return {
        "seq_len": t,
        "forward_projection_flops_per_token": fwd_params,
        "forward_attention_quadratic_flops_per_token": fwd_attn,
        "forward_total_flops_per_token": fwd,
        "training_flops_per_token": 3 * fwd,
        "training_attention_quadratic_flops_per_token": 3 * fwd_attn,
        "attention_quadratic_fraction": fwd_attn / fwd,
        "n_params_total": float(n_total),
        "n_params_non_embedding": float(n_ne),
        "flops_6n_total_per_token": 6.0 * n_total,
        "flops_6n_non_embedding_per_token": 6.0 * n_ne,
        "ratio_to_6nd_total": 3 * fwd / (6.0 * n_total),
        "causal_aware": float(causal_aware),
    }


def measured_peak_tflops(path: Optional[str] = None, sustained: bool = True) -> tuple[float, str]:
    """bf16 dense peak measured on this pool (MEASURED_PEAKS.json), with its
    provenance label; falls back to 1415 TFLOP/s sustained / 1590 burst."""
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    path = path or os.path.join(here, "MEASURED_PEAKS.json")
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    try:
        with open(path) as f:
            data = json.load(f)
        return float(data[key]), f"measured ({key})"
    except (OSError, KeyError, ValueError):
        return (1400.0 if sustained else 1590.0), "fallback"


@dataclass
class MFUReport:
    tokens_per_step: int
    step_time_s: float
    flops_per_token: float
    achieved_tflops: float
    peak_tflops: float
    peak_label: str
    mfu: float

    @property
    def tokens_per_s(self) -> float:
        return self.tokens_per_step / self.step_time_s

    def as_dict(self) -> dict:
        d = asdict(self)
        d["tokens_per_s"] = self.tokens_per_s
        return d


def mfu_on_published_gpu(flops_per_token: float, tokens_per_s: float, gpu: str = "B200",
                         dtype: str = "bf16") -> float:
    """MFU against a datasheet peak (labelled MODELLED by callers)."""
    return flops_per_token * tokens_per_s / (PUBLISHED_ACCELERATORS[gpu][dtype] * 1e12)


def measure_step_mfu(step_fn: Callable[[], None], cfg: GPTConfig, batch: int, seq_len: int,
                     steps: int = 10, warmup: int = 3, sync: Optional[Callable[[], None]] = None,
                     peak_tflops: Optional[float] = None, n_gpus: int = 1) -> MFUReport:
    """Time `step_fn` (minimum over steps) and report MFU."""
    sync = sync or (lambda: None)
    for _ in range(warmup):
        step_fn()
    sync()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step_fn()
        sync()
        times.append(time.perf_counter() - t0)
    dt = min(times)
    fpt = flops_per_token_exact(cfg, seq_len)["training_flops_per_token"]
    label = "given"
    if peak_tflops is None:
        peak_tflops, label = measured_peak_tflops()
    tokens = batch * seq_len * n_gpus
    achieved = fpt * tokens / dt / 1e12
    return MFUReport(tokens, dt, fpt, achieved, peak_tflops * n_gpus, label,
                     achieved / (peak_tflops * n_gpus))
