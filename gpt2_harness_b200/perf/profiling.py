"""Training-step profiling: per-kernel device time, folded into categories.

Reference: src/transformer_internals/perf/profiling.py:57-294 (torch.profiler
with a wait/warmup/active schedule, self-time top-K, category fold, Chrome
trace). Here the same wrapper also understands the native sm_100a kernels by
name, so a step of the B200 engine breaks down into GEMM / attention /
LayerNorm / loss / optimiser / communication shares.

Device times come from CUPTI through torch.profiler; they are for SHARES, not
for the headline number (bench.py times with CUDA events, outside any
profiler).

    python -m gpt2_harness_b200.perf.profiling --batch 16 --seq 1024
"""

from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass, field
from typing import Callable, Optional

import torch

__all__ = ["OP_CATEGORIES", "categorize_op", "ProfileReport", "profile_training_step",
           "profile_native_step"]

#: Category -> substrings of kernel / op names (first match wins, in order).
OP_CATEGORIES: dict[str, tuple[str, ...]] = {
    "matmul": ("gemm_tcgen05", "splitk_reduce", "gemm", "matmul", "mm", "addmm", "bmm", "linear",
               "cutlass", "sm90_xmma", "sm100_xmma", "nvjet", "cublas"),
    "attention": ("attn_", "flash", "sdpa", "scaled_dot_product", "softmax"),
    "normalization": ("ln_fwd", "ln_bwd", "layer_norm", "layernorm", "colsum"),
    "loss": ("ce_kernel", "loss_reduce", "cross_entropy", "nll", "log_softmax"),
    "optimizer": ("adamw", "sumsq", "sum_final", "clip_coef", "adam", "foreach", "multi_tensor"),
    "communication": ("allreduce", "nccl", "all_reduce", "all_gather", "reduce_scatter"),
    "embedding": ("emb_", "embedding", "index_select", "gather", "scatter", "index_add"),
    "elementwise": ("gelu", "tanh", "mul", "add", "div", "copy", "cast", "fill", "elementwise",
                    "vectorized", "reduce"),
}


def categorize_op(name: str) -> str:
    low = name.lower()
    for cat, keys in OP_CATEGORIES.items():
        if any(k in low for k in keys):
            return cat
    return "other"


@dataclass
class ProfileReport:
    total_device_us: float
    steps: int
    top: list = field(default_factory=list)          # (name, us per step, share, calls/step)
    categories: dict = field(default_factory=dict)   # category -> share
    trace_path: Optional[str] = None

    def as_dict(self) -> dict:
        return asdict(self)

    def memory_bound_fraction(self) -> float:
        """Share of kernel time in operators with no tensor-core work
        (normalisation, loss, optimiser, elementwise, embedding)."""
        return sum(v for k, v in self.categories.items()
                   if k in ("normalization", "loss", "optimizer", "elementwise", "embedding"))

    def format(self, k: int = 25) -> str:
        lines = [f"device time per step: {self.total_device_us / 1e3:.3f} ms over {self.steps} step(s)"]
        for name, us, share, calls in self.top[:k]:
            lines.append(f"  {share * 100:5.1f}%  {us / 1e3:8.3f} ms  x{calls:<4g} {name[:110]}")
        lines.append("categories: " + ", ".join(f"{c} {s * 100:.1f}%" for c, s in
                                                sorted(self.categories.items(), key=lambda x: -x[1])))
        return "\n".join(lines)


def profile_training_step(step_fn: Callable[[], None], wait: int = 1, warmup: int = 2,
                          active: int = 3, trace_path: Optional[str] = None,
                          record_shapes: bool = False) -> ProfileReport:
    """Profile `active` calls of `step_fn` (after `wait`+`warmup` untraced ones)
    and aggregate device (CUDA kernel) self time by kernel name."""
    from torch.profiler import ProfilerActivity, profile, schedule

    acts = [ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(ProfilerActivity.CUDA)
    sched = schedule(wait=wait, warmup=warmup, active=active, repeat=1)
    with profile(activities=acts, schedule=sched, record_shapes=record_shapes) as prof:
        for _ in range(wait + warmup + active):
            step_fn()
            if torch.cuda.is_available():
                torch.cuda.synchronize()
            prof.step()
    if trace_path:
        prof.export_chrome_trace(trace_path)
    per: dict[str, list] = {}
    on_gpu = torch.cuda.is_available()
    for ev in prof.events():
        dt = getattr(ev, "device_type", None)
        is_dev = dt is not None and str(dt).endswith("CUDA")
        if on_gpu:
            if not is_dev:
                continue
            dur = float(getattr(ev, "device_time", 0.0) or getattr(ev, "cuda_time", 0.0) or 0.0)
        else:
            # no GPU: aggregate the self CPU time of aten ops (the kernels of a CPU run)
            if is_dev or not ev.name.startswith("aten::"):
                continue
            dur = float(getattr(ev, "self_cpu_time_total", 0.0) or 0.0)
        if dur <= 0:
            continue
        rec = per.setdefault(ev.name, [0.0, 0])
        rec[0] += dur
        rec[1] += 1
    total = sum(v[0] for v in per.values()) or 1.0
    top = sorted(((n, v[0] / active, v[0] / total, v[1] / active) for n, v in per.items()),
                 key=lambda r: -r[1])
    cats: dict[str, float] = {}
    for n, v in per.items():
        c = categorize_op(n)
        cats[c] = cats.get(c, 0.0) + v[0] / total
    return ProfileReport(total / active, active, top, cats, trace_path)


def profile_native_step(batch: int = 16, seq: int = 1024, size: str = "gpt2", active: int = 3,
                        trace_path: Optional[str] = None) -> ProfileReport:
    """Profile the native engine's full training step at (batch, seq)."""
    from gpt2_harness_b200.config import TrainConfig, gpt2_config
    from gpt2_harness_b200.trainer import Trainer

    cfg = gpt2_config(size)
    tr = Trainer(cfg, batch, seq, train=TrainConfig(warmup_steps=0), schedule=False)
    idx = torch.randint(0, cfg.vocab_size, (batch, seq), device=tr.device)
    tgt = torch.randint(0, cfg.vocab_size, (batch, seq), device=tr.device)
    rep = profile_training_step(lambda: tr.step_async(idx, tgt), active=active, trace_path=trace_path)
    tr.check()
    return rep


def main() -> None:
    ap = argparse.ArgumentParser(description="profile one native training step")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--size", default="gpt2")
    ap.add_argument("--json", default=None)
    ap.add_argument("--trace", default=None)
    a = ap.parse_args()
    rep = profile_native_step(a.batch, a.seq, a.size, trace_path=a.trace)
    print(rep.format())
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rep.as_dict(), f, indent=1)


if __name__ == "__main__":
    main()
