"""Performance diagnosis: where a training step's time goes, ranked.

Reference: src/transformer_internals/perf/diagnose.py:82-957. Findings are
fractions of the step's wall clock, graded by fixed bands (>= 0.30 critical,
>= 0.10 significant, >= 0.03 minor, else healthy) and sorted by cost, each
with the measurements behind it and a recommendation:

* dataloader stall: fetch vs compute timed separately (a loader with an
  injectable stall gives the control arm);
* exposed collective time: a four-arm probe on real ranks (no comm; manual
  per-tensor all-reduce after backward; bucketed overlap at 25 MB and 1 MB),
  timed round robin (each arm sees the same ambient load), minimum statistic,
  each arm compared with a standalone issue of the same call pattern;
* memory-bound operator share (profiler categories) against the roofline
  ceiling of the op mix;
* batch saturation: throughput vs batch size.

On B200 the probe's GPU arms are the native engine with its fused P2P
all-reduce and with NCCL, both overlapped with backward.

    python -m gpt2_harness_b200.perf.diagnose --world 2
"""

from __future__ import annotations

import argparse
import json
import statistics
import time
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

import torch

from ..config import GPTConfig
from ..models.gpt import GPT
from .mfu import flops_per_token_exact
from .roofline import MachinePeak, op_roofline_table

__all__ = ["SEVERITY_BANDS", "severity", "SyntheticLoader", "StepBreakdown", "measure_step_breakdown",
           "sweep_batch_throughput", "collective_probe", "Finding", "DiagnosisReport", "diagnose"]

SEVERITY_BANDS = (0.30, 0.10, 0.03)


def severity(fraction: float) -> str:
    hi, mid, lo = SEVERITY_BANDS
    return "critical" if fraction >= hi else "significant" if fraction >= mid else "minor" if fraction >= lo \
        else "healthy"


def _sync(dev: torch.device) -> None:
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


class SyntheticLoader:
    """Random (x, y) batches that block ``stall_s`` seconds each (an IO-bound
    loader: the process sleeps, no CPU is stolen from compute)."""

    def __init__(self, vocab_size: int, batch: int, seq: int, device="cpu", stall_s: float = 0.0, seed: int = 0):
        self.vocab_size, self.batch, self.seq = vocab_size, batch, seq
        self.device = torch.device(device)
        self.stall_s = float(stall_s)
        self.generator = torch.Generator().manual_seed(seed)
        self.batches_served = 0

    def __iter__(self):
        return self

    def __next__(self):
        if self.stall_s > 0:
            time.sleep(self.stall_s)
        ids = torch.randint(0, self.vocab_size, (self.batch, self.seq + 1), generator=self.generator)
        self.batches_served += 1
        return ids[:, :-1].contiguous().to(self.device), ids[:, 1:].contiguous().to(self.device)


@dataclass
class StepBreakdown:
    """Fetch and compute seconds per timed step; the headline statistic is
    the minimum (contention only ever adds time), all samples are kept."""
    steps: int
    fetch_s: list = field(default_factory=list)
    compute_s: list = field(default_factory=list)

    @property
    def best_fetch_s(self) -> float:
        return min(self.fetch_s)

    @property
    def best_compute_s(self) -> float:
        return min(self.compute_s)

    @property
    def best_step_s(self) -> float:
        return self.best_fetch_s + self.best_compute_s

    @property
    def stall_fraction(self) -> float:
        return self.best_fetch_s / self.best_step_s

    def to_dict(self) -> dict:
        return {"steps": self.steps, "statistic": "minimum over the timed steps", "fetch_s": self.fetch_s,
                "compute_s": self.compute_s, "best_fetch_s": self.best_fetch_s, "best_compute_s": self.best_compute_s,
                "best_step_s": self.best_step_s, "median_fetch_s": statistics.median(self.fetch_s),
                "median_compute_s": statistics.median(self.compute_s), "stall_fraction": self.stall_fraction}


def measure_step_breakdown(step, loader, steps: int = 8, warmup: int = 2, device="cpu") -> StepBreakdown:
    """``step(x, y)`` runs one optimiser step (oracle or native). The device
    is synchronised after the compute, not between fetch and compute."""
    dev = torch.device(device)
    for _ in range(warmup):
        step(*next(loader))
    _sync(dev)
    out = StepBreakdown(steps)
    for _ in range(steps):
        t0 = time.perf_counter()
        x, y = next(loader)
        t1 = time.perf_counter()
        step(x, y)
        _sync(dev)
        t2 = time.perf_counter()
        out.fetch_s.append(t1 - t0)
        out.compute_s.append(t2 - t1)
    return out


def _oracle_step(model: GPT):
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4)

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        model(x, targets=y)["loss"].backward()
        opt.step()
    return step


def sweep_batch_throughput(cfg: GPTConfig, batch_sizes, seq: int, device="cpu", steps: int = 3, warmup: int = 1,
                           model: Optional[GPT] = None) -> list[dict]:
    dev = torch.device(device)
    model = (model or GPT(cfg)).to(dev).train()
    step = _oracle_step(model)
    rows = []
    for b in batch_sizes:
        x = torch.randint(0, cfg.vocab_size, (b, seq), device=dev)
        y = torch.randint(0, cfg.vocab_size, (b, seq), device=dev)
        for _ in range(warmup):
            step(x, y)
        _sync(dev)
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            step(x, y)
            _sync(dev)
            ts.append(time.perf_counter() - t0)
        rows.append({"batch": b, "step_s": min(ts), "tokens_per_s": b * seq / min(ts)})
    return rows


# ------------------------------------------------------- collective probe --
def _probe_worker(rank: int, world: int, model_config: dict, batch: int, seq: int, steps: int, warmup: int,
                  small_bucket_mb: float = 1.0) -> dict:
    """One rank of the collective probe (oracle model, any backend)."""
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    cfg = GPTConfig(**model_config)
    g = torch.Generator().manual_seed(rank)
    x = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g).to(dev)
    y = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g).to(dev)

    def fresh():
        torch.manual_seed(0)
        m = GPT(cfg).to(dev)
        return m, torch.optim.AdamW(m.parameters(), lr=1e-4)

    model, opt = fresh()
    params = [p for p in model.parameters() if p.requires_grad]
    n_el = sum(p.numel() for p in params)

    def local():
        opt.zero_grad(set_to_none=True)
        model(x, targets=y)["loss"].backward()
        opt.step()

    def manual():
        opt.zero_grad(set_to_none=True)
        model(x, targets=y)["loss"].backward()
        for p in params:
            dist.all_reduce(p.grad)
            p.grad /= world
        opt.step()

    arms = {"no_comm": local, "manual_allreduce": manual}
    keep = []
    for name, cap in (("ddp_default_buckets", 25), ("ddp_small_buckets", small_bucket_mb)):
        m, _ = fresh()
        d = DDP(m, bucket_cap_mb=cap)
        o = torch.optim.AdamW(d.parameters(), lr=1e-4)
        keep.append((m, d, o))

        def f(d=d, o=o):
            o.zero_grad(set_to_none=True)
            d(x, targets=y)["loss"].backward()
            o.step()
        arms[name] = f
    flat = torch.zeros(n_el, device=dev)
    per = [torch.zeros_like(p) for p in params]
    chunks = list(torch.split(flat, int(small_bucket_mb * (1 << 20)) // 4))
    arms["standalone_flat"] = lambda: dist.all_reduce(flat)
    arms["standalone_per_param"] = lambda: [dist.all_reduce(t) for t in per]
    arms["standalone_chunks"] = lambda: [dist.all_reduce(c) for c in chunks]
    for fn in arms.values():
        for _ in range(warmup):
            fn()
    _sync(dev)
    samples = {k: [] for k in arms}
    for _ in range(steps):
        for k, fn in arms.items():  # round robin: every arm sees the same ambient load
            dist.barrier()
            t0 = time.perf_counter()
            fn()
            _sync(dev)
            samples[k].append(time.perf_counter() - t0)
    return {"samples": samples, "n_grad_elements": n_el, "n_grad_tensors": len(params), "device": str(dev)}


def collective_probe(model_config: Optional[dict] = None, world_size: int = 2, batch: int = 2, seq: int = 64,
                     steps: int = 10, warmup: int = 3, backend: Optional[str] = None,
                     timeout_s: float = 600.0) -> dict[str, Any]:
    """Exposed collective time and overlap per arm (rank 0's samples)."""
    from ..parallel.comms import spawn_workers
    mc = model_config or GPTConfig(vocab_size=512, n_positions=seq, n_layer=2, n_head=2, n_embd=64).to_dict()
    res = spawn_workers(_probe_worker, world_size, dict(model_config=mc, batch=batch, seq=seq, steps=steps,
                                                        warmup=warmup), backend=backend, timeout=timeout_s)
    r0 = res[0].value
    best = {k: min(v) for k, v in r0["samples"].items()}
    floor = best["no_comm"]
    refs = {"manual_allreduce": "standalone_per_param", "ddp_default_buckets": "standalone_flat",
            "ddp_small_buckets": "standalone_chunks"}
    out: dict[str, Any] = {"world_size": world_size, "backend": res[0].backend,
                           "statistic": "minimum over round-robin timed steps",
                           "grad_bytes": r0["n_grad_elements"] * 4, "n_grad_tensors": r0["n_grad_tensors"],
                           "best_step_s": best, "samples": r0["samples"]}
    for arm, ref in refs.items():
        exposed = max(0.0, best[arm] - floor)
        comm = best[ref]
        out[arm] = {"step_s": best[arm], "step_without_comm_s": floor, "exposed_comm_s": exposed,
                    "exposed_fraction_of_step": exposed / best[arm], "standalone_comm_s": comm,
                    "reference_pattern": ref, "cost_beyond_standalone_s": exposed - comm,
                    "overlap_fraction": max(0.0, min(1.0, 1.0 - exposed / comm)) if comm > 0 else 0.0}
    return out


# ---------------------------------------------------------------- findings --
@dataclass
class Finding:
    name: str
    severity: str
    cost_fraction: float
    recoverable: bool
    headline: str
    evidence: dict = field(default_factory=dict)
    recommendation: str = ""

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass
class DiagnosisReport:
    label: str
    device: str
    shape: dict = field(default_factory=dict)
    throughput: dict = field(default_factory=dict)
    findings: list = field(default_factory=list)
    measurements: dict = field(default_factory=dict)
    meta: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["findings"] = [f.to_dict() for f in self.findings]
        return d

    def text(self) -> str:
        t = self.throughput
        lines = [f"diagnosis: {self.label}",
                 f"  device {self.device}  batch={self.shape.get('batch')} seq={self.shape.get('seq')}  "
                 f"{t.get('tokens_per_s', 0):,.0f} tokens/s  step {t.get('step_s', 0) * 1e3:.1f} ms  "
                 f"MFU {t.get('mfu_end_to_end', 0) * 100:.2f}% of {t.get('peak_flops_per_s', 0) / 1e12:.1f} TFLOP/s",
                 f"  roofline ceiling of this op mix: {t.get('roofline_ceiling_mfu', 0) * 100:.1f}%", "",
                 "  ranked findings (share of the step):"]
        for i, f in enumerate(self.findings, 1):
            lines.append(f"   {i}. [{f.severity:>11}] {f.cost_fraction * 100:5.1f}%  {f.name}"
                         + ("" if f.recoverable else "  [not recoverable by scheduling]"))
            lines.append(f"        {f.headline}")
            if f.recommendation:
                lines.append(f"        -> {f.recommendation}")
        return "\n".join(lines)


def diagnose(peak: MachinePeak, cfg: Optional[GPTConfig] = None, batch: int = 4, seq: int = 128, device="cpu",
             label: str = "run", loader_stall_s: float = 0.0, steps: int = 6, warmup: int = 2,
             batch_sweep=(1, 2, 4, 8), profile_ops: bool = True, collectives: Optional[dict] = None,
             collective_arm: str = "ddp_default_buckets", model: Optional[GPT] = None) -> DiagnosisReport:
    dev = torch.device(device)
    cfg = cfg or GPTConfig(n_layer=4, n_head=4, n_embd=256, vocab_size=4096, n_positions=max(seq, 64))
    model = (model or GPT(cfg)).to(dev).train()
    step = _oracle_step(model)
    loader = SyntheticLoader(cfg.vocab_size, batch, seq, dev, loader_stall_s)
    bd = measure_step_breakdown(step, loader, steps, warmup, dev)
    fpt = flops_per_token_exact(cfg, seq)["training_flops_per_token"]
    flops = fpt * batch * seq
    rows = op_roofline_table(peak, cfg, batch, seq)
    ceiling = (sum(r.flops for r in rows) / sum(r.roofline_seconds for r in rows)) / peak.peak_flops_per_s
    step_s = bd.best_step_s
    rep = DiagnosisReport(label, str(dev), {"batch": batch, "seq": seq, "config": cfg.to_dict()})
    rep.throughput = {"step_s": step_s, "tokens_per_s": batch * seq / step_s, "model_flops_per_step": flops,
                      "mfu_end_to_end": flops / step_s / peak.peak_flops_per_s,
                      "mfu_compute_only": flops / bd.best_compute_s / peak.peak_flops_per_s,
                      "peak_flops_per_s": peak.peak_flops_per_s, "roofline_ceiling_mfu": ceiling}
    rep.measurements["step_breakdown"] = bd.to_dict()
    f = bd.stall_fraction
    rep.findings.append(Finding(
        "dataloader stall", severity(f), f, True,
        f"{f * 100:.1f}% of the step blocked in next(loader) ({bd.best_fetch_s * 1e3:.1f} ms fetch vs "
        f"{bd.best_compute_s * 1e3:.1f} ms compute)",
        {"fetch_ms": bd.best_fetch_s * 1e3, "compute_ms": bd.best_compute_s * 1e3,
         "injected_stall_ms": loader_stall_s * 1e3},
        "prefetch on a background thread into pinned buffers (cluster.streaming.ShardedStream(prefetch=...))"
        if f >= SEVERITY_BANDS[2] else "input pipeline keeps up"))
    if collectives is not None:
        arm = collectives[collective_arm]
        ef = arm["exposed_fraction_of_step"]
        rep.findings.append(Finding(
            f"exposed collective time ({collective_arm})", severity(ef), ef, True,
            f"{ef * 100:.1f}% of the step is all-reduce not hidden behind compute; overlap "
            f"{arm['overlap_fraction'] * 100:.0f}%",
            {k: arm[k] for k in ("step_s", "step_without_comm_s", "exposed_comm_s", "standalone_comm_s",
                                 "overlap_fraction")},
            "launch bucketed all-reduces from backward hooks (NativeDDP) and size buckets so the first "
            "starts early" if arm["overlap_fraction"] < 0.5 else "communication already overlaps backward"))
    if profile_ops:
        from .profiling import profile_training_step
        x, y = next(SyntheticLoader(cfg.vocab_size, batch, seq, dev))
        prof = profile_training_step(lambda: step(x, y), wait=0, warmup=1, active=1)
        mb = prof.memory_bound_fraction() * bd.best_compute_s / step_s
        rep.measurements["profile_categories"] = prof.categories
        rep.findings.append(Finding(
            "memory-bound operators", severity(mb), mb, False,
            f"{mb * 100:.1f}% of the step in operators with no tensor-core work; the op mix's roofline "
            f"ceiling is {ceiling * 100:.1f}% MFU",
            {"categories": prof.categories},
            "fuse them into GEMM epilogues / prologues (the native engine does: bias, GELU, residual, LN)"))
    if batch_sweep:
        sw = sweep_batch_throughput(cfg, batch_sweep, seq, dev, model=model)
        rep.measurements["batch_sweep"] = sw
        if len(sw) >= 2:
            gain = sw[-1]["tokens_per_s"] / sw[-2]["tokens_per_s"] - 1.0
            at = next((r for r in sw if r["batch"] == batch), None)
            lost = 1.0 - at["tokens_per_s"] / max(r["tokens_per_s"] for r in sw) if at else 0.0
            rep.findings.append(Finding(
                "batch below saturation", severity(max(0.0, lost)), max(0.0, lost), True,
                f"throughput still rises {gain * 100:.0f}% at the largest batch; this run's batch reaches "
                f"{(1 - lost) * 100:.0f}% of the best", {"sweep": sw},
                "raise the micro-batch (or accumulate) until throughput flattens" if lost > 0.03 else
                "batch is at the saturation knee"))
    rep.findings.sort(key=lambda f: -f.cost_fraction)
    return rep


def _main() -> None:
    ap = argparse.ArgumentParser(description="diagnose a training configuration")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--stall-ms", type=float, default=0.0)
    ap.add_argument("--world", type=int, default=0, help="run the collective probe with this many ranks")
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    from .roofline import measure_machine_peak, peak_from_file
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    peak = peak_from_file() if dev == "cuda" else measure_machine_peak("cpu", gemm_sizes=(256, 512),
                                                                      stream_sizes_mib=(16, 64))
    coll = collective_probe(world_size=a.world) if a.world > 1 else None
    rep = diagnose(peak, batch=a.batch, seq=a.seq, device=dev, loader_stall_s=a.stall_ms / 1e3, collectives=coll)
    print(rep.text())
    if a.json:
        with open(a.json, "w") as fh:
            json.dump(rep.to_dict(), fh, indent=1, default=str)


if __name__ == "__main__":
    _main()
