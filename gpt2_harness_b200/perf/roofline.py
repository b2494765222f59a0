"""Roofline: machine peaks, per-operator FLOPs and bytes, and measured rates.

Reference: src/transformer_internals/perf/roofline.py:75-590 (peak FLOP/s
from a square-GEMM sweep, peak bytes/s from a STREAM triad, the ridge point
they imply, analytic per-operator FLOPs and compulsory bytes for one block,
a compute/memory classification against the ridge, and measured op rates to
check the model).

B200 additions:

* the denominators can come from ``MEASURED_PEAKS.json`` (driver-measured
  copy bandwidth and cuBLAS bf16 throughput) instead of a fresh sweep;
* two dataflows per block: ``eager`` (one kernel per primitive op, the
  reference's accounting: the T x T score matrix round-trips memory, GELU
  and residual adds are separate passes) and ``native`` (this framework's
  kernels: flash attention keeps scores on chip, bias/GELU/residual ride in
  GEMM epilogues), so the table shows what fusion buys in bytes;
* :func:`measure_op_rates` times both the eager PyTorch ops and the native
  sm_100a kernels at the same shapes.

    python -m gpt2_harness_b200.perf.roofline --batch 16 --seq 1024
"""

from __future__ import annotations

import argparse
import json
import math
import platform
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Callable, Optional

import torch

from ..config import GPTConfig

__all__ = ["ELEMENTWISE_COST", "MachinePeak", "measure_peak_flops", "measure_peak_bandwidth",
           "measure_machine_peak", "peak_from_file", "OpRoofline", "op_costs", "op_roofline_table",
           "measure_op_rates", "roofline_payload"]

#: FLOPs per element of the elementwise operators (counting convention).
ELEMENTWISE_COST = {"gelu_tanh": 9, "layernorm": 8, "softmax": 5, "residual_add": 1}


def _sync(dev: torch.device) -> None:
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


def _best_seconds(fn: Callable, dev: torch.device, repeats: int, warmup: int) -> float:
    """Minimum over repeats (the fastest run is the closest to the hardware's
    capability; slow samples are interference). CUDA events on GPUs."""
    for _ in range(warmup):
        fn()
    _sync(dev)
    best = math.inf
    for _ in range(repeats):
        if dev.type == "cuda":
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            best = min(best, a.elapsed_time(b) / 1e3)
        else:
            t0 = time.perf_counter()
            fn()
            best = min(best, time.perf_counter() - t0)
    return best


@dataclass
class MachinePeak:
    device: str
    dtype: str
    peak_flops_per_s: float
    peak_bytes_per_s: float
    ridge_flops_per_byte: float
    gemm_sweep: list = field(default_factory=list)
    bandwidth_sweep: list = field(default_factory=list)
    meta: dict = field(default_factory=dict)

    def attainable_flops_per_s(self, intensity: float) -> float:
        return min(self.peak_flops_per_s, intensity * self.peak_bytes_per_s)

    def to_dict(self) -> dict:
        return asdict(self)


def measure_peak_flops(device="cpu", sizes=(256, 512, 1024, 2048, 4096), dtype=torch.float32, repeats: int = 5,
                       warmup: int = 2):
    """Best FLOP/s over square GEMMs (2 N^3 FLOPs each)."""
    dev = torch.device(device)
    rec = []
    for n in sizes:
        a = torch.randn(n, n, device=dev, dtype=dtype)
        b = torch.randn(n, n, device=dev, dtype=dtype)
        s = _best_seconds(lambda: torch.matmul(a, b), dev, repeats, warmup)
        rec.append({"n": n, "seconds": s, "flops_per_s": 2.0 * n ** 3 / s})
    return max(r["flops_per_s"] for r in rec), rec


def measure_peak_bandwidth(device="cpu", sizes_mib=(16, 64, 256, 512), dtype=torch.float32, repeats: int = 7,
                           warmup: int = 2):
    """Best bytes/s of a triad ``a = b + s c`` (3 n elements moved); small
    sizes may sit in cache, so the per-size records show the cliff."""
    dev = torch.device(device)
    item = torch.empty((), dtype=dtype).element_size()
    rec = []
    for mib in sizes_mib:
        n = mib * 1024 * 1024 // item
        a, b, c = (torch.empty(n, device=dev, dtype=dtype), torch.randn(n, device=dev, dtype=dtype),
                   torch.randn(n, device=dev, dtype=dtype))
        s = _best_seconds(lambda: torch.add(b, c, alpha=3.0, out=a), dev, repeats, warmup)
        rec.append({"array_mib": mib, "elements": n, "seconds": s, "bytes_per_s": 3.0 * n * item / s})
    return max(r["bytes_per_s"] for r in rec), rec


def measure_machine_peak(device="cpu", dtype=torch.float32, gemm_sizes=(256, 512, 1024, 2048, 4096),
                         stream_sizes_mib=(16, 64, 256, 512)) -> MachinePeak:
    pf, g = measure_peak_flops(device, gemm_sizes, dtype)
    pb, s = measure_peak_bandwidth(device, stream_sizes_mib, dtype)
    return MachinePeak(str(device), str(dtype).replace("torch.", ""), pf, pb, pf / pb, g, s,
                       {"platform": platform.platform(), "torch": torch.__version__, "source": "measured here"})


def peak_from_file(path: Optional[str] = None, sustained: bool = True) -> MachinePeak:
    """B200 denominators from ``MEASURED_PEAKS.json`` (bf16 tensor GEMM and
    HBM copy bandwidth measured on this pool)."""
    p = Path(path) if path else Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    d = json.loads(p.read_text())
    flops = (d["bf16_tflops_sustained"] if sustained else d["bf16_tflops"]) * 1e12
    bw = d["hbm_gbs"] * 1e9
    return MachinePeak(d.get("gpu_name", "gpu"), "bf16", flops, bw, flops / bw,
                       meta={"source": str(p), "sustained": sustained, "how": d.get("how")})


@dataclass
class OpRoofline:
    name: str
    kind: str
    flops: float
    bytes_moved: float
    intensity: float
    bound: str
    attainable_flops_per_s: float
    roofline_seconds: float

    def to_dict(self) -> dict:
        return asdict(self)


def op_costs(cfg: GPTConfig, batch: int, seq: int, dtype_bytes: int = 4, dataflow: str = "eager",
             causal: bool = False) -> list[tuple[str, str, float, float]]:
    """``(name, kind, flops, bytes)`` for one block's forward.

    ``eager``: every op reads its inputs from and writes its outputs to
    memory (weights once per call); the reference's accounting.
    ``native``: this framework's kernels - LayerNorm reads the fp32 residual
    and writes bf16; bias+GELU live in the c_fc epilogue; the residual add in
    the projection epilogues (read old residual, write new); flash attention
    reads q, k, v once and writes o (scores never leave the SM). Activations
    are bf16 (``dtype_bytes`` is ignored), the residual stream fp32.
    ``causal`` halves the attention FLOPs (blocks above the diagonal skipped).
    """
    b, t, c, h = float(batch), float(seq), float(cfg.n_embd), float(cfg.n_head)
    hd = c / h
    kvc = cfg.kv_heads * hd
    act, scores = b * t * c, b * h * t * t
    att_f = (0.5 if causal else 1.0) * 2 * b * h * t * t * hd
    qkv_n = c + 2 * kvc
    if dataflow == "eager":
        d = float(dtype_bytes)
        return [
            ("ln_1 (LayerNorm)", "elementwise", ELEMENTWISE_COST["layernorm"] * act, (2 * act + 2 * c) * d),
            ("qkv projection (GEMM)", "gemm", 2 * b * t * c * qkv_n, (act + c * qkv_n + b * t * qkv_n) * d),
            ("attention scores QK^T (batched GEMM)", "batched_gemm", att_f, (act + b * t * kvc + scores) * d),
            ("softmax (+ causal mask)", "elementwise", (ELEMENTWISE_COST["softmax"] + 2) * scores, 2 * scores * d),
            ("attention x V (batched GEMM)", "batched_gemm", att_f, (scores + b * t * kvc + act) * d),
            ("output projection (GEMM)", "gemm", 2 * b * t * c * c, (2 * act + c * c) * d),
            ("residual add (attn)", "elementwise", act, 3 * act * d),
            ("ln_2 (LayerNorm)", "elementwise", ELEMENTWISE_COST["layernorm"] * act, (2 * act + 2 * c) * d),
            ("MLP up 4x (GEMM)", "gemm", 8 * b * t * c * c, (act + 4 * c * c + 4 * act) * d),
            ("GELU (tanh)", "elementwise", ELEMENTWISE_COST["gelu_tanh"] * 4 * act, 8 * act * d),
            ("MLP down (GEMM)", "gemm", 8 * b * t * c * c, (4 * act + 4 * c * c + act) * d),
            ("residual add (mlp)", "elementwise", act, 3 * act * d),
        ]
    if dataflow != "native":
        raise ValueError(f"dataflow must be 'eager' or 'native', got {dataflow!r}")
    bf, f32 = 2.0, 4.0
    return [
        ("ln_1 (native LN: fp32 in, bf16 out)", "elementwise", ELEMENTWISE_COST["layernorm"] * act,
         act * (f32 + bf) + 2 * c * f32),
        ("qkv projection + bias (tcgen05 GEMM)", "gemm", 2 * b * t * c * qkv_n,
         (act + c * qkv_n + b * t * qkv_n) * bf),
        ("flash attention fwd (tcgen05)", "attention", 2 * att_f + (ELEMENTWISE_COST["softmax"] + 2) * scores
         * (0.5 if causal else 1.0), (act + 2 * b * t * kvc + act) * bf + b * h * t * f32),
        ("output projection + residual (GEMM epilogue)", "gemm", 2 * b * t * c * c,
         act * bf + c * c * bf + 2 * act * f32),
        ("ln_2 (native LN)", "elementwise", ELEMENTWISE_COST["layernorm"] * act, act * (f32 + bf) + 2 * c * f32),
        ("MLP up + bias + GELU (GEMM epilogue, keeps pre-activation)", "gemm",
         8 * b * t * c * c + ELEMENTWISE_COST["gelu_tanh"] * 4 * act, (act + 4 * c * c + 8 * act) * bf),
        ("MLP down + residual (GEMM epilogue)", "gemm", 8 * b * t * c * c,
         (4 * act + 4 * c * c) * bf + 2 * act * f32),
    ]


def op_roofline_table(peak: MachinePeak, cfg: Optional[GPTConfig] = None, batch: int = 8, seq: int = 512,
                      dtype_bytes: int = 4, dataflow: str = "eager", causal: bool = False) -> list[OpRoofline]:
    cfg = cfg or GPTConfig()
    rows = []
    for name, kind, fl, by in op_costs(cfg, batch, seq, dtype_bytes, dataflow, causal):
        inten = fl / by
        att = peak.attainable_flops_per_s(inten)
        rows.append(OpRoofline(name, kind, fl, by, inten, "compute" if inten >= peak.ridge_flops_per_byte
                               else "memory", att, fl / att))
    return rows


def measure_op_rates(cfg: Optional[GPTConfig] = None, batch: int = 8, seq: int = 512, device="cpu",
                     dtype=torch.float32, repeats: int = 5, native: Optional[bool] = None) -> list[dict]:
    """Achieved FLOP/s of the eager PyTorch ops behind the table, and (on
    CUDA with the native library) of the fused sm_100a kernels."""
    cfg = cfg or GPTConfig()
    dev = torch.device(device)
    B, T, C, H = batch, seq, cfg.n_embd, cfg.n_head
    hd = C // H
    r = lambda *s: torch.randn(*s, device=dev, dtype=dtype)  # noqa: E731
    x, wqkv, wmlp, wout, wdown, h4 = r(B, T, C), r(C, 3 * C), r(C, 4 * C), r(C, C), r(4 * C, C), r(B, T, 4 * C)
    q, k, v = r(B, H, T, hd), r(B, H, T, hd), r(B, H, T, hd)
    probs = torch.softmax(r(B, H, T, T), dim=-1)
    ln = torch.nn.LayerNorm(C, device=dev, dtype=dtype)
    cases = [("qkv projection (GEMM)", lambda: x @ wqkv, 2.0 * B * T * C * 3 * C),
             ("output projection (GEMM)", lambda: x @ wout, 2.0 * B * T * C * C),
             ("MLP up 4x (GEMM)", lambda: x @ wmlp, 8.0 * B * T * C * C),
             ("MLP down (GEMM)", lambda: h4 @ wdown, 8.0 * B * T * C * C),
             ("attention scores QK^T (batched GEMM)", lambda: q @ k.transpose(-2, -1), 2.0 * B * H * T * T * hd),
             ("attention x V (batched GEMM)", lambda: probs @ v, 2.0 * B * H * T * T * hd),
             ("ln_1 (LayerNorm)", lambda: ln(x), 8.0 * B * T * C)]
    out = []
    for name, fn, fl in cases:
        s = _best_seconds(fn, dev, repeats, 2)
        out.append({"name": name, "impl": "eager", "seconds": s, "flops_per_s": fl / s})
    if native is None:
        native = dev.type == "cuda"
    if native:
        from ..ops import native as N
        bf = torch.bfloat16
        M = B * T
        xa = torch.randn(M, C, device=dev, dtype=bf)
        Wq = torch.randn(3 * C, C, device=dev, dtype=bf) * 0.02
        Wf = torch.randn(4 * C, C, device=dev, dtype=bf) * 0.02
        bq, bfc = torch.zeros(3 * C, device=dev, dtype=bf), torch.zeros(4 * C, device=dev, dtype=bf)
        qkv, hh, uu = (torch.empty(M, 3 * C, device=dev, dtype=bf), torch.empty(M, 4 * C, device=dev, dtype=bf),
                       torch.empty(M, 4 * C, device=dev, dtype=bf))
        o = torch.empty(M, C, device=dev, dtype=bf)
        lse = torch.empty(B, H, T, device=dev, dtype=torch.float32)
        ncases = [("qkv projection + bias (tcgen05 GEMM)", lambda: N.gemm(xa, Wq, qkv, bias=bq),
                   2.0 * M * C * 3 * C),
                  ("MLP up + bias + GELU (tcgen05 GEMM)",
                   lambda: N.gemm(xa, Wf, hh, epilogue=N.EPI_BIAS_GELU, bias=bfc, aux=uu), 8.0 * M * C * C),
                  ("flash attention fwd (tcgen05, causal)",
                   lambda: N.attention_fwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], o, lse, B, H, T),
                   2.0 * B * H * T * T * hd)]
        for name, fn, fl in ncases:
            s = _best_seconds(fn, dev, repeats, 2)
            out.append({"name": name, "impl": "native", "seconds": s, "flops_per_s": fl / s})
    return out


def roofline_payload(peak: MachinePeak, cfg: Optional[GPTConfig] = None, batch: int = 8, seq: int = 512,
                     rates: Optional[list] = None, causal: bool = True) -> dict[str, Any]:
    """JSON-ready record: peaks, both dataflows' tables, bytes saved by
    fusion, and (optionally) measured rates with their fraction of the bound."""
    cfg = cfg or GPTConfig()
    eager = op_roofline_table(peak, cfg, batch, seq, 2, "eager", causal)
    native = op_roofline_table(peak, cfg, batch, seq, 2, "native", causal)
    tot = lambda rows, k: sum(getattr(r, k) for r in rows)  # noqa: E731
    d = {"peak": peak.to_dict(), "config": cfg.to_dict(), "batch": batch, "seq": seq,
         "eager": [r.to_dict() for r in eager], "native": [r.to_dict() for r in native],
         "eager_bytes_per_block": tot(eager, "bytes_moved"), "native_bytes_per_block": tot(native, "bytes_moved"),
         "eager_roofline_s_per_block": tot(eager, "roofline_seconds"),
         "native_roofline_s_per_block": tot(native, "roofline_seconds")}
    if rates:
        d["measured"] = rates
    return d


def _main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--measure-peaks", action="store_true", help="sweep here instead of MEASURED_PEAKS.json")
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    try:
        peak = measure_machine_peak(dev, torch.bfloat16 if dev == "cuda" else torch.float32) if a.measure_peaks \
            else peak_from_file()
    except FileNotFoundError:
        peak = measure_machine_peak(dev)
    rates = measure_op_rates(batch=a.batch, seq=a.seq, device=dev,
                             dtype=torch.bfloat16 if dev == "cuda" else torch.float32)
    payload = roofline_payload(peak, batch=a.batch, seq=a.seq, rates=rates)
    s = json.dumps(payload, indent=1)
    if a.out:
        Path(a.out).write_text(s)
    print(json.dumps({k: payload[k] for k in ("eager_bytes_per_block", "native_bytes_per_block",
                                               "eager_roofline_s_per_block", "native_roofline_s_per_block")}))
    for r in rates:
        print(json.dumps(r))


if __name__ == "__main__":
    _main()
