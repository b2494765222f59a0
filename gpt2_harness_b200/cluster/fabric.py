"""Interconnect cost model (MODELLED unless a link says measured).

Reference: src/transformer_internals/cluster/fabric.py:65-515. Ring-model
times for all-reduce (2(n-1)/n of the buffer, 2(n-1) latency hops),
all-gather / reduce-scatter ((n-1)/n, n-1 hops) and point-to-point, priced on
a ``Link`` (published per-direction bandwidth derated by a fixed efficiency,
or a measured link whose rate is already achieved); per-strategy
communication seconds per step for a 4-D ``ParallelConfig(tp, pp, cp, dp)``;
the TP degree at which TP communication overtakes compute.

B200 additions: NVLink 5 / NVSwitch (900 GB/s per direction per GPU) and the
pool's measured NVLink figures (770 GB/s peer copy per direction, 725 GB/s
8-rank all-reduce bus bandwidth at 1 GiB) as links; compute priced at the
measured sustained bf16 GEMM rate of a B200 rather than an H100 datasheet.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any, Optional

__all__ = ["Link", "LINKS", "LINK_EFFICIENCY", "GPUDIRECT_PENALTY", "PEAK_BF16_TFLOPS", "ASSUMED_MFU",
           "ModelShape", "ParallelConfig", "link_from_measurement", "predicted_vs_measured", "all_reduce_time",
           "all_gather_time", "p2p_time", "compute_time_s", "step_costs", "format_report", "crossover_ranks",
           "GPT2_124M", "GPT2_XL", "LLAMA70B"]


@dataclass(frozen=True)
class Link:
    name: str
    gbytes_per_s: float       # per direction per GPU, 1e9 B/s
    latency_us: float         # per hop, assumed unless measured
    source: str
    inter_node: bool
    measured: bool = False
    efficiency_applied: bool = False


LINKS: dict[str, Link] = {
    "nvlink5": Link("NVLink 5 / NVSwitch (B200 HGX)", 900.0, 1.5,
                    "B200: 18 NVLink 5 links, 900 GB/s per direction per GPU, full bandwidth to every "
                    "peer through NVSwitch", False),
    "nvlink5_measured_p2p": Link("NVLink 5 peer copy (B200, measured on this pool)", 770.0, 1.5,
                                 "peer copy 770 GB/s per direction, measured", False, measured=True,
                                 efficiency_applied=True),
    "nvlink5_measured_ar": Link("NVLink 5 8-rank all-reduce bus BW (B200, measured on this pool)", 725.0, 1.5,
                                "NCCL all-reduce bus bandwidth 725 GB/s at 1 GiB, 8 ranks, measured", False,
                                measured=True, efficiency_applied=True),
    "nvlink4": Link("NVLink 4 / NVSwitch (H100 SXM)", 450.0, 2.0, "18 links x 25 GB/s per direction", False),
    "nvlink3": Link("NVLink 3 (A100 SXM)", 300.0, 2.0, "12 links x 25 GB/s per direction", False),
    "pcie5": Link("PCIe Gen5 x16", 63.0, 5.0, "32 GT/s x16, 128b/130b", False),
    "ib_xdr": Link("InfiniBand XDR 800G (per GPU)", 100.0, 2.0, "ConnectX-8 800 Gb/s per GPU", True),
    "ib_ndr": Link("InfiniBand NDR 400G (per GPU)", 50.0, 2.0, "ConnectX-7 400 Gb/s per GPU", True),
    "ib_hdr": Link("InfiniBand HDR 200G (per GPU)", 25.0, 2.0, "200 Gb/s per GPU", True),
    "roce200": Link("RoCE v2 200 GbE", 25.0, 5.0, "200 GbE line rate; needs a lossless fabric", True),
}
LINK_EFFICIENCY = 0.85                 # achieved / published, applied to datasheet links only
GPUDIRECT_PENALTY = (1.6, 5.0)         # bandwidth divisor, added latency (us) without GPUDirect RDMA
PEAK_BF16_TFLOPS = 1415.2              # B200, measured sustained cuBLAS bf16 on this pool
ASSUMED_MFU = 0.45


@dataclass(frozen=True)
class ModelShape:
    n_layer: int
    n_embd: int
    n_head: int
    vocab_size: int
    seq_len: int
    micro_batch: int
    grad_accum: int = 1
    bytes_per_elem: int = 2

    @property
    def params(self) -> int:
        h = self.n_embd
        return 12 * self.n_layer * h * h + 2 * self.vocab_size * h

    @property
    def tokens_per_microbatch(self) -> int:
        return self.micro_batch * self.seq_len


@dataclass(frozen=True)
class ParallelConfig:
    tp: int = 1
    pp: int = 1
    cp: int = 1
    dp: int = 1

    @property
    def world_size(self) -> int:
        return self.tp * self.pp * self.cp * self.dp


def _hops(op: str, n: int) -> int:
    return 0 if n < 2 else 2 * (n - 1) if op == "all_reduce" else n - 1


def link_from_measurement(name: str, fit: dict, ranks: int, op: str = "all_reduce",
                          peak_bus_gbytes_per_s: Optional[float] = None, inter_node: bool = False,
                          detail: str = "") -> Link:
    """A measured link from a collbench fit: fitted bus bandwidth (already
    achieved, so no efficiency derating) and the fitted intercept divided by
    the ring's hop count (this model's latency is per hop)."""
    hops = max(_hops(op, ranks), 1)
    peak = f", peak bus {peak_bus_gbytes_per_s:.1f} GB/s" if peak_bus_gbytes_per_s else ""
    return Link(name, float(fit["bandwidth_gbytes_per_s"]), max(float(fit["latency_us"]), 0.0) / hops,
                f"MEASURED {op} at {ranks} ranks: t = {fit['latency_us']:.1f} us + bytes / "
                f"{fit['bandwidth_gbytes_per_s']:.1f} GB/s (R^2 {fit['r_squared']:.4f}){peak}; latency / {hops} "
                f"hops. {detail}".strip(), inter_node, measured=True, efficiency_applied=True)


def _bw(link: Link, gpudirect: bool) -> float:
    bw = link.gbytes_per_s * (1.0 if link.efficiency_applied else LINK_EFFICIENCY) * 1e9
    return bw / GPUDIRECT_PENALTY[0] if link.inter_node and not gpudirect else bw


def _lat(link: Link, gpudirect: bool) -> float:
    return (link.latency_us + (GPUDIRECT_PENALTY[1] if link.inter_node and not gpudirect else 0.0)) * 1e-6


def all_reduce_time(nbytes: float, ranks: int, link: Link, *, gpudirect: bool = True) -> float:
    if ranks < 2:
        return 0.0
    return 2 * (ranks - 1) / ranks * nbytes / _bw(link, gpudirect) + 2 * (ranks - 1) * _lat(link, gpudirect)


def all_gather_time(nbytes: float, ranks: int, link: Link, *, gpudirect: bool = True) -> float:
    if ranks < 2:
        return 0.0
    return (ranks - 1) / ranks * nbytes / _bw(link, gpudirect) + (ranks - 1) * _lat(link, gpudirect)


def p2p_time(nbytes: float, link: Link, *, gpudirect: bool = True) -> float:
    return nbytes / _bw(link, gpudirect) + _lat(link, gpudirect)


def predicted_vs_measured(points: list, ranks: int, link: Link, op: str = "all_reduce") -> list[dict]:
    f = all_reduce_time if op == "all_reduce" else all_gather_time
    out = []
    for p in points:
        m, meas = f(float(p["bytes"]), ranks, link), float(p["median_s"])
        out.append({"op": op, "bytes": p["bytes"], "measured_s": meas, "modelled_s": m,
                    "modelled_over_measured": m / meas if meas else float("nan")})
    return out


def compute_time_s(shape: ModelShape, cfg: ParallelConfig, *, mfu: float = ASSUMED_MFU,
                   peak_tflops: float = PEAK_BF16_TFLOPS) -> float:
    """6 P T weight FLOPs + 12 L h T s attention FLOPs over the job's GPUs."""
    tokens = shape.tokens_per_microbatch * shape.grad_accum * cfg.dp
    flops = 6 * shape.params * tokens + 12 * shape.n_layer * shape.n_embd * tokens * shape.seq_len
    return flops / (cfg.world_size * peak_tflops * 1e12 * mfu)


def step_costs(shape: ModelShape, cfg: ParallelConfig, link_key: str, *, gpudirect: bool = True) -> dict:
    """Seconds of communication per optimiser step for each axis, each as if
    it ran over ``link_key``: tp = 4 all-reduces of [tokens, h] per layer per
    micro-batch; fsdp = 3 passes over the local parameter bytes; ddp = one
    all-reduce of them; pp = activations across each boundary both ways per
    micro-batch; cp = K and V around the ring per layer, both ways."""
    link = LINKS[link_key] if isinstance(link_key, str) else link_key
    h, b = shape.n_embd, shape.bytes_per_elem
    act = shape.tokens_per_microbatch * h * b
    params = shape.params / max(cfg.tp * cfg.pp, 1) * b
    out = {"tp": 4 * shape.n_layer * shape.grad_accum * all_reduce_time(act, cfg.tp, link, gpudirect=gpudirect)
           if cfg.tp > 1 else 0.0,
           "fsdp": 3 * all_gather_time(params, cfg.dp, link, gpudirect=gpudirect) if cfg.dp > 1 else 0.0,
           "ddp": all_reduce_time(params, cfg.dp, link, gpudirect=gpudirect) if cfg.dp > 1 else 0.0,
           "pp": 2 * (cfg.pp - 1) * shape.grad_accum * p2p_time(act / max(cfg.tp, 1), link, gpudirect=gpudirect)
           if cfg.pp > 1 else 0.0,
           "cp": 2 * shape.n_layer * shape.grad_accum * (cfg.cp - 1)
           * p2p_time(2 * act / (max(cfg.cp, 1) * max(cfg.tp, 1)), link, gpudirect=gpudirect)
           if cfg.cp > 1 else 0.0}
    return out


GPT2_124M = ModelShape(12, 768, 12, 50257, 1024, 16)
GPT2_XL = ModelShape(48, 1600, 25, 50304, 1024, 4)
LLAMA70B = ModelShape(80, 8192, 64, 128256, 8192, 1, 8)


def crossover_ranks(shape: ModelShape, link_key: str, *, max_tp: int = 64, world: int = 64) -> Optional[int]:
    """Smallest TP degree whose TP communication exceeds compute on the link."""
    for tp in (2, 4, 8, 16, 32, 64):
        if tp > max_tp:
            break
        cfg = ParallelConfig(tp=tp, dp=max(1, world // tp))
        if step_costs(shape, cfg, link_key)["tp"] > compute_time_s(shape, cfg):
            return tp
    return None


def format_report(shape: ModelShape = GPT2_XL, label: str = "GPT-2 XL, 1k context",
                  cfg: ParallelConfig = ParallelConfig(tp=8), keys=("nvlink5", "nvlink5_measured_ar", "nvlink4",
                                                                    "ib_xdr", "ib_ndr", "roce200")) -> str:
    lines = ["MODELLED unless a link is marked measured. Datasheet links are derated by "
             f"{LINK_EFFICIENCY}; MFU {ASSUMED_MFU} at {PEAK_BF16_TFLOPS} TFLOP/s per GPU.", "",
             f"Model: {label}: {shape.params / 1e9:.2f}B params, layers {shape.n_layer}, d {shape.n_embd}, "
             f"micro-batch {shape.micro_batch} x {shape.seq_len}, accum {shape.grad_accum}",
             f"Layout: tp={cfg.tp} pp={cfg.pp} cp={cfg.cp} dp={cfg.dp}  compute "
             f"{compute_time_s(shape, cfg) * 1e3:.1f} ms/step", "",
             f"{'link':<58}{'tp ms':>9}{'ddp ms':>9}{'fsdp ms':>9}{'pp ms':>9}{'cp ms':>9}"]
    for k in keys:
        c = step_costs(shape, cfg, k)
        tag = " [measured]" if LINKS[k].measured else ""
        lines.append(f"{(LINKS[k].name + tag)[:57]:<58}" + "".join(f"{c[a] * 1e3:9.2f}"
                                                                  for a in ("tp", "ddp", "fsdp", "pp", "cp")))
    return "\n".join(lines)


if __name__ == "__main__":
    print(format_report())
    print()
    for k in ("nvlink5", "nvlink4", "ib_xdr", "ib_ndr", "roce200"):
        n = crossover_ranks(LLAMA70B, k)
        print(f"70B-class: TP becomes communication-bound on {k} at tp={n}" if n
              else f"70B-class: TP stays compute-bound on {k} up to tp=64")
