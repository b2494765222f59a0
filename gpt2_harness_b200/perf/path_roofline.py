"""Per-strategy roofline of a training step: the slower of its compute at the
measured bf16 peak and the bytes that must cross each GPU's NVLink ports at
the measured peer-copy bandwidth, against the measured step time.

    t_roof = max(FLOPs_per_rank / peak, NVLink_bytes_per_direction / link_bw)
    fraction = t_roof / t_measured

Compute: the causal model FLOPs (the attention quadratic term halved: the
kernels skip the masked half) of the step's tokens, divided evenly over the
ranks. Communication: the bytes each rank's busiest direction must carry for
the native implementation of the strategy (fp32 gradients, bf16 parameters
and activations where those are what the kernels move), per optimiser step:

* DDP: all-reduce of the fp32 gradient G = 4N: 2(p-1)/p x G each way
  (reduce-scatter by peer loads, all-gather by peer stores).
* ZeRO-2: reduce-scatter of G plus all-gather of the bf16 parameters:
  (p-1)/p x (4N + 2N).
* ZeRO-3: two bf16 gathers of every block's parameters (forward and
  backward) and an fp32 reduce-scatter of their gradients, plus the fp32
  all-reduce of the replicated root (wte, wpe, ln_f): (p-1)/p x 8 N_blocks +
  2(p-1)/p x 4 N_root.
* TP + SP: 8 collectives of the [B*T, C] bf16 activations per block (AG and
  RS around c_attn/c_proj and c_fc/mlp-proj, forward and backward):
  8 L (p-1)/p x 2BTC.
* CP (all-gather-KV, zig-zag or contiguous): per layer the busiest rank moves
  2p-2 chunks of B x T/2p x 2C bf16 in the K/V gather and as many in the dK/dV
  reduce, plus the DDP all-reduce of the weight gradients.
* PP (x CP): each stage boundary carries m fp32 activations forward and m
  gradients back ([B, T/cp, C] each); a middle stage sends both ways, so its
  busiest direction carries 2m of them (m at the two end stages). The CP
  traffic of the stage's L/pp layers and its gradient all-reduce add on top.

Link bandwidth: the 770 GB/s per direction peer copy measured on this pool
(NVLink 5 nominal: 900 GB/s); the peak: MEASURED_PEAKS.json's sustained bf16
figure. ``python -m gpt2_harness_b200.perf.path_roofline`` prints the table
for the step times measured with bench.py.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass
from typing import Optional

from gpt2_harness_b200.config import GPTConfig, gpt2_config
from gpt2_harness_b200.perf.mfu import flops_per_token_exact, measured_peak_tflops, param_count

__all__ = ["LINK_GBS", "PathRoofline", "nvlink_bytes", "path_roofline", "MEASURED_RUNS"]

#: Peer copy bandwidth per direction per GPU measured on this pool (GB/s).
LINK_GBS = 770.0


def _block_params(cfg: GPTConfig) -> int:
    c = cfg.n_embd
    return 12 * c * c + 13 * c


def nvlink_bytes(strategy: str, cfg: GPTConfig, batch: int, seq: int, world: int, *,
                 pp: int = 1, cp: int = 1, micro_batches: int = 1) -> float:
    """Bytes per optimiser step on the busiest NVLink direction of the busiest
    rank (see the module docstring for each strategy's model)."""
    p = world
    if p <= 1 and strategy != "pp":
        return 0.0
    n = float(param_count(cfg))
    L, C = cfg.n_layer, cfg.n_embd
    if strategy == "ddp":
        return 2 * (p - 1) / p * 4 * n
    if strategy == "zero2":
        return (p - 1) / p * 6 * n
    if strategy == "zero3":
        n_blk = L * _block_params(cfg)
        n_root = n - n_blk
        return (p - 1) / p * 8 * n_blk + 2 * (p - 1) / p * 4 * n_root
    if strategy == "tp":
        return 8 * L * (p - 1) / p * 2.0 * batch * seq * C
    if strategy == "cp":
        return _cp_bytes(cfg, L, batch, seq, p) + 2 * (p - 1) / p * 4 * n
    if strategy == "pp":
        if pp * cp != world:
            raise ValueError("pp x cp must equal the world size")
        act = float(batch) * (seq // cp) * C * 4
        boundary = (2 if pp > 2 else 1) * micro_batches * act if pp > 1 else 0.0
        stage_params = n / pp
        cp_part = 0.0
        if cp > 1:
            cp_part = micro_batches * _cp_bytes(cfg, L // pp, batch, seq, cp)
            cp_part += 2 * (cp - 1) / cp * 4 * stage_params
        return boundary + cp_part
    raise ValueError(f"unknown strategy {strategy!r}")


def _cp_bytes(cfg: GPTConfig, layers: int, batch: int, seq: int, p: int) -> float:
    chunk = float(batch) * (seq / (2 * p)) * 2 * cfg.n_embd * 2
    return layers * 2 * (2 * p - 2) * chunk


@dataclass
class PathRoofline:
    strategy: str
    world: int
    tokens_per_step: int
    flops_per_rank: float
    nvlink_bytes: float
    t_compute_ms: float
    t_comm_ms: float
    t_roof_ms: float
    t_measured_ms: float
    fraction: float
    bound: str

    def to_dict(self) -> dict:
        return asdict(self)


def path_roofline(strategy: str, cfg: GPTConfig, batch: int, seq: int, world: int,
                  measured_ms: float, *, pp: int = 1, cp: int = 1, micro_batches: int = 1,
                  peak_tflops: Optional[float] = None, link_gbs: float = LINK_GBS) -> PathRoofline:
    """Roofline of one measured step. ``batch`` is per rank for ddp/zero*,
    global for tp/cp, and the micro-batch for pp (``micro_batches`` of them)."""
    if strategy in ("ddp", "zero2", "zero3"):
        tokens = batch * seq * world
    elif strategy in ("tp", "cp"):
        tokens = batch * seq
    elif strategy == "pp":
        tokens = micro_batches * batch * seq
    else:
        raise ValueError(f"unknown strategy {strategy!r}")
    if peak_tflops is None:
        peak_tflops, _ = measured_peak_tflops(sustained=True)
    fpt = flops_per_token_exact(cfg, seq, causal_aware=True)["training_flops_per_token"]
    flops = fpt * tokens / world
    nb = nvlink_bytes(strategy, cfg, batch, seq, world, pp=pp, cp=cp, micro_batches=micro_batches)
    t_c = flops / (peak_tflops * 1e12) * 1e3
    t_n = nb / (link_gbs * 1e9) * 1e3
    roof = max(t_c, t_n)
    return PathRoofline(strategy, world, tokens, flops, nb, round(t_c, 3), round(t_n, 3), round(roof, 3),
                        measured_ms, round(roof / measured_ms, 3), "compute" if t_c >= t_n else "NVLink")


#: Step times measured with bench.py on B200 (CUDA events, max over ranks):
#: (label, strategy, model, batch, seq, world, ms, extra kwargs).
MEASURED_RUNS = [
    ("DDP N=1, 124M 16x1024", "ddp", "gpt2", 16, 1024, 1, 20.27, {}),
    ("DDP N=2, 124M 16x1024/GPU", "ddp", "gpt2", 16, 1024, 2, 21.96, {}),
    ("DDP N=8, 124M 16x1024/GPU", "ddp", "gpt2", 16, 1024, 8, 22.22, {}),
    ("ZeRO-2 N=2, 124M 16x1024/GPU", "zero2", "gpt2", 16, 1024, 2, 21.51, {}),
    ("ZeRO-3 N=2, 350M 8x1024/GPU", "zero3", "gpt2-medium", 8, 1024, 2, 33.92, {}),
    ("TP=2+SP, XL global 32x1024", "tp", "gpt2-xl", 32, 1024, 2, 270.29, {}),
    ("TP=8+SP, XL global 32x1024", "tp", "gpt2-xl", 32, 1024, 8, 195.60, {}),
    ("CP=2 zig-zag, large 1x16384", "cp", "gpt2-large", 1, 16384, 2, 169.84, {}),
    ("PP=2 1F1B, large 8x(1x16384)", "pp", "gpt2-large", 1, 16384, 2, 1253.83,
     {"pp": 2, "cp": 1, "micro_batches": 8}),
    ("PP=2xCP=2 1F1B, large 8x(1x16384)", "pp", "gpt2-large", 1, 16384, 4, 904.00,
     {"pp": 2, "cp": 2, "micro_batches": 8}),
]


def table(runs=None) -> list[dict]:
    out = []
    for label, strat, model, b, t, w, ms, kw in (runs or MEASURED_RUNS):
        cfg = gpt2_config(model, n_positions=max(t, gpt2_config(model).n_positions))
        r = path_roofline(strat, cfg, b, t, w, ms, **kw).to_dict()
        r["label"] = label
        out.append(r)
    return out


def _main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()
    rows = table()
    if args.json:
        print(json.dumps(rows, indent=1))
        return
    print("| run | compute ms | NVLink ms | roofline ms | measured ms | fraction | bound |")
    print("|---|---|---|---|---|---|---|")
    for r in rows:
        print(f"| {r['label']} | {r['t_compute_ms']:.2f} | {r['t_comm_ms']:.2f} | {r['t_roof_ms']:.2f} | "
              f"{r['t_measured_ms']:.2f} | {r['fraction']:.2f} | {r['bound']} |")


if __name__ == "__main__":
    _main()
