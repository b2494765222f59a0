"""Collective benchmark: all-reduce / all-gather / reduce-scatter swept over
message sizes and world sizes, with bus bandwidth and a latency/bandwidth fit.

Reference: src/transformer_internals/cluster/collbench.py:88-401. Bus
bandwidth uses NCCL's convention (``S/t`` times 2(n-1)/n for all-reduce,
(n-1)/n for all-gather and reduce-scatter) so numbers compare with link
rates; ``t = a + b * bytes`` is fitted by least squares (latency from the
intercept, bus bandwidth from the slope).

On GPUs every size is timed with CUDA events on the issuing stream (median
and min of repeats, max over ranks), and the sweep also times this
framework's fused peer-memory all-reduce kernel (``impl="p2p"``) next to
NCCL. The world sizes run as spawned ranks (gloo on CPU, NCCL on GPUs).

    python -m gpt2_harness_b200.cluster.collbench --world 2 --backend nccl
"""

from __future__ import annotations

import argparse
import json
import statistics
import time
from typing import Any, Optional

import torch
import torch.distributed as dist

__all__ = ["OPS", "DEFAULT_SIZES", "bus_factor", "bus_bandwidth", "fit_link_model", "run"]

OPS = ("all_reduce", "all_gather", "reduce_scatter")
DEFAULT_SIZES = [1 << k for k in range(10, 29, 2)]  # 1 KiB .. 256 MiB


def bus_factor(op: str, world: int) -> float:
    if world < 2:
        return 0.0
    if op == "all_reduce":
        return 2.0 * (world - 1) / world
    if op in ("all_gather", "reduce_scatter"):
        return (world - 1) / world
    raise ValueError(f"unknown collective {op!r}; expected one of {OPS}")


def bus_bandwidth(op: str, nbytes: float, seconds: float, world: int) -> float:
    """Bytes/s on the bus for one call moving an ``nbytes`` (unsharded) buffer."""
    return 0.0 if seconds <= 0 or world < 2 else nbytes / seconds * bus_factor(op, world)


def fit_link_model(nbytes: list, seconds: list, ranks: int, op: str = "all_reduce") -> dict:
    """Least squares ``t = a + b x``; bus bandwidth = factor / b."""
    n = len(nbytes)
    mx, my = sum(nbytes) / n, sum(seconds) / n
    sxx = sum((x - mx) ** 2 for x in nbytes)
    slope = sum((x - mx) * (y - my) for x, y in zip(nbytes, seconds)) / sxx if sxx > 0 else 0.0
    icpt = my - slope * mx
    ss_tot = sum((y - my) ** 2 for y in seconds)
    ss_res = sum((y - icpt - slope * x) ** 2 for x, y in zip(nbytes, seconds))
    return {"op": op, "latency_us": icpt * 1e6,
            "bandwidth_gbytes_per_s": bus_factor(op, ranks) / slope / 1e9 if slope > 0 else float("nan"),
            "r_squared": 1 - ss_res / ss_tot if ss_tot > 0 else float("nan"), "slope_s_per_byte": slope,
            "intercept_s": icpt}


def _timer(dev: torch.device):
    if dev.type == "cuda":
        def t(fn):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            return a.elapsed_time(b) / 1e3
    else:
        def t(fn):
            t0 = time.perf_counter()
            fn()
            return time.perf_counter() - t0
    return t


def _worker(rank: int, world: int, sizes: list, ops: list, repeats: int, warmup: int, p2p: bool) -> dict:
    backend = dist.get_backend()
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    timer = _timer(dev)
    rows = []
    symm = None
    if p2p and dev.type == "cuda":
        from ..parallel.symm import P2PAllReducer
        symm = P2PAllReducer(max(sizes) + 4096, None, dev)
    for op in ops:
        for nbytes in sizes:
            n = max(world, nbytes // 4 // world * world)
            buf = torch.ones(n, device=dev)
            shard = torch.empty(n // world, device=dev)
            if op == "all_reduce":
                fn = lambda: dist.all_reduce(buf)  # noqa: E731
            elif op == "all_gather":
                fn = lambda: dist.all_gather_into_tensor(buf, shard)  # noqa: E731
            else:
                fn = lambda: dist.reduce_scatter_tensor(shard, buf)  # noqa: E731
            impls = [("backend", fn)]
            if symm is not None and op == "all_reduce":
                impls.append(("p2p", lambda n=n: symm.all_reduce(n)))
            for impl, f in impls:
                for _ in range(warmup):
                    f()
                ts = []
                for _ in range(repeats):
                    dist.barrier()
                    ts.append(timer(f))
                # max over ranks of the median (the collective is done when the slowest rank is)
                med = torch.tensor([statistics.median(ts), min(ts)], dtype=torch.float64)
                if backend == "nccl":
                    med = med.to(dev)
                dist.all_reduce(med, op=dist.ReduceOp.MAX)
                med = med.cpu()
                rows.append({"op": op, "impl": backend if impl == "backend" else "p2p", "bytes": n * 4,
                             "median_s": float(med[0]), "min_s": float(med[1]),
                             "bus_gbytes_per_s": bus_bandwidth(op, n * 4, float(med[0]), world) / 1e9})
    if symm is not None:
        symm.close()
    return {"rows": rows, "device": str(dev)}


def run(world_sizes=(2,), sizes: Optional[list] = None, ops=OPS, repeats: int = 5, warmup: int = 2,
        backend: Optional[str] = None, p2p: bool = True, timeout_s: float = 600.0) -> dict[str, Any]:
    """Sweep every (world size, op, size); fit each (world, op, impl)."""
    from ..parallel.comms import spawn_workers
    sizes = list(sizes or DEFAULT_SIZES)
    out: dict[str, Any] = {"sizes": sizes, "ops": list(ops), "results": [], "fits": []}
    for w in world_sizes:
        res = spawn_workers(_worker, w, dict(sizes=sizes, ops=list(ops), repeats=repeats, warmup=warmup, p2p=p2p),
                            backend=backend, timeout=timeout_s)
        rows = res[0].value["rows"]
        for r in rows:
            r["world_size"] = w
        out["results"] += rows
        out["backend"] = res[0].backend
        for op in ops:
            for impl in sorted({r["impl"] for r in rows if r["op"] == op}):
                pts = [r for r in rows if r["op"] == op and r["impl"] == impl]
                fit = fit_link_model([p["bytes"] for p in pts], [p["median_s"] for p in pts], w, op)
                fit.update(world_size=w, impl=impl,
                           peak_bus_gbytes_per_s=max(p["bus_gbytes_per_s"] for p in pts))
                out["fits"].append(fit)
    return out


def _main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--world", type=int, nargs="+", default=[2])
    ap.add_argument("--backend", default=None)
    ap.add_argument("--max-mib", type=int, default=64)
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    sizes = [s for s in DEFAULT_SIZES if s <= a.max_mib << 20]
    res = run(a.world, sizes, backend=a.backend, repeats=a.repeats)
    for f in res["fits"]:
        print(json.dumps(f))
    if a.json:
        with open(a.json, "w") as fh:
            json.dump(res, fh, indent=1)


if __name__ == "__main__":
    _main()
