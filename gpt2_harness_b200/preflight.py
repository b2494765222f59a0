"""Machine preflight: resolve every placement / backend / precision decision
before a run, live or against a fabricated node.

Reference: scripts/gpu_preflight.py:52-243. Live mode reads the machine (GPU
count, names, compute capability, driver, NCCL, NVLink topology); dry-run
mode (``--dry-run --stub-gpus 8``) builds a fake B200 node and takes every
decision the real run will take, so the CUDA branches are exercised on a
laptop. Both also evaluate the arithmetic parts at GPU shapes (activation
bytes of the BASELINE configs, fabric cost of TP=8 over NVLink 5) so a wrong
shape shows up before a box is rented. Exit 0 when everything requested is
possible, 1 otherwise, with the problems listed once.

    python -m gpt2_harness_b200.preflight --dry-run --stub-gpus 8 --world-sizes 1 2 4 8
"""

from __future__ import annotations

import argparse
import json
import sys
from typing import Any, Optional

from . import hardware
from .hardware import Capabilities, HardwareError

__all__ = ["resolve", "arithmetic_checks", "run", "main"]


def resolve(caps: Capabilities, world_sizes: list[int], backend: Optional[str]) -> dict[str, Any]:
    rep: dict[str, Any] = {"backend": None, "placements": {}, "precision": {}, "native_kernels": None,
                           "problems": []}
    try:
        be = hardware.select_backend(caps, backend)
        rep["backend"] = be
    except HardwareError as e:
        rep["problems"].append(str(e))
        return rep
    for w in world_sizes:
        try:
            rep["placements"][str(w)] = hardware.check_placement(caps, w, be)
        except HardwareError as e:
            rep["problems"].append(f"world size {w}: {e}")
    from .precision import resolve_amp
    dev = "cuda" if be == "nccl" else "cpu"
    for dt in ("bf16", "fp16"):
        try:
            rep["precision"][dt] = resolve_amp(True, dt, dev, caps=caps).to_dict()
        except (HardwareError, ValueError) as e:
            rep["precision"][dt] = {"refused": str(e)}
    rep["native_kernels"] = hardware.native_kernels_supported(caps)
    if caps.cuda_available and not rep["native_kernels"]:
        rep["problems"].append("the sm_100a native kernels need a Blackwell (B200-class) GPU; "
                               f"found {caps.accelerator}")
    return rep


def arithmetic_checks() -> dict[str, Any]:
    """Analytic numbers at BASELINE shapes (no device needed)."""
    from .cluster.fabric import GPT2_XL, LINKS, ParallelConfig, compute_time_s, step_costs
    from .config import gpt2_config
    from .perf.mfu import flops_per_token_exact, param_count
    out: dict[str, Any] = {}
    for size, (b, t) in {"gpt2": (16, 1024), "gpt2-medium": (8, 1024), "gpt2-xl": (4, 1024)}.items():
        cfg = gpt2_config(size)
        out[size] = {"params": param_count(cfg), "train_flops_per_token": flops_per_token_exact(cfg, t)[
            "training_flops_per_token"], "batch": b, "seq": t}
    tp8 = ParallelConfig(tp=8)
    out["gpt2-xl_tp8_nvlink5"] = {"comm_s": step_costs(GPT2_XL, tp8, "nvlink5"),
                                  "compute_s": compute_time_s(GPT2_XL, tp8), "link": LINKS["nvlink5"].name}
    try:
        from .perf.activation_memory import analytic_activation_bytes
        cfg = gpt2_config("gpt2")
        out["gpt2_activation_bytes_fp32_b16_t1024"] = analytic_activation_bytes(cfg, 16, 1024, 4)["total"]
    except Exception as e:  # the analytic count refuses configurations it does not enumerate
        out["gpt2_activation_bytes_fp32_b16_t1024"] = f"not enumerated: {e}"
    return out


def run(dry_run: bool = False, stub_gpus: int = 8, world_sizes=(1, 2, 4, 8), backend: Optional[str] = None,
        topology: bool = True) -> dict[str, Any]:
    caps = Capabilities.stub(stub_gpus) if dry_run else Capabilities.detect()
    rep = {"mode": "dry-run (fabricated node)" if dry_run else "live", "machine": caps.to_dict(),
           "decisions": resolve(caps, list(world_sizes), backend), "arithmetic": arithmetic_checks()}
    if not dry_run and topology:
        rep["nvlink_topology"] = hardware.nvidia_smi("topo", "-m")
    rep["ok"] = not rep["decisions"]["problems"]
    return rep


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--stub-gpus", type=int, default=8)
    ap.add_argument("--world-sizes", type=int, nargs="+", default=[1, 2, 4, 8])
    ap.add_argument("--backend", default="auto")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rep = run(a.dry_run, a.stub_gpus, a.world_sizes, None if a.backend == "auto" else a.backend)
    print(hardware.describe(Capabilities.stub(a.stub_gpus) if a.dry_run else Capabilities.detect()))
    d = rep["decisions"]
    print(f"backend {d['backend']}  native kernels {'yes' if d['native_kernels'] else 'no'}  "
          f"placements {', '.join(d['placements'])}")
    for p in d["problems"]:
        print(f"  PROBLEM: {p}")
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rep, f, indent=1, default=str)
    print("preflight OK" if rep["ok"] else "preflight FAILED")
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
