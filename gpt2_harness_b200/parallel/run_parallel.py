"""Strategy driver and closed-form checker.

Reference: scripts/run_parallel.py:55-755. Runs every strategy's equivalence
worker on ``world_size`` ranks (gloo on CPU, NCCL on GPUs), records the
numerical error against the single-process reference, and checks each
counted per-step payload against its closed form in the counter convention
(all-reduce = buffer, all-gather = output, reduce-scatter = input):

* DDP: all-reduce 4N;
* ZeRO-1: all-reduce 4N (+ all-gather of the padded params);
* ZeRO-2: reduce-scatter and all-gather 4 * N_pad each;
* ZeRO-3: sum_u 12 P_u + 4 N_root;
* TP (parity mode): 4 all-reduces of B*T*C*4 bytes per block; with sequence
  parallelism the raw payload doubles and the all-reduce equivalent matches;
* PP: B*T*C*4 sent per boundary (summed over micro-batches);
* CP: all-gather-KV 2*4*B*T*C; ring sends 2(p-1)/p of it forward, and in backward
  K/V again plus dK/dV for p hops (home).

Writes a JSON report and exits non-zero when any check or tolerance fails.

    python -m gpt2_harness_b200.parallel.run_parallel --world-size 2 --out results/parallel_comms.json
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path
from typing import Any

import torch

from .. import hardware
from .comms import spawn_workers
from .common import parallel_config

FP32 = 4
TOLERANCE = 1e-5  # the reference's strategy tolerance (fp32, CPU tier)


def _per_step(payload: dict, op: str, field: str = "payload_bytes") -> float:
    rec = payload.get("per_collective", {}).get(op)
    return 0.0 if rec is None else rec[field] / max(payload.get("steps", 1), 1)


def _check(name: str, measured: float, formula: str, predicted: float) -> dict[str, Any]:
    return {"name": name, "formula": formula, "measured": measured, "predicted": predicted,
            "ok": abs(measured - predicted) <= 1e-9 * max(1.0, abs(predicted))}


def run(world_size: int = 2, pipeline_stages: int = 4, steps: int = 4, batch: int = 8, seq: int = 16,
        backend: str | None = None, allow_oversubscribe: bool = False, progress: bool = True) -> dict[str, Any]:
    caps = hardware.Capabilities.detect()
    be = hardware.select_backend(caps, backend)
    p = world_size
    cfg = parallel_config()

    def spawn(fn, w, kw):
        return spawn_workers(fn, w, kw, backend=backend, caps=caps, allow_oversubscribe=allow_oversubscribe)

    say = print if progress else (lambda *a, **k: None)
    say(f"{be} | world {p} | pipeline stages {pipeline_stages} | torch {torch.__version__}")
    eq, comms, checks = {}, {}, []
    t0 = time.time()

    from .data_parallel import ddp_equivalence_worker
    say("[1/6] data parallel")
    r = spawn(ddp_equivalence_worker, p, {"batch": batch, "seq": seq, "steps": steps})
    n = r[0].value["n_params"] if "n_params" in r[0].value else sum(
        x.numel() for x in __import__("gpt2_harness_b200.models.gpt", fromlist=["GPT"]).GPT(cfg).parameters())
    eq["data_parallel"] = {"max_grad_error": max(x.value["max_grad_error"] for x in r),
                           "max_param_error": max(x.value["max_param_error"] for x in r)}
    comms["data_parallel"] = r[0].payload
    checks.append(_check("data_parallel.all_reduce", _per_step(r[0].payload, "all_reduce"), "4 * N", FP32 * n))

    from .zero import zero3_equivalence_worker, zero_equivalence_worker
    say("[2/6] ZeRO-1/2/3")
    for stage in (1, 2):
        r = spawn(zero_equivalence_worker, p, {"stage": stage, "steps": steps})
        v = r[0].value
        eq[f"zero_{stage}"] = {"max_param_error": max(x.value["max_param_error"] for x in r),
                               "sharded_bytes": v["sharded_bytes"], "replicated_bytes": v["replicated_bytes"]}
        comms[f"zero_{stage}"] = r[0].payload
        pad = v["padded_numel"]
        if stage == 1:
            checks.append(_check("zero_1.all_reduce", _per_step(r[0].payload, "all_reduce"), "4 * N", FP32 * n))
        else:
            checks.append(_check("zero_2.reduce_scatter", _per_step(r[0].payload, "reduce_scatter"), "4 * N_pad",
                                 FP32 * pad))
        checks.append(_check(f"zero_{stage}.all_gather", _per_step(r[0].payload, "all_gather"), "4 * N_pad",
                             FP32 * pad))
    r = spawn(zero3_equivalence_worker, p, {"steps": steps})
    v = r[0].value
    eq["zero_3"] = {"max_param_error": max(x.value["max_param_error"] for x in r)}
    comms["zero_3"] = r[0].payload
    cf = v["closed_form_payload_bytes"]
    total = sum(rec["payload_bytes"] for rec in r[0].payload["per_collective"].values()) / max(
        r[0].payload["steps"], 1)
    checks.append(_check("zero_3.total", total, "sum_u 12 P_u + 4 N_root",
                         cf["total"] if isinstance(cf, dict) else cf))

    from .tensor_parallel import tp_equivalence_worker
    say("[3/6] tensor parallel")
    for sp in (False, True):
        r = spawn(tp_equivalence_worker, p, {"batch": 4, "seq": 12, "sequence_parallel": sp})
        key = "tensor_parallel_sp" if sp else "tensor_parallel"
        eq[key] = {"max_forward_error": max(x.value["forward_error"] for x in r),
                   "max_backward_error": max(x.value["max_grad_error"] for x in r)}
        comms[key] = r[0].payload
        c = r[0].value["closed_form"]
        if sp:
            raw = _per_step(r[0].payload, "all_gather") + _per_step(r[0].payload, "reduce_scatter")
            checks.append(_check("tensor_parallel_sp.raw", raw, "8 * B*T*C*4 per block", c["raw"]))
        else:
            checks.append(_check("tensor_parallel.all_reduce", _per_step(r[0].payload, "all_reduce"),
                                 "4 * 4 * B * T * C per block", c["allreduce_equivalent"]))

    from .pipeline_parallel import pipeline_worker
    say("[4/6] pipeline parallel")
    for kind in ("gpipe", "1f1b"):
        r = spawn(pipeline_worker, pipeline_stages, {"kind": kind, "micro_batches": 4, "batch": batch, "seq": seq})
        eq[f"pipeline_{kind}"] = {"max_grad_error": max(x.value["max_grad_error"] for x in r)}
        comms[f"pipeline_{kind}"] = r[0].payload
        # rank 0 (first stage) sends the activations of every micro-batch once
        checks.append(_check(f"pipeline_{kind}.send", _per_step(r[0].payload, "send"),
                             "B * T * C * 4 (summed over micro-batches)", r[0].value["closed_form_send_bytes"]))

    from .sequence_parallel import sequence_parallel_worker
    say("[5/6] context parallel")
    for path in ("all_gather", "ring"):
        r = spawn(sequence_parallel_worker, p, {"path": path})
        eq[f"cp_{path}"] = {"forward_error": max(x.value["forward_error"] for x in r),
                            "input_grad_error": max(x.value["input_grad_error"] for x in r),
                            "weight_grad_error": max(x.value["weight_grad_error"] for x in r)}
        comms[f"cp_{path}"] = r[0].payload
        c = r[0].value["closed_form"]
        if path == "all_gather":
            checks.append(_check("cp.all_gather", _per_step(r[0].payload, "all_gather"), "2 * 4 * B * T * C",
                                 c["all_gather_kv_forward"]))
        else:
            checks.append(_check("cp_ring.send", _per_step(r[0].payload, "send"),
                                 "fwd 2(p-1)/p + bwd (2(p-1) + 2p)/p, times 4 * B * T * C", c["ring_send_total"]))

    from .dtensor_demo import dtensor_worker
    say("[6/6] DTensor")
    r = spawn(dtensor_worker, p, {})
    eq["dtensor"] = {"dtensor_error": max(x.value["dtensor_error"] for x in r),
                     "manual_vs_dtensor": max(x.value["manual_vs_dtensor"] for x in r)}

    errs = []
    for k, d in eq.items():
        for f, v in d.items():
            if f.endswith("error") and isinstance(v, (int, float)) and v > TOLERANCE:
                errs.append(f"{k}.{f}={v:.2e}")
    ok = all(c["ok"] for c in checks) and not errs
    for c in checks:
        say(f"  {'ok ' if c['ok'] else 'BAD'} {c['name']:<32} measured {c['measured']:>14,.0f}  "
            f"predicted {c['predicted']:>14,.0f}  ({c['formula']})")
    if errs:
        say("  tolerance failures: " + ", ".join(errs))
    return {"backend": be, "world_size": p, "pipeline_stages": pipeline_stages, "n_params": n,
            "tolerance": TOLERANCE, "equivalence": eq, "comms": comms, "checks": checks,
            "tolerance_failures": errs, "ok": ok, "seconds": time.time() - t0}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--world-size", type=int, default=2)
    ap.add_argument("--pipeline-stages", type=int, default=4)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=16)
    ap.add_argument("--backend", default=None, choices=[None, "gloo", "nccl"])
    ap.add_argument("--allow-oversubscribe", action="store_true")
    ap.add_argument("--out", default="results/parallel_comms.json")
    a = ap.parse_args(argv)
    res = run(a.world_size, a.pipeline_stages, a.steps, a.batch, a.seq, a.backend, a.allow_oversubscribe)
    out = Path(a.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(res, indent=1, default=str))
    print(f"{'all checks passed' if res['ok'] else 'CHECKS FAILED'} -> {out}")
    return 0 if res["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
