"""Cluster-operations runner: resharding, async save, prefetch, kill-and-resume,
collectives and the fabric model, into one results JSON.

Reference: scripts/run_cluster.py:74-437. Each measurement is a function so
it can be run alone:

* ``measure_resharding``: a GPT-2 TP-plan checkpoint saved at W ranks and
  reloaded at W' (up, down, to 1), every tensor bitwise identical to the
  original, with the number of shard files each rank had to open;
* ``measure_async_save``: training-loop stall of the background checkpointer
  (host snapshot only) against a synchronous save of the same state;
* ``measure_prefetch``: a slow source consumed with and without prefetch;
* ``measure_failure_restart``: a 2-rank job SIGKILLed mid-run and relaunched
  from its last checkpoint, losses compared bit for bit with an undisturbed
  run;
* ``measure_collectives``: the collective sweep (gloo on CPU, NCCL and the
  fused peer kernel on GPUs) with fitted latency / bandwidth;
* ``model_the_fabric``: the fabric cost report at BASELINE shapes.

    python -m gpt2_harness_b200.cluster.run_cluster --out results/cluster.json
"""

from __future__ import annotations

import argparse
import json
import tempfile
import time
from pathlib import Path
from typing import Any

import torch

__all__ = ["measure_resharding", "measure_async_save", "measure_prefetch", "measure_failure_restart",
           "measure_collectives", "model_the_fabric", "main"]


def measure_resharding(tmp: Path) -> dict[str, Any]:
    from ..config import GPTConfig
    from ..models.gpt import GPT
    from .checkpoint import gpt2_tp_plan, load_reshard, save_sharded, shard_state_dict
    torch.manual_seed(0)
    cfg = GPTConfig(vocab_size=512, n_positions=64, n_layer=2, n_head=4, n_embd=64)
    full = {k: v.clone() for k, v in GPT(cfg).state_dict().items() if not k.endswith("causal_mask")}
    full.pop("lm_head.weight", None)
    plan = gpt2_tp_plan(full, vocab_parallel=True)
    shapes = {k: list(v.shape) for k, v in full.items()}
    out = {}
    for src, dsts in ((2, (4, 1)), (4, (2, 1))):
        d = tmp / f"ckpt_w{src}"
        for r in range(src):
            save_sharded(d, shard_state_dict(full, plan, r, src), plan, rank=r, world_size=src, step=7,
                         global_shapes=shapes)
        for dst in dsts:
            pieces, files = [], []
            for r in range(dst):
                local, idx, nread = load_reshard(d, rank=r, world_size=dst, plan=plan if dst > 1 else {})
                pieces.append(local)
                files.append(nread)
            ok = True
            for k, v in full.items():
                from .checkpoint import merge_pieces
                spec = plan[k] if dst > 1 else None
                got = pieces[0][k] if spec is None or spec.replicated else merge_pieces([p[k] for p in pieces], spec)
                ok &= torch.equal(got[: v.shape[0]] if got.shape != v.shape else got, v)
            out[f"{src}->{dst}"] = {"bitwise_identical": bool(ok), "files_read_per_rank": files}
    return {"reshards": out}


def measure_async_save(tmp: Path, repeats: int = 3) -> dict[str, Any]:
    from .checkpoint import AsyncCheckpointer, save_sharded
    state = {f"w{i}": torch.randn(1024, 1024) for i in range(16)}  # 64 MiB
    shapes = {k: list(v.shape) for k, v in state.items()}
    sync_s, stall_s = [], []
    for i in range(repeats):
        t0 = time.perf_counter()
        save_sharded(tmp / f"sync{i}", state, {}, rank=0, world_size=1, global_shapes=shapes)
        sync_s.append(time.perf_counter() - t0)
        ck = AsyncCheckpointer()
        t0 = time.perf_counter()
        ck.save(tmp / f"async{i}", state, plan={}, rank=0, world_size=1, global_shapes=shapes)
        stall_s.append(time.perf_counter() - t0)
        ck.wait()
    return {"bytes": sum(v.numel() * 4 for v in state.values()), "sync_save_s": min(sync_s),
            "async_stall_s": min(stall_s), "stall_fraction_of_sync": min(stall_s) / min(sync_s)}


def measure_prefetch(repeats: int = 2) -> dict[str, Any]:
    from .streaming import DelayedSource, measure_throughput
    src = DelayedSource(list(range(64)), 0.004)
    off = max(measure_throughput(src, 40, prefetch=0, work_s=0.004) for _ in range(repeats))
    on = max(measure_throughput(src, 40, prefetch=8, work_s=0.004) for _ in range(repeats))
    return {"samples_per_s_no_prefetch": off, "samples_per_s_prefetch8": on, "speedup": on / off}


def measure_failure_restart(tmp: Path) -> dict[str, Any]:
    from .failure import JobSpec, make_corpus, read_log, run_with_recovery

    def spec(sub):
        data = make_corpus(tmp / sub / "corpus.bin", n_tokens=30_000, vocab=128, seed=0)
        return JobSpec(data_path=str(data), ckpt_dir=str(tmp / sub / "ckpt"), log_path=str(tmp / sub / "log.jsonl"),
                       steps=14, ckpt_every=5, micro_batch=4, block_size=32)

    def losses(p):
        return {r["step"]: r["loss"] for r in read_log(p) if r.get("event") == "step"}

    a, b = spec("clean"), spec("crash")
    run_with_recovery(2, a)
    rep = run_with_recovery(2, b, kill_rank_at_step=(1, 12))
    la, lb = losses(a.log_path), losses(b.log_path)
    common = sorted(set(la) & set(lb))
    return {"launches": rep.launches, "resumed_from_step": rep.resumed_from_step,
            "time_to_recover_s": rep.time_to_recover_s,
            "max_abs_loss_difference": max(abs(la[s] - lb[s]) for s in common), "steps_compared": len(common)}


def measure_collectives(world_size: int = 2) -> dict[str, Any]:
    from .collbench import run
    return run((world_size,), sizes=[1 << k for k in range(12, 23, 2)], repeats=3, warmup=1)


def model_the_fabric() -> dict[str, Any]:
    from .fabric import GPT2_XL, LINKS, LLAMA70B, ParallelConfig, crossover_ranks, format_report, step_costs
    return {"report": format_report(), "tp8_gpt2_xl": {k: step_costs(GPT2_XL, ParallelConfig(tp=8), k)
                                                       for k in ("nvlink5", "nvlink5_measured_ar", "ib_ndr")},
            "tp_crossover_70b": {k: crossover_ranks(LLAMA70B, k) for k in ("nvlink5", "nvlink4", "ib_ndr")},
            "links": {k: vars(v) for k, v in LINKS.items()}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--out", default="results/cluster.json")
    ap.add_argument("--skip", nargs="*", default=[])
    a = ap.parse_args(argv)
    res: dict[str, Any] = {}
    with tempfile.TemporaryDirectory(prefix="g2b_cluster_") as d:
        tmp = Path(d)
        for name, fn in (("resharding", lambda: measure_resharding(tmp)),
                         ("async_save", lambda: measure_async_save(tmp)),
                         ("prefetch", measure_prefetch),
                         ("failure_restart", lambda: measure_failure_restart(tmp)),
                         ("collectives", measure_collectives), ("fabric", model_the_fabric)):
            if name in a.skip:
                continue
            print(f"[{name}]", flush=True)
            res[name] = fn()
    out = Path(a.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(res, indent=1, default=str))
    ok = all(v["bitwise_identical"] for v in res.get("resharding", {}).get("reshards", {}).values()) and \
        res.get("failure_restart", {}).get("max_abs_loss_difference", 0.0) == 0.0
    print(("ok" if ok else "FAILED") + f" -> {out}")
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
