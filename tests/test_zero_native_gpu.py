"""Native ZeRO-2 (bucketed peer-memory reduce-scatter + fused clip/AdamW/bf16
all-gather) against the unsharded engine with an NCCL-averaged gradient, over
three optimiser steps with clipping active, each step started from the same
state. Child processes, one per GPU; the
2-GPU case is skipped when fewer GPUs are visible."""

import json
import os
import socket
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = textwrap.dedent(r'''
    import os, sys, json, datetime
    import torch, torch.distributed as dist
    sys.path.insert(0, os.environ["G2B_ROOT"])
    from gpt2_harness_b200.config import gpt2_config
    from gpt2_harness_b200.models.engine import Engine, OptimConfig, ParamLayout
    from gpt2_harness_b200.parallel.zero_native import NativeZeRO
    from gpt2_harness_b200.parallel import comms
    from gpt2_harness_b200.ops import native as N

    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cfg = gpt2_config("gpt2", **json.loads(os.environ.get("G2B_CFG", '{"n_layer": 2, "n_positions": 256}')))
    layout = ParamLayout(cfg)
    opt = dict(lr=1e-3, grad_clip=0.5)   # small enough that clipping is active
    zero = NativeZeRO(layout, bucket_bytes=4 * 1024 * 1024)
    eng = Engine(cfg, "cuda", optim=OptimConfig(**opt), grad_buffer=zero.grad_buffer,
                 shadow_buffer=zero.shadow_buffer, seed=0, optimizer_state=False)
    zero.attach(eng)
    ref = Engine(cfg, "cuda", optim=OptimConfig(**opt), seed=0)
    g = torch.Generator().manual_seed(100 + rank)
    losses, ref_losses, grad_errs, merrs = [], [], [], []
    with comms.counter_scope(world) as ctr:
        for step in range(3):
            # bf16 parameters make multi-step trajectories chaotic (a last-bit
            # master difference can flip a bf16 rounding), so every step starts
            # the unsharded engine from the sharded one's exact state
            with comms.counter_scope(world):
                ref.master.copy_(zero.full_master()); ref.sync_shadow()
                ref.exp_avg.copy_(zero.gather_full(zero.exp_avg))
                ref.exp_avg_sq.copy_(zero.gather_full(zero.exp_avg_sq))
            idx = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).cuda()
            tgt = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).cuda()
            losses.append(float(eng.forward(idx, tgt).item()))
            eng.backward(idx); zero.finish(); eng.optimizer_step()
            ctr.steps += 1
            ref_losses.append(float(ref.forward(idx, tgt).item()))
            ref.backward(idx)
            dist.all_reduce(ref.grad); ref.grad /= world
            # the averaged gradient shard against the NCCL-averaged gradient
            gerr = 0.0
            for f0, n, off in zero.plan.owned(rank):
                if n:
                    d = (zero.gsh[off:off + n] - ref.grad[f0:f0 + n]).abs().max().item()
                    gerr = max(gerr, d / (ref.grad.abs().max().item() + 1e-30))
            grad_errs.append(gerr)
            ref.optimizer_step()
            with comms.counter_scope(world):
                full = zero.full_master()
            merrs.append(((full - ref.master).abs().max() / ref.master.abs().max()).item())
        torch.cuda.synchronize()
        N.check_errors()
        summary = ctr.summary()
    err = max(merrs)
    sh_err = ((eng.shadow.float() - ref.shadow.float()).abs().max()).item()
    other = eng.shadow.clone(); dist.broadcast(other, 0)
    out = {"rank": rank, "master_rel_err": err, "shadow_max_abs": sh_err,
           "ranks_equal": bool(torch.equal(other, eng.shadow)),
           "loss_diff": max(abs(a - b) for a, b in zip(losses, ref_losses)),
           "norm": float(zero.grad_norm.item()), "ref_norm": float(ref.grad_norm.item()),
           "payload_per_step": summary["payload_bytes_per_step"], "total": layout.total,
           "device_bytes": int(zero.byte_counter.item()),
           "shard_numel": zero.plan.shard_numel, "grad_errs": grad_errs, "master_errs": merrs}
    print("RESULT " + json.dumps(out), flush=True)
    zero.close()
    dist.destroy_process_group()
''')


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, cfg: dict | None = None):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), G2B_ROOT=ROOT,
                   NCCL_NVLS_ENABLE="0")
        if cfg is not None:
            env["G2B_CFG"] = json.dumps(cfg)
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    results = []
    for p in procs:
        out, _ = p.communicate(timeout=300)
        assert p.returncode == 0, out[-3000:]
        line = [l for l in out.splitlines() if l.startswith("RESULT ")]
        assert line, out[-3000:]
        results.append(json.loads(line[-1][7:]))
    return results


@pytest.mark.parametrize("world", [1, 2, 8])
def test_native_zero2_matches_unsharded(world):
    res = _run(world)
    print(res)
    for r in res:
        assert max(r["grad_errs"]) < 1e-6, r
        # the reference's 1e-5 class: at 8 ranks the fp32 sums run in another
        # order than the unsharded step's (measured 2.0e-6)
        assert r["master_rel_err"] < 1e-5, r
        assert r["shadow_max_abs"] < 1e-2, r
        assert r["ranks_equal"], r
        assert r["loss_diff"] < 1e-4, r
        assert abs(r["norm"] - r["ref_norm"]) <= 1e-4 * r["ref_norm"], r
        # reduce-scatter 4T + bf16 all-gather 2T + 4-byte norm all-reduce
        assert r["payload_per_step"] == 6 * r["total"] + 4, r
        assert r["device_bytes"] == 3 * (6 * r["total"] + 4), r
        assert r["shard_numel"] * world >= r["total"]
