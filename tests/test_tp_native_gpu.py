"""Native tensor + sequence parallelism (csrc/tp.cu kernels around the engine
GEMM/attention/LayerNorm) against the single-GPU engine on the same weights
and batch: loss, every reference-named gradient and the AdamW update. A
3-head model so that 2 ranks split the heads unevenly (2 + 1); the optimiser is then checked on identical gradients. Child
processes, one per GPU; the 2-GPU case is skipped when fewer are visible."""

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
    from gpt2_harness_b200.models.engine import Engine, OptimConfig
    from gpt2_harness_b200.parallel.tp_native import TPEngine
    from gpt2_harness_b200.parallel import comms
    from gpt2_harness_b200.ops import native as N

    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cfg = gpt2_config("gpt2", **json.loads(os.environ.get("G2B_CFG", '{"n_layer": 2, "n_embd": 192, "n_head": 3, "n_positions": 256}')))
    B, T = 2, 256
    opt = OptimConfig(lr=1e-3, grad_clip=1.0)
    tp = TPEngine(cfg, B, T, optim=opt, seed=0)
    ref = Engine(cfg, "cuda", optim=OptimConfig(lr=1e-3, grad_clip=1.0), seed=0)
    ref.fuse_bias_grad_into_ln = False
    g = torch.Generator().manual_seed(7)   # the same global batch on every rank
    idx = torch.randint(0, cfg.vocab_size, (B, T), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (B, T), generator=g).cuda()
    print("init done", flush=True)
    dev0 = int(tp.byte_counter.item())
    with comms.counter_scope(world) as ctr:
        loss = float(tp.forward(idx, tgt).item())
        print("forward done", loss, flush=True)
        N.check_errors()
        tp.backward()
        torch.cuda.synchronize()
        print("backward done", flush=True)
        ctr.steps += 1
        torch.cuda.synchronize()
        N.check_errors()
        summary = ctr.summary()
    device_bytes = int(tp.byte_counter.item()) - dev0
    ref_loss = float(ref.forward(idx, tgt).item())
    ref.backward(idx)
    grads = tp.full_state("grad")
    errs = {}
    for name, gv in grads.items():
        r = ref.g32(name)
        errs[name] = ((gv - r).norm() / (r.norm() + 1e-12)).item()
    # the optimiser in isolation: the same gradients on both sides
    tp.load_full_grads(ref.layout, ref.grad)
    tp.optimizer_step(); ref.optimizer_step()
    torch.cuda.synchronize()
    N.check_errors()
    master = tp.full_state("master")
    upd = max(((master[n] - ref.p32(n)).abs().max() / (ref.p32(n).abs().max() + 1e-12)).item()
              for n in master)
    worst = max(errs, key=errs.get)
    print("grad errors", sorted(errs.items(), key=lambda kv: -kv[1])[:8], flush=True)
    out = {"rank": rank, "loss": loss, "ref_loss": ref_loss, "worst_grad": worst,
           "worst_grad_err": errs[worst], "update_err": upd,
           "payload": summary["payload_bytes_per_step"], "device_bytes": device_bytes,
           "M": B * T, "C": cfg.n_embd,
           "norm": float(tp.grad_norm.item()), "ref_norm": float(ref.grad_norm.item())}
    print("RESULT " + json.dumps(out), flush=True)
    tp.close()
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
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            outs = [q.communicate()[0] for q in procs]
            raise AssertionError("TP workers timed out:\n" + "\n-----\n".join(o[-4000:] for o in outs))
        assert p.returncode == 0, out[-3000:]
        line = [l for l in out.splitlines() if l.startswith("RESULT ")]
        assert line, out[-3000:]
        results.append(json.loads(line[-1][7:]))
    return results


# the BASELINE tensor-parallel mesh: 8 ranks at GPT-2 XL widths (25 heads split
# 4 + 3 x 7, 2 of its 48 layers)
XL = {"n_layer": 2, "n_embd": 1600, "n_head": 25, "n_positions": 256}


@pytest.mark.parametrize("world,cfg", [(1, None), (2, None), (8, XL)])
def test_native_tp_matches_single_gpu(world, cfg):
    res = _run(world, cfg)
    print(res)
    for r in res:
        assert abs(r["loss"] - r["ref_loss"]) < 2e-3 * abs(r["ref_loss"]), r
        assert r["worst_grad_err"] < 3e-2, r
        assert abs(r["norm"] - r["ref_norm"]) < 1e-5 * r["ref_norm"], r  # same gradients
        assert r["update_err"] < 1e-5, r
        if world > 1:
            # the kernels' own byte counters charge the reference convention
            assert r["device_bytes"] == r["payload"], r
    assert len({round(r["loss"], 6) for r in res}) == 1  # every rank sees the same loss
