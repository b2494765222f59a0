"""Native context parallelism (per-layer causal all-gather of K/V over peer
memory, dK/dV reduce-scatter, weight gradients averaged over the group)
against the single-GPU engine on the full sequences: loss and every
gradient. Child processes, one per GPU; the 2-GPU case is skipped when fewer
are visible."""

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
    from gpt2_harness_b200.parallel.cp_native import NativeCP
    from gpt2_harness_b200.parallel.ddp_native import NativeDDP
    from gpt2_harness_b200.parallel import comms
    from gpt2_harness_b200.ops import native as N

    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cfg = gpt2_config("gpt2", **json.loads(os.environ.get("G2B_CFG", '{"n_layer": 2, "n_positions": 1024}')))
    B, T = 2, int(os.environ.get("G2B_T", "1024"))
    Tl = T // world
    cp = NativeCP(cfg, B, T, balance=os.environ["G2B_BALANCE"], kv=os.environ.get("G2B_KV", "gather"))
    ddp = NativeDDP(ParamLayout(cfg), comm="p2p")
    eng = Engine(cfg, "cuda", grad_buffer=ddp.grad_buffer, seed=0)
    ddp.attach(eng)
    cp.attach(eng)
    ref = Engine(cfg, "cuda", seed=0)
    g = torch.Generator().manual_seed(11)
    idx = torch.randint(0, cfg.vocab_size, (B, T), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (B, T), generator=g).cuda()
    idx_l = cp.local_tokens(idx, torch.empty(B, Tl, dtype=idx.dtype, device="cuda"))
    tgt_l = cp.local_tokens(tgt, torch.empty(B, Tl, dtype=tgt.dtype, device="cuda"))
    with comms.counter_scope(world) as ctr:
        loss = eng.forward(idx_l, tgt_l)
        eng.backward(idx_l); ddp.finish()
        ctr.steps += 1
        torch.cuda.synchronize()
        N.check_errors()
        summary = ctr.summary()
    mean_loss = loss.clone(); dist.all_reduce(mean_loss); mean_loss /= world
    ref_loss = float(ref.forward(idx, tgt).item())
    ref.backward(idx)
    torch.cuda.synchronize()
    errs = {}
    for s in ref.layout.specs:
        r = ref.g32(s.name)
        errs[s.name] = ((eng.g32(s.name) - r).norm() / (r.norm() + 1e-12)).item()
    worst = max(errs, key=errs.get)
    out = {"rank": rank, "loss": float(mean_loss.item()), "ref_loss": ref_loss, "worst": worst,
           "worst_err": errs[worst], "payload": summary["payload_bytes_per_step"],
           "device_bytes": int(cp.byte_counter.item()) + int(ddp.byte_counter.item())}
    print("RESULT " + json.dumps(out), flush=True)
    ddp.close(); cp.close()
    dist.destroy_process_group()
''')


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, balance: str, cfg: dict | None = None, kv: str = "gather"):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), G2B_ROOT=ROOT,
                   NCCL_NVLS_ENABLE="0", G2B_BALANCE=balance, G2B_KV=kv)
        if cfg is not None:
            env["G2B_CFG"] = json.dumps(cfg)
            env["G2B_T"] = str(cfg["n_positions"])
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
            raise AssertionError("CP workers timed out:\n" + "\n-----\n".join(o[-4000:] for o in outs))
        assert p.returncode == 0, out[-3000:]
        line = [l for l in out.splitlines() if l.startswith("RESULT ")]
        assert line, out[-3000:]
        results.append(json.loads(line[-1][7:]))
    return results


# zig-zag at 8 ranks needs T / 16 a multiple of 128: T = 2048
LARGE = {"n_layer": 2, "n_embd": 1280, "n_head": 20, "n_positions": 2048}


@pytest.mark.parametrize("world,balance,cfg", [(1, "zigzag", None), (2, "contiguous", None),
                                               (2, "zigzag", None), (8, "zigzag", LARGE)])
def test_native_cp_matches_single_gpu(world, balance, cfg):
    res = _run(world, balance, cfg)
    print(res)
    for r in res:
        assert abs(r["loss"] - r["ref_loss"]) < 1e-3 * abs(r["ref_loss"]), r
        assert r["worst_err"] < 2e-2, r
        if world > 1:
            # K/V gathers, dK/dV reduce-scatters and the weight-gradient
            # all-reduce, charged by the kernels in the reference convention
            assert r["device_bytes"] == r["payload"], r


# Keys and values streamed from their owners inside the attention kernels
# (NativeCP(kv="stream")). These kernels have not yet run on a GPU; until
# they have, the cases run only with G2B_CP_STREAM_GPU=1 (after the one-GPU
# checks in test_cp_stream_gpu.py).
@pytest.mark.skipif(os.environ.get("G2B_CP_STREAM_GPU") != "1",
                    reason="streamed-KV kernels: set G2B_CP_STREAM_GPU=1 to run")
@pytest.mark.parametrize("world,balance,cfg", [(2, "contiguous", None), (2, "zigzag", None),
                                               (8, "zigzag", LARGE)])
def test_native_cp_streamed_kv_matches_single_gpu(world, balance, cfg):
    res = _run(world, balance, cfg, kv="stream")
    print(res)
    for r in res:
        assert abs(r["loss"] - r["ref_loss"]) < 1e-3 * abs(r["ref_loss"]), r
        assert r["worst_err"] < 2e-2, r
        assert r["device_bytes"] == r["payload"], r
