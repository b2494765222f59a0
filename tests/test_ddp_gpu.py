"""Native DDP on 2 GPUs: the fused peer-memory all-reduce (and the NCCL arm)
against the mean of each rank's own gradients; exact payload accounting;
bounded-wait failure path. Runs as child processes (one per GPU); skipped
when fewer than 2 GPUs are visible."""

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
    from gpt2_harness_b200.models.engine import Engine, ParamLayout
    from gpt2_harness_b200.parallel.ddp_native import NativeDDP
    from gpt2_harness_b200.parallel import comms
    from gpt2_harness_b200.ops import native as N

    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    comm = os.environ["G2B_COMM"]
    cfg = gpt2_config("gpt2", **json.loads(os.environ.get("G2B_CFG", '{"n_layer": 2, "n_positions": 256}')))
    layout = ParamLayout(cfg)
    ddp = NativeDDP(layout, comm=comm, bucket_bytes=4 * 1024 * 1024,
                    reduce_dtype=os.environ.get("G2B_REDUCE", "fp32"))
    eng = Engine(cfg, "cuda", grad_buffer=ddp.grad_buffer, seed=0)
    ddp.attach(eng)
    solo = Engine(cfg, "cuda", seed=0)      # same weights, no communication
    g = torch.Generator().manual_seed(100 + rank)
    idx = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).cuda()
    out = {}
    with comms.counter_scope(world) as ctr:
        for step in range(2):
            eng.forward(idx, tgt); eng.backward(idx); ddp.finish()
            ctr.steps += 1
        torch.cuda.synchronize()
        N.check_errors()
        summary = ctr.summary()
    solo.forward(idx, tgt); solo.backward(idx)
    mine = solo.grad.clone()
    dist.all_reduce(mine)                    # NCCL reference: sum, then mean
    mine /= world
    got = eng.grad if comm != "nccl" else eng.grad * ddp.grad_scale
    err = ((got - mine).abs().max() / (mine.abs().max() + 1e-12)).item()
    other = got.clone(); dist.broadcast(other, 0)
    out = {"rank": rank, "rel_err": err, "ranks_equal": bool(torch.equal(other, got)),
           "payload_per_step": summary["payload_bytes_per_step"],
           "n_params": layout.num_parameters,
           "device_bytes": int(ddp.byte_counter.item()), "calls": summary["total_calls"]}
    print("RESULT " + json.dumps(out), flush=True)
    ddp.close()
    dist.destroy_process_group()
''')


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(comm: str, world: int = 2, cfg: dict | None = None, reduce_dtype: str = "fp32"):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import json
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), G2B_ROOT=ROOT, G2B_COMM=comm,
                   G2B_REDUCE=reduce_dtype)
        if comm != "mc":
            env["NCCL_NVLS_ENABLE"] = "0"
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


# 2 ranks on a 2-layer GPT-2 small; the BASELINE data-parallel mesh (8 ranks)
# at GPT-2 small widths with 2 of its 12 layers
@pytest.mark.parametrize("comm,world", [("p2p", 2), ("nccl", 2), ("mc", 2), ("p2p", 8), ("mc", 8)])
def test_native_ddp_two_gpus(comm, world):
    if comm == "mc" and not _multicast():
        pytest.skip("no NVLink multicast on this system")
    res = _run(comm, world)
    for r in res:
        assert r["rel_err"] < 1e-5, r
        assert r["ranks_equal"], r
        # reference convention: one fp32 copy of every gradient per step
        assert r["payload_per_step"] == 4 * r["n_params"], r
    if comm in ("p2p", "mc"):
        # the in-kernel counter charges the same payload: 4N per step x 2 steps
        assert res[0]["device_bytes"] == 2 * 4 * res[0]["n_params"], res[0]


@pytest.mark.parametrize("comm", ["p2p", "nccl"])
def test_native_ddp_bf16_wire(comm):
    """The reference's bf16 gradient wire: buckets cast to bf16 copies, reduced
    (the P2P kernel sums in fp32), cast back; 2N bytes a step."""
    res = _run(comm, 2, reduce_dtype="bf16")
    for r in res:
        assert r["rel_err"] < 1e-2, r
        assert r["ranks_equal"], r
        assert r["payload_per_step"] == 2 * r["n_params"], r
    if comm == "p2p":
        assert res[0]["device_bytes"] == 2 * 2 * res[0]["n_params"], res[0]


def _multicast() -> bool:
    from gpt2_harness_b200.parallel.symm import multicast_supported
    return torch.cuda.device_count() > 1 and multicast_supported(torch.device("cuda", 0))


GRAPH_WORKER = textwrap.dedent(r'''
    import os, sys, json, datetime
    import torch, torch.distributed as dist
    sys.path.insert(0, os.environ["G2B_ROOT"])
    from gpt2_harness_b200.config import gpt2_config, TrainConfig
    from gpt2_harness_b200.trainer import Trainer

    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cfg = gpt2_config("gpt2", n_layer=2, n_positions=256)
    tc = TrainConfig(lr=1e-3, warmup_steps=0)
    out = {"rank": rank}
    for graph in (False, True):
        tr = Trainer(cfg, 2, 256, train=tc, schedule=False, seed=0, comm=os.environ["G2B_COMM"],
                     bucket_bytes=4 * 1024 * 1024, graph=graph)
        losses = []
        for step in range(5):
            g = torch.Generator().manual_seed(100 * step + rank)
            idx = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).pin_memory()
            tgt = torch.randint(0, cfg.vocab_size, (2, 256), generator=g).pin_memory()
            losses.append(tr.step(idx, tgt))
        tr.check()
        out["graph" if graph else "eager"] = losses
        out["master_" + ("graph" if graph else "eager")] = float(tr.engine.master.double().sum().item())
        out["launches"] = tr.graph_launches
        tr.close()
    print("RESULT " + json.dumps(out), flush=True)
    dist.destroy_process_group()
''')


@pytest.mark.parametrize("comm", ["p2p", "mc"])
def test_ddp_graph_replay_matches_eager(comm):
    """The DDP step captured as one CUDA graph (bucket all-reduces on the comm
    stream, device-side epochs) replays the eager step exactly on 2 ranks."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if comm == "mc" and not _multicast():
        pytest.skip("no NVLink multicast on this system")
    import json
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), G2B_ROOT=ROOT, G2B_COMM=comm)
        if comm != "mc":
            env["NCCL_NVLS_ENABLE"] = "0"
        procs.append(subprocess.Popen([sys.executable, "-c", GRAPH_WORKER], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    for p in procs:
        out, _ = p.communicate(timeout=300)
        assert p.returncode == 0, out[-3000:]
        line = [l for l in out.splitlines() if l.startswith("RESULT ")]
        assert line, out[-3000:]
        r = json.loads(line[-1][7:])
        if comm == "p2p":  # fixed-order sums: bit-identical
            assert r["graph"] == r["eager"], r
            assert r["master_graph"] == r["master_eager"], r
        else:              # the switch's summation order is its own
            assert all(abs(a - b) <= 1e-5 * abs(b) for a, b in zip(r["graph"], r["eager"])), r
        assert r["launches"] > 0, r
