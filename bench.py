#!/usr/bin/env python3
"""Headline benchmark: GPT-2 124M training throughput, data parallel, on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

For N > 1 launch under torchrun (one process per GPU; RANK/LOCAL_RANK/
WORLD_SIZE/MASTER_* from the environment), e.g.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \
        --master-addr 127.0.0.1 --master-port 29500 bench.py --gpus 8

Config: GPT-2 small (12L, d=768, 12 heads, ctx 1024,
vocab 50257, tied embeddings), per-GPU micro-batch 16 x 1024 of uniform-random
tokens, random init, bf16 compute with fp32 master weights and fp32 gradient
all-reduce in 25 MiB buckets, AdamW (lr 3e-4, betas 0.9/0.95, wd 0.1) with
global-norm clipping at 1.0 -- every step is a full forward, backward,
all-reduce and optimiser update.

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the compute
stream; the step time is the MAX over ranks. Every step's working set (~10 GB
of activations and weights) is far larger than the 126 MB L2, so no L2 flush is
inserted. `value` is whole-job tokens/s (all N GPUs); `e2e` repeats the
measurement through the public `Trainer.step` call with each step's inputs
copied from pinned host memory and the loss read back to the host.

`--impl reference` runs the UNMODIFIED reference (baseline/_ref, installed from
the reference repository) through its own public API: its `GPT` under bf16
autocast, `torch.optim.AdamW` from `configure_optimizers`, its
`average_gradients` (25 MiB buckets over NCCL) for N > 1, and clipping.

`--strategy zero2` measures the same model and batch under ZeRO-2 instead of
DDP: natively the bucketed peer-memory reduce-scatter overlapped with backward
plus the fused clip/AdamW/bf16 all-gather kernel; on the reference arm its
`ShardedAdamW(stage=2, grad_clip=1.0, param_dtype=bf16)` over NCCL.
`--strategy zero3 --model gpt2-medium --batch 8` is BASELINE config 3: block
parameters sharded, gathered one block ahead over NVLink, gradients
reduce-scattered per block; the reference arm runs its `Zero3Model`
(param_dtype bf16) with `Zero3AdamW(grad_clip=1.0)`.
`--strategy tp --model gpt2-xl --batch 32` is BASELINE config 4: tensor +
sequence parallelism over all N GPUs with `--batch` the GLOBAL batch (strong
scaling); the reference has no tensor-parallel GPT training entry point (and
its TensorParallelBlock needs n_head % N == 0; XL has 25 heads), so its arm
prints `unavailable` for N > 1.
`--strategy cp --model gpt2-large --batch 1 --seq 16384` runs context
parallelism over all N GPUs (each GPU computes T/N tokens of every sequence,
causal all-gather of K/V over peer memory, weight gradients averaged like
DDP); the reference has no such entry point.
`--strategy pp --pp 4 --cp 2 --model gpt2-large --batch 1 --seq 16384
--micro-batches 8` is BASELINE config 5: pipeline parallelism (1F1B over NCCL
point-to-point, `--schedule gpipe` for GPipe) with context parallelism inside
every stage; `--batch` is the micro-batch and every step runs all
micro-batches (strong scaling: the global batch is fixed). The reference's
pipeline runs only inside its equivalence harness (pipeline_worker on the tiny
config), so its arm prints `unavailable`.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "GPT-2 train tokens/s & MFU at 1/2/4/8 B200 per strategy, max over ranks"
#: Reference's published GPT-2 124M training throughput (README.md:395; Apple
#: M1 Max, MPS, fp32, B4 x T256) -- the only published throughput it has.
BASELINE_TOKENS_PER_S = 4024.0


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 200 ms in a thread."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
                sm = float(parts[1])
                smax = float(parts[2])
                power = float(parts[3]) if parts[3] not in ("[N/A]", "N/A") else 0.0
            except ValueError:
                continue
            if idx in self.gpus:
                self.samples.append((idx, sm, smax, power, parts[5:9]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sms = [s[1] for s in self.samples]
        reasons = set()
        for s in self.samples:
            for name, val in zip(self.REASONS, s[4]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(s[2] for s in self.samples),
                "reasons": sorted(reasons), "samples": len(self.samples),
                "power_w_max": max(s[3] for s in self.samples)}


# ------------------------------------------------------------- distributed --
def setup_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch with torchrun for N>1")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier(device_ids=[torch.cuda.current_device()])


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def timed(step, steps: int, warmup: int, world: int, on_start=None, on_stop=None) -> float:
    """ms per step: warmup, then K steps bracketed by barrier+sync, CUDA events."""
    for i in range(warmup):
        step(i)
    barrier(world)
    torch.cuda.synchronize()
    if on_start:
        on_start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step(warmup + i)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    if on_stop:
        on_stop()
    ms = start.elapsed_time(end) / steps
    return max_over_ranks(ms, world)


def make_data(cfg, B, T, rank, pool=4):
    g = torch.Generator().manual_seed(1234 + rank)
    host = []
    for _ in range(pool):
        x = torch.randint(0, cfg.vocab_size, (B, T + 1), generator=g, dtype=torch.int64)
        host.append((x[:, :-1].contiguous().pin_memory(), x[:, 1:].contiguous().pin_memory()))
    dev = [(a.cuda(non_blocking=True), b.cuda(non_blocking=True)) for a, b in host]
    torch.cuda.synchronize()
    return host, dev


# ------------------------------------------------------------------- arms --
def tokens_per_step(args, world) -> int:
    if args.strategy == "pp":
        return args.micro_batches * args.batch * args.seq
    return args.batch * args.seq * (1 if args.strategy in ("tp", "cp") else world)


def run_pipeline(args, world, rank):
    """PP (x CP) arm: every rank receives the same global batch."""
    from gpt2_harness_b200.config import TrainConfig, gpt2_config
    from gpt2_harness_b200.ops import native as N
    from gpt2_harness_b200.trainer import PipelineTrainer

    cfg = gpt2_config(args.model, n_positions=max(args.seq, gpt2_config(args.model).n_positions))
    tc = TrainConfig(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, grad_clip=1.0, warmup_steps=0)
    cp = args.cp
    pp = args.pp or world // cp
    trainer = PipelineTrainer(cfg, args.batch, args.seq, args.micro_batches, pp=pp, cp=cp,
                              schedule=args.schedule, train=tc, comm_blocks=args.comm_blocks,
                              cp_balance=args.cp_balance, cp_kv=args.cp_kv)
    trainer.schedule = False
    host, dev = make_data(cfg, args.micro_batches * args.batch, args.seq, 0, pool=2)
    L = N.lib()

    def dev_step(i):
        idx, tgt = dev[i % len(dev)]
        trainer.step_async(idx, tgt)

    sampler = ClockSampler(gpu_list(world)) if rank == 0 else None
    launches = {}

    def start():
        launches["a"] = L.launch_count()
        if sampler:
            sampler.start()

    def stop():
        launches["b"] = L.launch_count()
        if sampler:
            sampler.stop()

    ms = timed(dev_step, args.steps, args.warmup, world, start, stop)
    trainer.check()
    n_launch = sum_over_ranks(launches["b"] - launches["a"], world)

    def e2e_step(i):
        idx, tgt = host[i % len(host)]
        trainer.step(idx, tgt)  # H2D of this rank's inputs + loss read back on the last stage

    ms_e2e = timed(e2e_step, args.steps, 1, world)
    trainer.check()
    bi = int(max_over_ranks(trainer.h2d_bytes_per_step, world))
    out = finish_line(args, world, cfg, ms, ms_e2e, bi, 4, sampler, impl="native")
    out["gpu_launches"] = int(n_launch)
    out["config"]["comm"] = "nccl p2p between stages, peer-memory kernels inside a CP group"
    out["config"]["pp"], out["config"]["cp"] = pp, cp
    out["config"]["micro_batches"], out["config"]["schedule"] = args.micro_batches, args.schedule
    out["config"]["cp_balance"] = args.cp_balance if cp > 1 else None
    out["config"]["cp_kv"] = args.cp_kv if cp > 1 else None
    trainer.close()
    return out


def run_native(args, world, rank):
    from gpt2_harness_b200.config import TrainConfig, gpt2_config
    from gpt2_harness_b200.ops import native as N
    from gpt2_harness_b200.trainer import Trainer

    if args.strategy == "pp":
        return run_pipeline(args, world, rank)

    # learned positions extended to the benchmark context when it is longer
    cfg = gpt2_config(args.model, n_positions=max(args.seq, gpt2_config(args.model).n_positions))
    tc = TrainConfig(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, grad_clip=1.0, warmup_steps=0)
    # default: one rank replays its step as a CUDA graph; several ranks only
    # with --graph on (measured at 2 ranks; at 8 its one run stalled)
    graph = (args.strategy == "ddp" and torch.cuda.is_available()
             and (args.graph == "on" or (args.graph == "auto" and world == 1))
             and (world == 1 or args.comm != "nccl"))
    trainer = Trainer(cfg, args.batch, args.seq, train=tc, comm=args.comm, schedule=False,
                      strategy=args.strategy, bucket_bytes=int(args.bucket_mb * 2**20),
                      comm_blocks=args.comm_blocks, cp_balance=args.cp_balance, cp_kv=args.cp_kv, graph=graph,
                      reduce_dtype=args.reduce_dtype)
    # tensor and context parallel ranks all take the same global batch
    host, dev = make_data(cfg, args.batch, args.seq, 0 if args.strategy in ("tp", "cp") else rank)
    L = N.lib()

    def dev_step(i):
        idx, tgt = dev[i % len(dev)]
        trainer.step_async(idx, tgt)

    sampler = ClockSampler(gpu_list(world)) if rank == 0 else None
    launches = {}

    def start():
        launches["a"] = L.launch_count()
        if sampler:
            sampler.start()

    def stop():
        launches["b"] = L.launch_count()
        if sampler:
            sampler.stop()

    ms = timed(dev_step, args.steps, args.warmup, world, start, stop)
    trainer.check()
    n_launch = sum_over_ranks(launches["b"] - launches["a"], world)
    if graph:
        # replays launch the captured kernels without passing the launchers
        n_launch = sum_over_ranks(trainer.graph_launches * args.steps, world)

    def e2e_step(i):
        idx, tgt = host[i % len(host)]
        trainer.step(idx, tgt)  # H2D from pinned memory + loss read back

    ms_e2e = timed(e2e_step, args.steps, 1, world)
    trainer.check()
    bi = 2 * args.batch * args.seq * 8  # idx + targets, int64
    bo = 4  # fp32 loss scalar
    out = finish_line(args, world, cfg, ms, ms_e2e, bi, bo, sampler, impl="native")
    out["gpu_launches"] = int(n_launch)
    out["config"]["comm"] = (args.comm if args.strategy == "ddp" else "p2p") if world > 1 else "none"
    out["config"]["cuda_graph"] = graph
    if args.reduce_dtype != "fp32":
        out["config"]["reduce_dtype"] = args.reduce_dtype
    if args.strategy == "cp":
        out["config"]["cp_balance"] = args.cp_balance
        out["config"]["cp_kv"] = args.cp_kv
    if args.strategy == "zero3":
        out["config"]["activations"] = "kept (no recompute): MFU counts the model FLOPs run"
        out["config"]["reduce_dtype"] = args.reduce_dtype
    trainer.close()
    return out


def run_reference(args, world, rank):
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "transformer_internals")):
        return {"impl": "reference", "unavailable": "baseline/_ref not installed"}
    sys.path.insert(0, ref_dir)
    from transformer_internals.config import gpt2_config as ref_config
    from transformer_internals.model import GPT as RefGPT
    from transformer_internals.parallel.data_parallel import average_gradients

    cfg = ref_config(args.model)
    if args.strategy == "pp":
        return {"impl": "reference", "unavailable": (
            "the reference's pipeline parallelism runs only inside its equivalence harness "
            "(pipeline_worker on the tiny config, blocking send/recv per micro-batch); it has no "
            "GPT-2 training entry point for a pipeline, and none composed with context parallelism")}
    if args.strategy == "cp":
        return {"impl": "reference", "unavailable": (
            "the reference has no context-parallel GPT training entry point (all_gather_kv_attention "
            "covers one attention call); at the long contexts CP is for, its single-GPU model "
            "materialises T x T attention scores per layer")}
    if args.strategy == "tp" and world > 1:
        why = ("the reference has no tensor-parallel GPT training entry point (its "
               "TensorParallelBlock covers single blocks, without a vocabulary-parallel head)")
        if cfg.n_head % world:
            why += f"; it also requires n_head % world == 0 ({args.model}: {cfg.n_head} heads)"
        return {"impl": "reference", "unavailable": why}
    torch.manual_seed(0)
    model = RefGPT(cfg).cuda()
    if world > 1:
        for p in model.parameters():
            dist.broadcast(p.data, src=0)
    host, dev = make_data(cfg, args.batch, args.seq, rank)
    if args.strategy == "zero3" and world > 1:
        from transformer_internals.parallel.zero import Zero3AdamW, Zero3Model

        zmodel = Zero3Model(model, rank, world, param_dtype=torch.bfloat16)
        zopt = Zero3AdamW(zmodel, lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, grad_clip=1.0)

        def train_step(idx, tgt):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = zmodel(idx, tgt)["loss"]
            zopt.zero_grad()
            loss.backward()
            zopt.step()
            return loss
    elif args.strategy == "zero2":
        from transformer_internals.parallel.zero import ShardedAdamW

        zopt = ShardedAdamW(list(model.parameters()), rank, world, stage=2, lr=3e-4,
                            betas=(0.9, 0.95), weight_decay=0.1, grad_clip=1.0,
                            param_dtype=torch.bfloat16)

        def train_step(idx, tgt):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = model(idx, tgt)["loss"]
            for p in model.parameters():
                p.grad = None
            loss.backward()
            zopt.step()
            return loss
    else:
        opt = model.configure_optimizers(0.1, 3e-4, (0.9, 0.95))

        def train_step(idx, tgt):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = model(idx, tgt)["loss"]
            opt.zero_grad(set_to_none=True)
            loss.backward()
            if world > 1:
                average_gradients(model.parameters(), world)
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            opt.step()
            return loss

    def dev_step(i):
        idx, tgt = dev[i % len(dev)]
        train_step(idx, tgt)

    sampler = ClockSampler(gpu_list(world)) if rank == 0 else None
    ms = timed(dev_step, args.steps, args.warmup, world,
               sampler.start if sampler else None, sampler.stop if sampler else None)

    def e2e_step(i):
        idx, tgt = host[i % len(host)]
        loss = train_step(idx.cuda(non_blocking=True), tgt.cuda(non_blocking=True))
        loss.item()

    ms_e2e = timed(e2e_step, args.steps, 1, world)
    bi = 2 * args.batch * args.seq * 8
    return finish_line(args, world, cfg, ms, ms_e2e, bi, 4, sampler, impl="reference")


def gpu_list(world):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return [int(x) for x in vis.split(",")][:world]
        except ValueError:
            pass
    return list(range(world))


def finish_line(args, world, cfg, ms, ms_e2e, bi, bo, sampler, impl):
    from gpt2_harness_b200.perf.mfu import flops_per_token_exact, measured_peak_tflops

    tokens = tokens_per_step(args, world)
    tps = tokens / (ms / 1e3)
    tps_e2e = tokens / (ms_e2e / 1e3)
    fpt = flops_per_token_exact(cfg, args.seq)["training_flops_per_token"]
    peak, label = measured_peak_tflops(sustained=True)
    mfu = fpt * tps / (peak * 1e12 * world)
    clocks = sampler.summary() if sampler else {}
    line = {
        "metric": METRIC,
        "value": round(tps, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "strong" if args.strategy in ("tp", "cp", "pp") else "weak",
        "vs_baseline": round(tps / BASELINE_TOKENS_PER_S, 2),
        "dtype": "bf16",
        "data": "synthetic uniform-random tokens, random-init weights",
        "mfu": round(mfu, 4),
        "mfu_peak": f"{peak} TFLOP/s per GPU, {label}",
        "flops_per_token": fpt,
        "config": {
            "model": {"gpt2": "gpt2 (124M)", "gpt2-medium": "gpt2-medium (350M)",
                      "gpt2-large": "gpt2-large (774M)", "gpt2-xl": "gpt2-xl (1.5B)"}.get(args.model, args.model),
            "global_batch": tokens // args.seq,
            "per_gpu_batch": args.batch if args.strategy not in ("tp", "cp", "pp") else None,
            "seq_len": args.seq,
            "parallelism": (f"dp{world}" if args.strategy == "ddp" else
                            f"tp{world}-sp" if args.strategy == "tp" else
                            f"cp{world}" if args.strategy == "cp" else
                            f"pp{args.pp or world // args.cp}xcp{args.cp}-{args.schedule}"
                            if args.strategy == "pp" else f"{args.strategy}-dp{world}"),
            "strategy": args.strategy,
            "bucket_mb": args.bucket_mb,
            "optimizer": "AdamW + clip 1.0, fp32 master",
            "l2": "inputs larger than L2 (per-step working set ~10 GB >> 126 MB), no flush",
            "baseline": "README.md:395 (M1 Max MPS fp32, B4xT256, 4024 tokens/s)",
        },
        "e2e": {"value": round(tps_e2e, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                "ms_per_step": round(ms_e2e, 3)},
        "clocks": {k: clocks.get(k) for k in ("sm_mhz", "sm_max_mhz", "reasons")},
        "peak_mem_gb": round(max_over_ranks(torch.cuda.max_memory_allocated() / 1e9, world), 2),
        "impl": impl,
    }
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--model", default="gpt2")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--comm", choices=["p2p", "mc", "nccl"], default="p2p")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="DDP: replay the step (forward, backward, bucket all-reduces, optimiser) "
                         "as one CUDA graph; auto = one rank only")
    ap.add_argument("--strategy", choices=["ddp", "zero2", "zero3", "tp", "cp", "pp"], default="ddp")
    ap.add_argument("--reduce-dtype", choices=["fp32", "bf16"], default="fp32",
                    help="gradient wire of DDP buckets and ZeRO-3 reduce-scatters / root all-reduces")
    ap.add_argument("--pp", type=int, default=0, help="pipeline stages (pp strategy; default N / cp)")
    ap.add_argument("--cp", type=int, default=1, help="context-parallel ranks per stage (pp strategy)")
    ap.add_argument("--micro-batches", type=int, default=8, help="micro-batches per step (pp strategy)")
    ap.add_argument("--schedule", choices=["1f1b", "gpipe"], default="1f1b")
    ap.add_argument("--cp-balance", choices=["zigzag", "contiguous"], default="zigzag",
                    help="context-parallel split (cp and pp strategies)")
    ap.add_argument("--cp-kv", choices=["gather", "stream"], default="gather",
                    help="context-parallel keys/values: gathered before attention, or read in place "
                         "from their owners by the attention kernels")
    ap.add_argument("--bucket-mb", type=float, default=25.0, help="gradient bucket size (MiB)")
    ap.add_argument("--comm-blocks", type=int, default=128,
                    help="CTAs of each fused all-reduce that overlaps backward")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world, rank, _ = setup_dist(args.gpus)
    try:
        if args.impl == "reference":
            out = run_reference(args, world, rank)
        else:
            out = run_native(args, world, rank)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
