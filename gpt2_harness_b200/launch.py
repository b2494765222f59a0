"""Distributed training job (one process per GPU, under torchrun / srun / a
Kubernetes indexed job / Ray): the native B200 engine with fused,
backward-overlapped gradient all-reduce, a resumable sharded token stream,
and asynchronous sharded checkpoints in the reference's format.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m gpt2_harness_b200.launch \\
        --model gpt2 --data tokens.bin --steps 5000 --ckpt-dir ckpt --ckpt-every 500

On start it resumes from the newest complete checkpoint under ``--ckpt-dir``
(model, AdamW moments, optimiser step, every rank's stream position), so a
requeued job (Slurm ``--requeue``, a restarted pod) continues where it left
off; checkpoints are written by rank 0 to ``step_<n>/`` and swapped in
atomically. ``SIGUSR1`` / ``SIGTERM`` (the pre-emption warning of most
schedulers) trigger a checkpoint at the next step boundary, then a clean exit.

Strategies: ``ddp`` / ``zero2`` / ``zero3`` (each rank reads its own shard of
the token stream, ``--batch`` per GPU); ``tp`` (tensor + sequence
parallelism) and ``cp`` (context parallelism): every rank reads the same
``--batch`` sequences;
``pp`` (pipeline x context parallelism over a ``--pp`` x ``--cp`` mesh: every
rank reads the same ``--micro-batches`` x ``--batch`` sequences per step). A
pipeline checkpoint holds the full model with the untied ``lm_head.weight``
and every stage's AdamW moments, gathered on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import time
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist

from .cluster.checkpoint import AsyncCheckpointer, engine_state_dict, load_full, load_extra, load_into_engine
from .cluster.streaming import ShardedStream, StreamState, TokenShardSource
from .config import TrainConfig, gpt2_config
from .trainer import PipelineTrainer, Trainer

__all__ = ["latest_checkpoint", "main"]

_STOP = {"flag": False}
#: Set to a list to record every step's loss in-process (tests).
LOSSES: Optional[list] = None


def _on_signal(signum, _frame) -> None:
    _STOP["flag"] = True


def latest_checkpoint(ckpt_dir) -> Optional[Path]:
    d = Path(ckpt_dir)
    if not d.is_dir():
        return None
    steps = sorted((int(p.name.split("_")[1]), p) for p in d.glob("step_*") if (p / "index.json").exists())
    return steps[-1][1] if steps else None


class _SyntheticTokens:
    """Uniform random windows (the benchmark's data) as a stream source."""

    def __init__(self, vocab: int, block: int, n: int = 1 << 20, seed: int = 0) -> None:
        self.vocab, self.block, self.n, self.seed = vocab, block, n, seed

    def __len__(self) -> int:
        return self.n

    def __getitem__(self, i: int):
        g = torch.Generator().manual_seed(self.seed * 1_000_003 + int(i))
        w = torch.randint(0, self.vocab, (self.block + 1,), generator=g)
        return w[:-1], w[1:]


def _pipeline_checkpoint(trainer: "PipelineTrainer", world: int) -> tuple[dict, dict]:
    """(tensors, optimiser state by name) of the whole pipeline on rank 0
    (a collective: every rank sends its stage; CP ranks of a stage hold
    identical copies, the first one's is kept)."""
    mine = trainer.state_dict()
    mine = {"model": {k: v.cpu() for k, v in mine["model"].items()},
            "optim": {"step": mine["optim"]["step"],
                      "exp_avg": {k: v.cpu() for k, v in mine["optim"]["exp_avg"].items()},
                      "exp_avg_sq": {k: v.cpu() for k, v in mine["optim"]["exp_avg_sq"].items()}}}
    parts = [None] * world if dist.get_rank() == 0 else None
    dist.gather_object(mine, parts, dst=0)
    if dist.get_rank() != 0:
        return {}, {}
    model, ea, eq = {}, {}, {}
    for p in parts:
        for k, v in p["model"].items():
            model.setdefault(k, v)
        for k, v in p["optim"]["exp_avg"].items():
            ea.setdefault(k, v)
        for k, v in p["optim"]["exp_avg_sq"].items():
            eq.setdefault(k, v)
    return model, {"step": parts[0]["optim"]["step"], "exp_avg": ea, "exp_avg_sq": eq}


def _load_tp(engine, full: dict, extra: dict) -> None:
    """Restore a tensor-parallel engine from a full-model checkpoint (and the
    AdamW moments a tensor-parallel checkpoint carries)."""
    from .models.engine import ParamLayout

    layout = ParamLayout(engine.config)

    def flat(named):
        v = torch.zeros(layout.total, dtype=torch.float32, device=engine.device)
        for s in layout.specs:
            layout.view(v, s.name).copy_(named[s.name].to(v.device, torch.float32).view(s.shape))
        return v

    m = extra.get("tp_exp_avg")
    engine.load_full(layout, flat(full), flat(m) if m else None,
                     flat(extra["tp_exp_avg_sq"]) if m else None)
    engine.step_count = int(extra.get("optim_step", engine.step_count))


def main(argv=None, device: Optional[torch.device] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="gpt2")
    ap.add_argument("--data", default=None, help="uint16 token file; synthetic tokens when absent")
    ap.add_argument("--batch", type=int, default=16, help="per-GPU micro-batch")
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--lr", type=float, default=6e-4)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--comm", choices=["p2p", "mc", "nccl"], default="p2p")
    ap.add_argument("--ckpt-dir", default=None)
    ap.add_argument("--ckpt-every", type=int, default=500)
    ap.add_argument("--log", default=None, help="JSONL metrics (rank 0)")
    ap.add_argument("--strategy", choices=["ddp", "zero2", "zero3", "tp", "cp", "pp"], default="ddp")
    ap.add_argument("--pp", type=int, default=0, help="pipeline stages (pp; default WORLD_SIZE / --cp)")
    ap.add_argument("--cp", type=int, default=1, help="context-parallel ranks per stage (pp)")
    ap.add_argument("--micro-batches", type=int, default=8, help="micro-batches per step (pp)")
    ap.add_argument("--schedule", choices=["1f1b", "gpipe"], default="1f1b")
    ap.add_argument("--cp-balance", choices=["zigzag", "contiguous"], default="zigzag")
    ap.add_argument("--cp-kv", choices=["gather", "stream"], default="gather",
                    help="context-parallel keys/values: gathered, or streamed from their owners")
    ap.add_argument("--stop-at", type=int, default=0,
                    help="checkpoint and exit after this step (a time-boxed allocation); the LR "
                         "schedule still spans --steps")
    ap.add_argument("--config", default=None,
                    help="GPTConfig overrides as a JSON object or a path to one (e.g. a smaller model)")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)

    if dist.is_initialized():
        world, rank = dist.get_world_size(), dist.get_rank()
    else:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if device is None:
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    dev = torch.device(device)
    _external_group = dist.is_initialized()
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(minutes=10))
    for s in (signal.SIGUSR1, signal.SIGTERM):
        signal.signal(s, _on_signal)

    overrides = {}
    if a.config:
        text = a.config if a.config.lstrip().startswith("{") else Path(a.config).read_text()
        overrides = json.loads(text)
    base = gpt2_config(a.model, **overrides)
    cfg = gpt2_config(a.model, **{**overrides, "n_positions": max(a.seq, base.n_positions)})
    tc = TrainConfig(steps=a.steps, batch_size=a.batch, block_size=a.seq, lr=a.lr, warmup_steps=a.warmup)
    pipeline = a.strategy == "pp"
    if pipeline:
        trainer = PipelineTrainer(cfg, a.batch, a.seq, a.micro_batches, pp=a.pp or world // a.cp, cp=a.cp,
                                  schedule=a.schedule, train=tc, device=dev, seed=a.seed,
                                  cp_balance=a.cp_balance, cp_kv=a.cp_kv)
    else:
        trainer = Trainer(cfg, a.batch, a.seq, train=tc, comm=a.comm, device=dev, seed=a.seed,
                          strategy=a.strategy, cp_balance=a.cp_balance, cp_kv=a.cp_kv)
    # data-parallel ranks read disjoint shards of the stream; the ranks of a
    # context-parallel group or a pipeline all read the same sequences
    shared = a.strategy in ("tp", "cp", "pp")
    s_rank, s_world = (0, 1) if shared else (rank, world)
    rows = a.micro_batches * a.batch if pipeline else a.batch
    src = TokenShardSource(a.data, a.seq) if a.data else _SyntheticTokens(cfg.vocab_size, a.seq, seed=a.seed)

    start_step, state = 0, None
    ck = latest_checkpoint(a.ckpt_dir) if a.ckpt_dir else None
    if ck is not None:
        (full, _), extra = load_full(ck), load_extra(ck, 0)
        if pipeline:
            trainer.load_state_dict({"model": full, "optim": extra.get("pipeline_optim")})
        elif a.strategy == "tp":
            _load_tp(trainer.engine, full, extra)
        else:
            zero = trainer.ddp if trainer.strategy in ("zero2", "zero3") else None
            load_into_engine(trainer.engine, {k: v.to(dev) for k, v in full.items()}, extra, zero=zero)
            if trainer.ddp is not None and zero is None:
                trainer.engine.sync_shadow()
        start_step = int(extra.get("step", 0))
        state = StreamState.from_dict(extra["stream"]) if "stream" in extra else None
        trainer.step_num = start_step
    stream = ShardedStream(src, rank=s_rank, world_size=s_world, state=state, seed=a.seed, prefetch=4)
    batches = stream.batches(rows, pin=True)
    ckpt = AsyncCheckpointer()
    logf = open(a.log, "a") if a.log and rank == 0 else None
    loss_log = LOSSES if LOSSES is not None else None
    t0, tok0 = time.perf_counter(), 0
    step = start_step
    try:
        while step < a.steps:
            trainer.h2d_done.synchronize()  # the previous batch's buffers are free again
            x, y = next(batches)
            loss = trainer.step_async(x, y)
            step += 1
            tok0 += rows * a.seq * (1 if shared else world)
            stop = _STOP["flag"] or (a.stop_at > 0 and step >= a.stop_at)
            if world > 1 and step % 10 == 0:  # agree on a pre-emption signal every 10 steps
                flag = torch.tensor([1 if stop else 0], device=dev)
                dist.all_reduce(flag, op=dist.ReduceOp.MAX)
                stop = bool(flag.item())
            due = a.ckpt_dir and (step % a.ckpt_every == 0 or step == a.steps or stop)
            if due and pipeline:
                sd, popt = _pipeline_checkpoint(trainer, world) if world > 1 else (
                    trainer.state_dict()["model"], trainer.state_dict()["optim"])
                if rank == 0:
                    extra = {"step": step, "stream": stream.state_dict([stream.position]),
                             "pipeline_optim": popt, "optim_step": popt["step"]}
                    ckpt.save(Path(a.ckpt_dir) / f"step_{step}", sd, plan={}, rank=0, world_size=1, step=step,
                              global_shapes={k: list(v.shape) for k, v in sd.items()}, extra=extra)
                if world > 1:
                    dist.barrier()
            elif due and a.strategy == "tp":
                st = trainer.state_dict()          # collective: every rank gathers the shards
                if rank == 0:
                    extra = {"step": step, "stream": stream.state_dict([stream.position]),
                             "optim_step": st["optim_step"], "tp_exp_avg": st["exp_avg"],
                             "tp_exp_avg_sq": st["exp_avg_sq"]}
                    sd = st["model"]
                    ckpt.save(Path(a.ckpt_dir) / f"step_{step}", sd, plan={}, rank=0, world_size=1, step=step,
                              global_shapes={k: list(v.shape) for k, v in sd.items()}, extra=extra)
                if world > 1:
                    dist.barrier()
            elif due:
                pos = [stream.position]
                if world > 1 and not shared:
                    allp = [None] * world
                    dist.all_gather_object(allp, stream.position)
                    pos = allp
                zero = trainer.ddp if trainer.strategy in ("zero2", "zero3") else None
                if zero is not None:  # gathering the shards is a collective
                    sd, extra = engine_state_dict(trainer.engine, with_optimizer=True, zero=zero)
                if rank == 0:
                    if zero is None:
                        sd, extra = engine_state_dict(trainer.engine, with_optimizer=True)
                    extra.update(step=step, stream=stream.state_dict(pos))
                    ckpt.save(Path(a.ckpt_dir) / f"step_{step}", sd, plan={}, rank=0, world_size=1, step=step,
                              global_shapes={k: list(v.shape) for k, v in sd.items()}, extra=extra)
                if world > 1:
                    dist.barrier()
            log_due = step % 10 == 0 or step == a.steps
            if log_due or loss_log is not None:
                lv = loss.detach().reshape(1).clone()
                if pipeline and world > 1:
                    # the loss lives on the last stage: sum it there, mean over its CP ranks
                    dist.all_reduce(lv)
                    lv /= a.cp
                lv = float(lv.item())
                if logf and log_due:
                    dt = time.perf_counter() - t0
                    logf.write(json.dumps({"step": step, "loss": lv, "tokens_per_s": tok0 / dt}) + "\n")
                    logf.flush()
                if loss_log is not None:
                    loss_log.append(lv)
            if stop:
                break
        trainer.check()
    finally:
        ckpt.wait()
        if logf:
            logf.close()
        trainer.close()
        if world > 1 and not _external_group:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
