"""Failure detection and checkpoint/restart recovery for multi-process jobs.

Reference semantics (src/transformer_internals/cluster/failure.py:80-479): a
real multi-process DDP job (one OS process per rank, env rendezvous over
127.0.0.1); a rank can crash itself (``os._exit(137)`` at ``crash_step``) or
be SIGKILLed by the supervisor once the log shows a given step; on the first
non-zero exit the supervisor kills the survivors and relaunches with
``resume=True`` from the last checkpoint (model, optimizer, stream position);
the resumed losses must equal an uninterrupted run's exactly.

Added: hung-rank detection. Every rank appends a heartbeat (step, time) each
step; the supervisor's watchdog declares the job hung when a live rank's
heartbeat is older than ``heartbeat_timeout_s``, kills every rank and
recovers like a crash. Ranks also run with a short process-group timeout, so a
rank blocked on a dead peer fails on its own. Injection is host-side only
(``hang_step``/``hang_rank`` make a rank sleep): no GPU fault is ever caused.

Run a worker:  ``python -m gpt2_harness_b200.cluster.failure`` (reads the job
spec path from ``G2B_JOB_SPEC``).
"""

from __future__ import annotations

import contextlib
import datetime
import json
import os
import socket
import subprocess
import sys
import time
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path
from typing import Any, Iterator, Optional

import numpy as np
import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

from gpt2_harness_b200.cluster.checkpoint import REPLICATE, load_extra, load_full, save_sharded
from gpt2_harness_b200.cluster.streaming import ShardedStream, StreamState, TokenShardSource
from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.gpt import GPT

__all__ = ["JobSpec", "RunReport", "free_port", "reserved_port", "port_is_free", "read_log",
           "worker_main", "launch", "run_with_recovery", "make_corpus"]


def free_port() -> int:
    with reserved_port() as p:
        return p


@contextlib.contextmanager
def reserved_port() -> Iterator[int]:
    """A loopback port held bound (unavailable to others) until exit."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        s.listen(1)
        yield int(s.getsockname()[1])


def port_is_free(port: int) -> bool:
    try:
        with socket.socket() as s:
            s.bind(("127.0.0.1", port))
    except OSError:
        return False
    return True


@dataclass
class JobSpec:
    """What the supervisor and every rank agree on."""

    data_path: str
    ckpt_dir: str
    log_path: str
    block_size: int = 32
    micro_batch: int = 4
    steps: int = 20
    lr: float = 3e-4
    seed: int = 1234
    ckpt_every: int = 5
    master_port: int = 0
    crash_step: Optional[int] = None
    crash_rank: int = 1
    hang_step: Optional[int] = None
    hang_rank: int = 1
    heartbeat_timeout_s: float = 0.0   # 0 = watchdog off
    pg_timeout_s: float = 60.0
    resume: bool = False
    n_layer: int = 2
    n_head: int = 2
    n_embd: int = 32
    vocab_size: int = 128

    def to_dict(self) -> dict:
        return asdict(self)

    def model_config(self) -> GPTConfig:
        return GPTConfig(vocab_size=self.vocab_size, n_positions=self.block_size, n_layer=self.n_layer,
                         n_head=self.n_head, n_embd=self.n_embd, dropout=0.0)


@dataclass
class RunReport:
    launches: int = 0
    crashed_at: Optional[float] = None
    recovered_at: Optional[float] = None
    resumed_from_step: Optional[int] = None
    time_to_recover_s: Optional[float] = None
    hung_detected: bool = False
    events: list = field(default_factory=list)


def _log(path: str, record: dict) -> None:
    with Path(path).open("a") as fh:
        fh.write(json.dumps(record) + "\n")
        fh.flush()
        os.fsync(fh.fileno())


def read_log(path) -> list[dict]:
    p = Path(path)
    if not p.exists():
        return []
    return [json.loads(l) for l in p.read_text().splitlines() if l.strip()]


def _heartbeat_path(spec: JobSpec, rank: int) -> Path:
    return Path(spec.ckpt_dir).parent / f"heartbeat_{spec.master_port}_{rank}.json"


def worker_main(rank: int, world_size: int, spec_dict: dict) -> None:
    spec = JobSpec(**spec_dict)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(spec.master_port)
    dist.init_process_group("gloo", rank=rank, world_size=world_size,
                            timeout=datetime.timedelta(seconds=spec.pg_timeout_s))
    try:
        _train(rank, world_size, spec)
    finally:
        with contextlib.suppress(Exception):
            dist.destroy_process_group()


def _train(rank: int, world: int, spec: JobSpec) -> None:
    torch.manual_seed(spec.seed)
    model = GPT(spec.model_config())
    source = TokenShardSource(spec.data_path, spec.block_size)
    start = 0
    stream_state: Optional[StreamState] = None
    optim_state = None
    ck = Path(spec.ckpt_dir)
    if spec.resume and (ck / "index.json").exists():
        state, index = load_full(ck)
        model.load_state_dict(state)
        extra = load_extra(ck, 0)
        start = index.step
        optim_state = extra["optimizer"]
        stream_state = StreamState.from_dict(extra["stream"])
    ddp = DDP(model)
    opt = torch.optim.AdamW(model.parameters(), lr=spec.lr, betas=(0.9, 0.95), weight_decay=0.0)
    if optim_state is not None:
        opt.load_state_dict(optim_state)
    if stream_state is None:
        stream_state = StreamState(len(source), spec.seed, 0, world, [0] * world, True)
    stream = ShardedStream(source, rank=rank, world_size=world, state=stream_state, prefetch=2)
    it = iter(stream)
    hb = _heartbeat_path(spec, rank)
    step = start
    for step in range(start + 1, spec.steps + 1):
        hb.write_text(json.dumps({"rank": rank, "step": step, "t": time.time()}))
        if spec.crash_step is not None and step == spec.crash_step and rank == spec.crash_rank:
            _log(spec.log_path, {"event": "crash", "rank": rank, "step": step, "t": time.time()})
            os._exit(137)
        if spec.hang_step is not None and step == spec.hang_step and rank == spec.hang_rank:
            _log(spec.log_path, {"event": "hang", "rank": rank, "step": step, "t": time.time()})
            time.sleep(3600)  # host-side hang: the watchdog must notice and kill it
        items = [next(it) for _ in range(spec.micro_batch)]
        x = torch.stack([a for a, _ in items])
        y = torch.stack([b for _, b in items])
        loss = ddp(x, targets=y)["loss"]
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        red = loss.detach().clone()
        dist.all_reduce(red)
        red /= world
        if rank == 0:
            _log(spec.log_path, {"event": "step", "step": step, "loss": float(red), "resumed_from": start,
                                 "t": time.time()})
        if step % spec.ckpt_every == 0:
            _checkpoint(rank, world, spec, model, opt, stream, step)
    if rank == 0:
        _log(spec.log_path, {"event": "done", "step": step, "t": time.time()})


def _checkpoint(rank, world, spec, model, opt, stream, step) -> None:
    """All-gather the stream positions (also the consistent cut), rank 0 writes."""
    pos = torch.tensor([stream.position], dtype=torch.long)
    got = [torch.zeros_like(pos) for _ in range(world)]
    dist.all_gather(got, pos)
    positions = [int(t.item()) for t in got]
    if rank == 0:
        state = {k: v.detach().cpu() for k, v in model.state_dict().items()}
        save_sharded(spec.ckpt_dir, state, dict.fromkeys(state, REPLICATE), rank=0, world_size=1, step=step,
                     global_shapes={k: list(v.shape) for k, v in state.items()},
                     extra={"optimizer": opt.state_dict(), "stream": stream.state_dict(positions)},
                     meta={"world_size": world, "wrote_at": time.time()})
    dist.barrier()


def _rank_env(rank: int, world: int, spec: JobSpec, spec_path: Path) -> dict:
    env = dict(os.environ)
    env.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(spec.master_port), "RANK": str(rank),
                "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world), "G2B_JOB_SPEC": str(spec_path),
                "OMP_NUM_THREADS": "1", "MKL_NUM_THREADS": "1", "CUDA_VISIBLE_DEVICES": ""})
    return env


def _usable_port(spec: JobSpec, attempts: int = 8) -> JobSpec:
    """Re-test the rendezvous port just before the spawn; replace it if taken."""
    if spec.master_port and port_is_free(spec.master_port):
        return spec
    for _ in range(attempts):
        p = free_port()
        if port_is_free(p):
            return replace(spec, master_port=p)
    raise OSError(f"no free loopback port after {attempts} attempts")


def _reached_step(log_path: str, step: int) -> bool:
    return any(r.get("event") == "step" and r.get("step", 0) >= step for r in read_log(log_path))


def _stale_rank(spec: JobSpec, world: int, now: float) -> Optional[int]:
    if spec.heartbeat_timeout_s <= 0:
        return None
    for r in range(world):
        p = _heartbeat_path(spec, r)
        try:
            hb = json.loads(p.read_text())
        except (OSError, ValueError):
            continue
        if now - float(hb["t"]) > spec.heartbeat_timeout_s:
            return r
    return None


def launch(world_size: int, spec: JobSpec, *, kill_rank_at_step: Optional[tuple] = None,
           timeout_s: float = 300.0) -> tuple:
    """Start one OS process per rank and supervise: optional external SIGKILL
    of (rank, at step), fail-fast on the first non-zero exit, watchdog on
    heartbeats. Returns (all_clean, exit_codes, kill_time, hung_rank)."""
    spec = _usable_port(spec)
    spec_path = Path(spec.ckpt_dir).parent / f"jobspec_{spec.master_port}.json"
    spec_path.parent.mkdir(parents=True, exist_ok=True)
    spec_path.write_text(json.dumps(spec.to_dict()))
    for r in range(world_size):
        with contextlib.suppress(OSError):
            _heartbeat_path(spec, r).unlink()
    procs = [subprocess.Popen([sys.executable, "-m", "gpt2_harness_b200.cluster.failure"],
                              env=_rank_env(r, world_size, spec, spec_path)) for r in range(world_size)]
    kill_time = None
    hung = None
    deadline = time.time() + timeout_s
    try:
        while time.time() < deadline:
            if kill_rank_at_step is not None and kill_time is None:
                victim, at = kill_rank_at_step
                if _reached_step(spec.log_path, at):
                    with contextlib.suppress(ProcessLookupError):
                        os.kill(procs[victim].pid, 9)
                    kill_time = time.time()
                    _log(spec.log_path, {"event": "killed", "rank": victim, "t": kill_time})
            codes = [p.poll() for p in procs]
            if any(c is not None and c != 0 for c in codes):
                break
            if all(c == 0 for c in codes):
                return True, codes, kill_time, None
            stale = _stale_rank(spec, world_size, time.time())
            if stale is not None and procs[stale].poll() is None:
                hung = stale
                _log(spec.log_path, {"event": "hung", "rank": stale, "t": time.time()})
                break
            time.sleep(0.002)
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
        for p in procs:
            with contextlib.suppress(Exception):
                p.wait(timeout=10)
    return False, [p.returncode for p in procs], kill_time, hung


def run_with_recovery(world_size: int, spec: JobSpec, *, kill_rank_at_step: Optional[tuple] = None,
                      max_restarts: int = 3, timeout_s: float = 300.0) -> RunReport:
    """Run, and on a crash / kill / hang relaunch from the last checkpoint."""
    rep = RunReport()
    cur = spec
    kill = kill_rank_at_step
    while rep.launches <= max_restarts:
        rep.launches += 1
        clean, codes, ktime, hung = launch(world_size, cur, kill_rank_at_step=kill, timeout_s=timeout_s)
        rep.events.append({"launch": rep.launches, "clean": clean, "codes": codes, "hung": hung})
        if clean:
            break
        t_fail = ktime or time.time()
        rep.crashed_at = rep.crashed_at or t_fail
        rep.hung_detected = rep.hung_detected or hung is not None
        idx = Path(cur.ckpt_dir) / "index.json"
        rep.resumed_from_step = json.loads(idx.read_text())["step"] if idx.exists() else 0
        cur = replace(cur, resume=True, crash_step=None, hang_step=None, master_port=0)
        kill = None
    steps_after = [r for r in read_log(spec.log_path)
                   if r.get("event") == "step" and rep.crashed_at and r["t"] > rep.crashed_at]
    if steps_after:
        rep.recovered_at = steps_after[0]["t"]
        rep.time_to_recover_s = rep.recovered_at - rep.crashed_at
    return rep


def make_corpus(path, n_tokens: int = 20_000, vocab: int = 128, seed: int = 0) -> Path:
    rng = np.random.default_rng(seed)
    return TokenShardSource.write(path, rng.integers(0, vocab, size=n_tokens))


def _main() -> None:
    spec = json.loads(Path(os.environ["G2B_JOB_SPEC"]).read_text())
    worker_main(int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), spec)


if __name__ == "__main__":
    _main()
