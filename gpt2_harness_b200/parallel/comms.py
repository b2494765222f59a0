"""Counted collectives, per-rank byte counters and the multi-process launcher.

Public API of the reference's ``parallel.comms`` (src/transformer_internals/
parallel/comms.py:106-569): ``CommCounter`` / ``counter_scope`` /
``get_counter``, counted wrappers over ``torch.distributed`` and
``spawn_workers``. The payload convention is the reference's, because the
closed-form byte checks depend on it:

* ``all_reduce``: the full buffer;
* ``all_gather``: the OUTPUT buffer;
* ``reduce_scatter``: the INPUT buffer;
* ``send``/``recv``/``broadcast``: the tensor.

``wire_bytes`` models what a ring moves per rank (2(p-1)/p S for all-reduce,
(p-1)/p S for gather/scatter/broadcast, S point to point).

The native peer-memory kernels of this framework count their payload on the
device; :func:`record_external` lets them report into the same counter, so a
fused path and the NCCL path produce identical ``summary()`` dictionaries.
"""

from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import queue as queue_mod
import tempfile
import time
import traceback
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any, Callable, Optional, Sequence

import torch
import torch.distributed as dist

__all__ = [
    "CollectiveRecord",
    "CommCounter",
    "SendHandle",
    "WorkerResult",
    "all_gather_into",
    "all_gather_list",
    "all_reduce",
    "barrier",
    "broadcast",
    "counter",
    "counter_scope",
    "get_counter",
    "isend",
    "record_external",
    "recv",
    "reduce_scatter_into",
    "send",
    "spawn_workers",
    "synchronize",
]


@dataclass
class CollectiveRecord:
    """Tally of one collective kind on one rank."""

    op: str
    calls: int = 0
    elements: int = 0
    payload_bytes: int = 0
    wire_bytes: float = 0.0

    def as_dict(self) -> dict[str, Any]:
        return {
            "calls": self.calls,
            "elements": self.elements,
            "payload_bytes": self.payload_bytes,
            "wire_bytes_ring_model": self.wire_bytes,
        }


def ring_wire_bytes(op: str, payload: int, world: int) -> float:
    """Per-rank bytes a ring implementation moves for `payload` (a model)."""
    p = max(int(world), 1)
    if p == 1:
        return 0.0
    if op == "all_reduce":
        return 2.0 * (p - 1) / p * payload
    if op in ("all_gather", "reduce_scatter", "broadcast"):
        return (p - 1) / p * payload
    return float(payload)


class CommCounter:
    """Exact per-rank collective volume (calls, elements, payload bytes)."""

    def __init__(self, world_size: int = 1) -> None:
        self.world_size = world_size
        self.records: dict[str, CollectiveRecord] = {}
        self.steps = 0

    def record(self, op: str, tensors) -> None:
        if isinstance(tensors, torch.Tensor):
            tensors = (tensors,)
        elements = sum(int(t.numel()) for t in tensors)
        payload = sum(int(t.numel()) * int(t.element_size()) for t in tensors)
        self.record_bytes(op, elements, payload)

    def record_bytes(self, op: str, elements: int, payload: int) -> None:
        """Tally one call of `op` moving `payload` bytes (`elements` elements)."""
        rec = self.records.setdefault(op, CollectiveRecord(op=op))
        rec.calls += 1
        rec.elements += elements
        rec.payload_bytes += payload
        rec.wire_bytes += ring_wire_bytes(op, payload, self.world_size)

    def reset(self) -> None:
        self.records.clear()
        self.steps = 0

    @property
    def total_payload_bytes(self) -> int:
        return sum(r.payload_bytes for r in self.records.values())

    @property
    def total_wire_bytes(self) -> float:
        return sum(r.wire_bytes for r in self.records.values())

    @property
    def total_calls(self) -> int:
        return sum(r.calls for r in self.records.values())

    def summary(self) -> dict[str, Any]:
        steps = max(self.steps, 1)
        return {
            "world_size": self.world_size,
            "steps": self.steps,
            "per_collective": {op: r.as_dict() for op, r in sorted(self.records.items())},
            "total_calls": self.total_calls,
            "total_payload_bytes": self.total_payload_bytes,
            "total_wire_bytes_ring_model": self.total_wire_bytes,
            "calls_per_step": self.total_calls / steps,
            "payload_bytes_per_step": self.total_payload_bytes / steps,
            "wire_bytes_per_step_ring_model": self.total_wire_bytes / steps,
        }


_ACTIVE = CommCounter()


def get_counter() -> CommCounter:
    return _ACTIVE


counter = get_counter


@contextmanager
def counter_scope(world_size: int):
    """Install a fresh counter for the block and yield it."""
    global _ACTIVE
    prev = _ACTIVE
    _ACTIVE = CommCounter(world_size=world_size)
    try:
        yield _ACTIVE
    finally:
        _ACTIVE = prev


def record_external(op: str, elements: int, payload_bytes: int) -> None:
    """Charge a collective executed outside torch.distributed (a native kernel)."""
    _ACTIVE.record_bytes(op, elements, payload_bytes)


# ----------------------------------------------------------------- wrappers --
def all_reduce(tensor: torch.Tensor, op: Any = None, group: Any = None) -> torch.Tensor:
    """In-place SUM (default) all-reduce, counted as the full buffer."""
    get_counter().record("all_reduce", tensor)
    dist.all_reduce(tensor, op=op or dist.ReduceOp.SUM, group=group)
    return tensor


def all_gather_into(output: torch.Tensor, tensor: torch.Tensor, group: Any = None) -> torch.Tensor:
    """Gather `tensor` from every rank into flat `output`; charged the output."""
    get_counter().record("all_gather", output)
    dist.all_gather_into_tensor(output, tensor.contiguous(), group=group)
    return output


def all_gather_list(tensor: torch.Tensor, world_size: int, group: Any = None) -> list[torch.Tensor]:
    """Gather into a list of per-rank tensors; charged the outputs."""
    out = [torch.empty_like(tensor) for _ in range(world_size)]
    get_counter().record("all_gather", out)
    dist.all_gather(out, tensor.contiguous(), group=group)
    return out


def reduce_scatter_into(output: torch.Tensor, tensor: torch.Tensor, op: Any = None,
                        group: Any = None) -> torch.Tensor:
    """Reduce-scatter `tensor` into this rank's shard `output`; charged the
    input. (gloo services this as all-reduce + slice.)"""
    get_counter().record("reduce_scatter", tensor)
    dist.reduce_scatter_tensor(output, tensor.contiguous(), op=op or dist.ReduceOp.SUM, group=group)
    return output


def broadcast(tensor: torch.Tensor, src: int = 0, group: Any = None) -> torch.Tensor:
    get_counter().record("broadcast", tensor)
    dist.broadcast(tensor, src=src, group=group)
    return tensor


def send(tensor: torch.Tensor, dst: int, tag: int = 0, group: Any = None) -> None:
    get_counter().record("send", tensor)
    dist.send(tensor.contiguous(), dst=dst, tag=tag, group=group)


def recv(tensor: torch.Tensor, src: int, tag: int = 0, group: Any = None) -> torch.Tensor:
    get_counter().record("recv", tensor)
    dist.recv(tensor, src=src, tag=tag, group=group)
    return tensor


class SendHandle:
    """Pending non-blocking send that keeps its buffer alive until waited:
    dropping the only reference while the transfer is in flight would let the
    allocator recycle the memory under it."""

    def __init__(self, work: Any, buffer: torch.Tensor) -> None:
        self._work = work
        self._buffer = buffer

    def wait(self) -> None:
        self._work.wait()
        self._buffer = None

    def is_completed(self) -> bool:
        return bool(self._work.is_completed())


def isend(tensor: torch.Tensor, dst: int, tag: int = 0, group: Any = None) -> SendHandle:
    get_counter().record("send", tensor)
    buf = tensor if tensor.is_contiguous() else tensor.contiguous()
    return SendHandle(dist.isend(buf, dst=dst, tag=tag, group=group), buf)


def _current_device() -> torch.device:
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def synchronize() -> None:
    """Wait for queued device work (no-op on CPU)."""
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()


def barrier(group: Any = None) -> None:
    """Process-group barrier, told its device on NCCL."""
    if dist.get_backend(group) == "nccl":
        dist.barrier(group=group, device_ids=[torch.cuda.current_device()])
    else:
        dist.barrier(group=group)


# ----------------------------------------------------------------- launcher --
@dataclass
class WorkerResult:
    """What one rank returns: the worker's value plus its counter summary."""

    rank: int
    value: Any
    payload: dict = field(default_factory=dict)
    backend: str = "gloo"
    device: str = "cpu"


def _entry(fn, rank, world, backend, init_file, timeout_s, device_kind, kwargs, out_q):
    try:
        torch.set_num_threads(1)
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
        device = "cpu"
        if device_kind == "cuda":
            torch.cuda.set_device(rank % max(torch.cuda.device_count(), 1))
            device = f"cuda:{torch.cuda.current_device()}"
        dist.init_process_group(
            backend=backend,
            init_method=f"file://{init_file}",
            rank=rank,
            world_size=world,
            timeout=datetime.timedelta(seconds=max(60, int(timeout_s))),
        )
        with counter_scope(world) as ctr:
            value = fn(rank, world, **kwargs)
            summary = ctr.summary()
        synchronize()
        out_q.put(("ok", rank, WorkerResult(rank, value, summary, backend, device)))
        dist.destroy_process_group()
    except BaseException:  # report and exit non-zero
        out_q.put(("error", rank, traceback.format_exc()))
        raise


def spawn_workers(fn: Callable, world_size: int, kwargs: Optional[dict] = None,
                  backend: Optional[str] = None, timeout: float = 300.0, caps=None,
                  allow_oversubscribe: bool = False) -> list[WorkerResult]:
    """Run ``fn(rank, world_size, **kwargs)`` in `world_size` fresh processes.

    The backend is chosen (or a request validated) from the machine's
    capabilities and the placement is checked in the parent, so an impossible
    placement fails before any process starts. One spawned process per rank,
    FileStore rendezvous, the device bound before ``init_process_group``.
    Fails fast: if any rank raises or dies without reporting, the others are
    terminated and RuntimeError carries the first traceback. ``fn`` must be
    importable (module-level).
    """
    from gpt2_harness_b200 import hardware

    kwargs = dict(kwargs or {})
    caps = caps if caps is not None else hardware.Capabilities.detect()
    backend = hardware.select_backend(caps, backend)
    hardware.check_placement(caps, world_size, backend, allow_oversubscribe)
    device = "cuda" if backend == "nccl" else "cpu"
    timeout_s = float(timeout)
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    tmpdir = tempfile.mkdtemp(prefix="g2b_rdzv_")
    init_file = os.path.join(tmpdir, "store")
    procs = []
    for r in range(world_size):
        p = ctx.Process(target=_entry, args=(fn, r, world_size, backend, init_file, timeout_s,
                                             device, kwargs, out_q), daemon=False)
        p.start()
        procs.append(p)
    results: dict[int, WorkerResult] = {}
    error: Optional[str] = None
    deadline = time.monotonic() + timeout_s
    try:
        while len(results) < world_size and error is None:
            try:
                kind, rank, payload = out_q.get(timeout=0.2)
                if kind == "ok":
                    results[rank] = payload
                else:
                    error = f"rank {rank} failed:\n{payload}"
            except queue_mod.Empty:
                dead = [i for i, p in enumerate(procs) if not p.is_alive() and p.exitcode not in (0, None)
                        and i not in results]
                if dead:
                    # give the queue a moment in case the report is in flight
                    try:
                        kind, rank, payload = out_q.get(timeout=1.0)
                        if kind == "ok":
                            results[rank] = payload
                            continue
                        error = f"rank {rank} failed:\n{payload}"
                    except queue_mod.Empty:
                        error = f"rank(s) {dead} exited with {[procs[i].exitcode for i in dead]} without reporting"
                if time.monotonic() > deadline:
                    error = f"timed out after {timeout_s}s waiting for ranks {sorted(set(range(world_size)) - set(results))}"
    finally:
        for p in procs:
            p.join(timeout=5 if error is None else 0.5)
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
    if error:
        raise RuntimeError(error)
    return [results[r] for r in range(world_size)]
