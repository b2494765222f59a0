"""Resumable, elastic, sharded token streaming.

Reference semantics (src/transformer_internals/cluster/streaming.py:68-335):

* one global permutation per epoch derived from (seed, epoch) alone, so every
  rank computes it without communication and a restart rebuilds it exactly
  (same generator and seed mixing as the reference, so a stream position
  checkpointed by either framework resumes in the other);
* rank r reads the strided deal ``order[r::W]``;
* the checkpointed state is every rank's consumed count; an elastic resume
  at a different world size re-deals exactly the samples not yet consumed;
* a prefetch thread advances the position only when the consumer takes a
  sample, so a checkpoint never skips data that was read but not used.

B200 addition: :meth:`ShardedStream.batches` stacks samples into a reusable
pinned host buffer (``pin=True``) so the host->device copy of each step is an
asynchronous DMA from page-locked memory.
"""

from __future__ import annotations

import queue
import threading
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Iterator, Optional, Sequence

import numpy as np
import torch

__all__ = ["StreamState", "global_order", "plan_indices", "TokenShardSource", "ShardedStream",
           "DelayedSource", "measure_throughput"]


@dataclass
class StreamState:
    """Epoch, permutation seed and each rank's consumed count (checkpointable)."""

    num_samples: int
    seed: int = 0
    epoch: int = 0
    world_size: int = 1
    positions: list = field(default_factory=lambda: [0])
    shuffle: bool = True

    def to_dict(self) -> dict:
        return asdict(self)

    @staticmethod
    def from_dict(d: dict) -> "StreamState":
        return StreamState(int(d["num_samples"]), int(d["seed"]), int(d["epoch"]), int(d["world_size"]),
                           [int(x) for x in d["positions"]], bool(d.get("shuffle", True)))

    @property
    def consumed(self) -> int:
        return sum(self.positions)


def global_order(num_samples: int, seed: int, epoch: int, shuffle: bool) -> np.ndarray:
    """The job-wide sample order of one epoch (a function of seed and epoch)."""
    if not shuffle:
        return np.arange(num_samples, dtype=np.int64)
    return np.random.default_rng(seed * 1_000_003 + epoch).permutation(num_samples).astype(np.int64)


def plan_indices(state: StreamState, rank: int, world_size: int) -> np.ndarray:
    """Global indices rank `rank` of `world_size` reads next (fresh, same-world
    resume, or elastic resume at a different world size)."""
    order = global_order(state.num_samples, state.seed, state.epoch, state.shuffle)
    if state.consumed == 0:
        return order[rank::world_size]
    used = np.zeros(state.num_samples, dtype=bool)
    for r, pos in enumerate(state.positions):
        if pos:
            used[r:r + pos * state.world_size:state.world_size] = True
    return order[~used][rank::world_size]


class TokenShardSource:
    """Sample i = tokens[i*block : i*block + block + 1] of a flat token file
    (memory-mapped lazily per process)."""

    def __init__(self, path, block_size: int, dtype: str = "uint16") -> None:
        self.path = Path(path)
        self.block_size = block_size
        self.dtype = dtype
        self._map: Optional[np.memmap] = None
        total = self.path.stat().st_size // np.dtype(dtype).itemsize
        self.num_samples = max(0, (total - 1) // block_size)

    @staticmethod
    def write(path, tokens: np.ndarray, dtype: str = "uint16") -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        tokens.astype(dtype).tofile(path)
        return path

    def _mm(self) -> np.memmap:
        if self._map is None:
            self._map = np.memmap(self.path, dtype=self.dtype, mode="r")
        return self._map

    def __len__(self) -> int:
        return self.num_samples

    def window(self, i: int) -> np.ndarray:
        lo = i * self.block_size
        return np.asarray(self._mm()[lo:lo + self.block_size + 1], dtype=np.int64)

    def __getitem__(self, i: int):
        w = self.window(int(i))
        return torch.from_numpy(w[:-1].copy()), torch.from_numpy(w[1:].copy())


class ShardedStream:
    """Iterate this rank's shard with a checkpointable position."""

    def __init__(self, source: Sequence[Any], *, rank: int, world_size: int,
                 state: Optional[StreamState] = None, seed: int = 0, shuffle: bool = True,
                 prefetch: int = 0) -> None:
        self.source, self.rank, self.world_size, self.prefetch = source, rank, world_size, prefetch
        self.state = state or StreamState(len(source), seed, 0, world_size, [0] * world_size, shuffle)
        if len(source) != self.state.num_samples:
            raise ValueError(f"source has {len(source)} samples but the checkpointed stream state "
                             f"describes {self.state.num_samples}; the corpus changed under the checkpoint")
        self._plan = plan_indices(self.state, rank, world_size)
        self.consumed_here = 0
        self._base = self.state.positions[rank] if world_size == self.state.world_size else 0

    @property
    def plan(self) -> np.ndarray:
        return self._plan

    @property
    def position(self) -> int:
        return self._base + self.consumed_here

    def state_dict(self, all_positions: Optional[list] = None) -> dict:
        """Checkpoint contribution; pass every rank's position (gathered by the
        caller) for an elastic-resumable state."""
        pos = list(all_positions) if all_positions else list(self.state.positions)
        if not all_positions:
            pos = pos + [0] * (self.world_size - len(pos))
            pos[self.rank] = self.position
        return StreamState(self.state.num_samples, self.state.seed, self.state.epoch, self.world_size,
                           pos, self.state.shuffle).to_dict()

    def __iter__(self) -> Iterator[Any]:
        if self.prefetch <= 0:
            for idx in self._plan:
                item = self.source[int(idx)]
                self.consumed_here += 1
                yield item
            return
        q: queue.Queue = queue.Queue(maxsize=self.prefetch)
        stop = threading.Event()

        def reader() -> None:
            for idx in self._plan:
                if stop.is_set():
                    break
                q.put(self.source[int(idx)])
            q.put(_END)

        th = threading.Thread(target=reader, name=f"prefetch-{self.rank}", daemon=True)
        th.start()
        try:
            while True:
                item = q.get()
                if item is _END:
                    return
                self.consumed_here += 1
                yield item
        finally:
            stop.set()
            while th.is_alive():
                try:
                    q.get_nowait()
                except queue.Empty:
                    time.sleep(0.001)
            th.join()

    def batches(self, batch_size: int, pin: bool = True, drop_last: bool = True):
        """Yield (idx, targets) int64 batches [B, T] assembled in reusable
        (pinned) host buffers; the position advances per consumed sample."""
        bufs = None
        cur = []
        for x, y in self:
            cur.append((x, y))
            if len(cur) == batch_size:
                if bufs is None:
                    T = x.shape[0]
                    bufs = [torch.empty(batch_size, T, dtype=torch.int64, pin_memory=pin and torch.cuda.is_available())
                            for _ in range(2)]
                torch.stack([a for a, _ in cur], out=bufs[0])
                torch.stack([b for _, b in cur], out=bufs[1])
                yield bufs[0], bufs[1]
                cur = []
        if cur and not drop_last:
            yield torch.stack([a for a, _ in cur]), torch.stack([b for _, b in cur])


_END = object()


class DelayedSource:
    """A source with a fixed per-read delay (stands in for slow storage; the
    sleep releases the GIL so prefetch can overlap it)."""

    def __init__(self, source: Sequence[Any], delay_s: float) -> None:
        self.source, self.delay_s = source, delay_s

    def __len__(self) -> int:
        return len(self.source)

    def __getitem__(self, i: int):
        time.sleep(self.delay_s)
        return self.source[i]


def measure_throughput(source: Sequence[Any], n: int, prefetch: int, work_s: float = 0.0) -> float:
    """Samples/s of consuming `n` samples with `work_s` of consumer work each."""
    stream = ShardedStream(source, rank=0, world_size=1, prefetch=prefetch, shuffle=False)
    t0 = time.perf_counter()
    for i, _ in enumerate(stream):
        if work_s:
            time.sleep(work_s)
        if i + 1 >= n:
            break
    return n / (time.perf_counter() - t0)
