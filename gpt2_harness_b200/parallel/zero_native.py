"""ZeRO-2 for the native engine: reduce-scatter overlapped with backward, then
one fused kernel for the sharded global-norm clip, AdamW and the bf16
parameter all-gather, all over NVLink peer memory.

Reference semantics (src/transformer_internals/parallel/zero.py:241-486,
``ShardedAdamW`` at stage 2): gradients are reduce-scattered and divided by
p, every rank runs AdamW (torch single-tensor order, decay on matmul weights)
on the slice it owns, clipping uses the global norm of the averaged gradient
(one 4-byte all-reduce of the shard sums of squares), and the updated slices
are all-gathered in the parameter dtype.

B200 design:

* Slices follow the DDP gradient buckets (25 MiB, backward order): rank r
  owns slice r of every bucket, so each bucket is reduce-scattered as soon
  as backward has finished it, on a communication stream
  (csrc/zero.cu ``zero_rs_kernel``: P2P loads of the slice from every peer).
* After backward one kernel (``zero_adamw_ag_kernel``) exchanges the
  sums of squares, forms the clip coefficient, updates the fp32 master,
  exp_avg and exp_avg_sq shards, and writes the new bf16 values into every
  peer's parameter buffer. AdamW touches N/p elements per rank instead of N.
* fp32 master weights and both moments exist only as shards (3 x 4N/p bytes
  per rank); the full bf16 parameter buffer and the fp32 gradient buffer are
  symmetric (peer-mapped) so that the kernels can reach them.

Payload per rank per step, charged in the reference convention: reduce-scatter
of each bucket's fp32 input (4 x its aligned length), all-gather of the bf16
output (2 x the aligned layout length) and 4 bytes for the norm all-reduce:
4T + 2T + 4 bytes, T = the aligned flat length (``ParamLayout.total``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.models.engine import ALIGN, ParamLayout
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.ddp_native import DEFAULT_BUCKET_BYTES, build_layout_buckets, group_order
from gpt2_harness_b200.parallel.symm import SymmetricBuffer

__all__ = ["ShardPlan", "plan_shards", "NativeZeRO"]


@dataclass
class ShardPlan:
    """Slices of every bucket: rank r owns [lo + r*slice, min(hi, lo + (r+1)*slice))."""

    table: list          # [(lo, hi, slice, shard_offset)] per bucket
    shard_numel: int     # sum of slices: elements of every shard-sized buffer
    ready: list          # gradient-group index that completes each bucket

    def owned(self, rank: int) -> list[tuple[int, int, int]]:
        """(flat_start, count, shard_offset) of every slice owned by `rank`."""
        out = []
        for lo, hi, s, off in self.table:
            f0 = lo + rank * s
            n = max(0, min(hi, f0 + s) - f0)
            out.append((f0, n, off))
        return out


def plan_shards(layout: ParamLayout, world: int, bucket_bytes: int = DEFAULT_BUCKET_BYTES) -> ShardPlan:
    buckets = build_layout_buckets(layout, bucket_bytes)
    table, off = [], 0
    for b in buckets:
        span = b.hi - b.lo
        s = -(-span // world)
        s = -(-s // ALIGN) * ALIGN
        table.append((b.lo, b.hi, s, off))
        off += s
    return ShardPlan(table, off, [b.ready for b in buckets])


class NativeZeRO:
    """Sharded AdamW (ZeRO-2) for :class:`~gpt2_harness_b200.models.engine.Engine`.

    Construct it first, build the engine with ``grad_buffer=zero.grad_buffer,
    shadow_buffer=zero.shadow_buffer, optimizer_state=False``, then call
    :meth:`attach` (which shards the engine's master weights and frees the
    full-size copy). Call :meth:`finish` after ``engine.backward``.
    """

    def __init__(self, layout: ParamLayout, group=None, bucket_bytes: int = DEFAULT_BUCKET_BYTES,
                 device: Optional[torch.device] = None, rs_blocks: int = 148, opt_blocks: int = 148,
                 wait_budget_ns: int = 2_000_000_000) -> None:
        if not dist.is_initialized():
            raise RuntimeError("NativeZeRO needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        L = N.lib()
        if self.world > 8:
            raise ValueError("NativeZeRO supports up to 8 ranks (one NVSwitch domain)")
        self.layout = layout
        self.plan = plan_shards(layout, self.world, bucket_bytes)
        self.order = {g: i for i, g in enumerate(group_order(layout))}
        nb = len(self.plan.table)
        self.rs_blocks = rs_blocks
        self.opt_blocks = min(opt_blocks, L.zero_max_blocks())
        n = layout.total
        dev = self.device
        self._grad_symm = SymmetricBuffer(n * 4, group, dev)
        self._shadow_symm = SymmetricBuffer(n * 2, group, dev)
        self._flags = SymmetricBuffer(L.zero_flag_words() * 4, group, dev)
        self._norm = SymmetricBuffer(L.zero_norm_words() * 8, group, dev)
        self.grad_buffer = self._grad_symm.view(torch.float32, n)
        self.shadow_buffer = self._shadow_symm.view(torch.bfloat16, n)
        S = self.plan.shard_numel
        self.gsh = torch.zeros(S, dtype=torch.float32, device=dev)
        self.master = torch.zeros(S, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(S, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(S, dtype=torch.float32, device=dev)
        self.sumsq_parts = torch.zeros(nb * rs_blocks, dtype=torch.float32, device=dev)
        self.buckets_dev = torch.tensor([x for row in self.plan.table for x in row], dtype=torch.int64,
                                        device=dev)
        self.byte_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.epoch = 0
        self._next = 0
        self.engine = None
        self._args = {
            "peer_grad": self._grad_symm.peer_ptrs_dev.data_ptr(),
            "peer_shadow": self._shadow_symm.peer_ptrs_dev.data_ptr(),
            "peer_flags": self._flags.peer_ptrs_dev.data_ptr(),
            "peer_norm": self._norm.peer_ptrs_dev.data_ptr(),
            "rank": self.rank, "world": self.world,
            "buckets": self.buckets_dev.data_ptr(), "nb": nb, "bucket": 0,
            "rs_blocks": rs_blocks,
            "gsh": self.gsh.data_ptr(), "master": self.master.data_ptr(),
            "exp_avg": self.exp_avg.data_ptr(), "exp_avg_sq": self.exp_avg_sq.data_ptr(),
            "sumsq_parts": self.sumsq_parts.data_ptr(),
            "decay_ranges": 0, "nr": 0, "hp": 0, "max_norm": 0.0,
            "scale": 1.0 / self.world, "epoch": 0,
            "byte_counter": self.byte_counter.data_ptr(), "norm_out": self.grad_norm.data_ptr(),
            "err": N.error_word(dev).data_ptr(), "wait_budget_ns": int(wait_budget_ns),
        }

    # -------------------------------------------------------------- setup --
    def attach(self, engine) -> None:
        """Shard the engine's (identical on every rank) fp32 master weights,
        free the full copy and take over the optimiser step."""
        if engine.grad.data_ptr() != self.grad_buffer.data_ptr():
            raise ValueError("build the engine with grad_buffer=zero.grad_buffer")
        if engine.shadow.data_ptr() != self.shadow_buffer.data_ptr():
            raise ValueError("build the engine with shadow_buffer=zero.shadow_buffer")
        self.engine = engine
        with torch.no_grad():
            for f0, n, off in self.plan.owned(self.rank):
                if n:
                    self.master[off:off + n].copy_(engine.master[f0:f0 + n])
        engine.master = None  # the shards are the master weights from now on
        self.decay_ranges = engine.decay_ranges
        self._args["decay_ranges"] = self.decay_ranges.data_ptr()
        self._args["nr"] = self.decay_ranges.numel() // 2
        self._args["hp"] = engine.hp.data_ptr()
        self._args["max_norm"] = float(engine.optim.grad_clip or 0.0)
        engine.grad_ready_hook = self.on_grads_ready
        engine.grad_scale = 1.0  # the 1/p is applied in the reduce-scatter
        engine.optimizer_impl = self._optimizer_step
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    # ----------------------------------------------------------- backward --
    def on_grads_ready(self, group: str) -> None:
        idx = self.order[group]
        while self._next < len(self.plan.table) and self.plan.ready[self._next] <= idx:
            self._launch_rs(self._next)
            self._next += 1

    def _launch_rs(self, b: int) -> None:
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        lo, hi, _, _ = self.plan.table[b]
        comms.record_external("reduce_scatter", hi - lo, (hi - lo) * 4)
        self.epoch += 1
        a = self._args
        a["bucket"] = b
        a["epoch"] = self.epoch & 0xFFFFFFFF
        N.lib().zero_rs(a, self.stream.cuda_stream)

    def finish(self) -> None:
        """Launch any bucket backward did not announce and make the compute
        stream wait for every reduce-scatter."""
        while self._next < len(self.plan.table):
            self._launch_rs(self._next)
            self._next += 1
        torch.cuda.current_stream().wait_stream(self.stream)
        self._next = 0

    # ---------------------------------------------------------- optimiser --
    def _optimizer_step(self, hp: torch.Tensor) -> None:
        T = self.layout.total
        comms.record_external("all_gather", T, T * 2)
        if self._args["max_norm"] > 0:
            comms.record_external("all_reduce", 1, 4)
        self.epoch += 1
        a = self._args
        a["epoch"] = self.epoch & 0xFFFFFFFF
        a["hp"] = hp.data_ptr()
        N.lib().zero_adamw_ag(a, self.opt_blocks, torch.cuda.current_stream().cuda_stream)

    # ------------------------------------------------------------- state --
    def gather_full(self, shard: torch.Tensor) -> torch.Tensor:
        """Full flat vector (layout order) from every rank's shard of it.
        A collective: every rank calls it and receives the result."""
        S = self.plan.shard_numel
        parts = torch.empty(self.world * S, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(parts, shard.contiguous(), group=self.group)
        full = torch.zeros(self.layout.total, dtype=torch.float32, device=self.device)
        for r in range(self.world):
            base = r * S
            for f0, n, off in self.plan.owned(r):
                if n:
                    full[f0:f0 + n].copy_(parts[base + off: base + off + n])
        return full

    def full_master(self) -> torch.Tensor:
        """The full fp32 master vector (collective)."""
        return self.gather_full(self.master)

    def full_moments(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Full exp_avg and exp_avg_sq vectors (collective)."""
        return self.gather_full(self.exp_avg), self.gather_full(self.exp_avg_sq)

    @torch.no_grad()
    def load_full(self, master: torch.Tensor, exp_avg: Optional[torch.Tensor] = None,
                  exp_avg_sq: Optional[torch.Tensor] = None) -> None:
        """Take this rank's slices of full flat vectors (identical on every
        rank) and refresh the full bf16 parameter buffer from `master`."""
        for f0, n, off in self.plan.owned(self.rank):
            if not n:
                continue
            self.master[off:off + n].copy_(master[f0:f0 + n])
            if exp_avg is not None:
                self.exp_avg[off:off + n].copy_(exp_avg[f0:f0 + n])
            if exp_avg_sq is not None:
                self.exp_avg_sq[off:off + n].copy_(exp_avg_sq[f0:f0 + n])
        self.shadow_buffer.copy_(master[: self.layout.total])

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for b in (self._grad_symm, self._shadow_symm, self._flags, self._norm):
            b.close()
