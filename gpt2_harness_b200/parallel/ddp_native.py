"""Data parallelism for the native engine, overlapped with backward.

Reference semantics (src/transformer_internals/parallel/data_parallel.py:
45-152): gradients are averaged with SUM all-reduces over 25 MiB buckets built
greedily in reverse parameter order, then divided by p; a bf16 wire casts each
bucket down before the reduction. Payload per rank per step is 4N bytes (2N on
a bf16 wire) in the reference's counting convention.

B200 design:

* The engine's flat fp32 gradient buffer IS a :class:`SymmetricBuffer`: every
  rank's buffer is mapped into every other rank, so no bucket is ever
  flattened or copied (reference :136-151 concatenates and copies back).
* The engine calls :meth:`NativeDDP.on_grads_ready` as soon as a block's
  gradients are final; every bucket whose last tensor is now final is
  launched on a dedicated communication stream, ordered after the compute
  stream by an event. Communication overlaps the rest of backward.
* ``comm="p2p"`` (default): one fused kernel per bucket
  (csrc/comm.cu ``allreduce_p2p``) performs reduce-scatter, the 1/p scale and
  all-gather over NVLink with in-kernel flags; ``comm="mc"``: the gradient
  buffer is also bound to an NVLink multicast object and one kernel per
  bucket (``allreduce_mc``) reads each element of its slice already summed by
  the NVSwitch (``multimem.ld_reduce``) and writes the scaled result to every
  rank with one ``multimem.st`` -- half the NVLink bytes of the P2P form and
  no reduction arithmetic on the SMs; ``comm="nccl"``: the bucket is a
  ``dist.all_reduce`` view of the flat buffer and the 1/p is folded into the
  AdamW kernel. All charge the same counter entries; the in-kernel counters
  charge each bucket's parameters (padding excluded), the reference's 4N.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.models.engine import ALIGN, ParamLayout
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.utils.nvtx import nvtx_range
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.symm import MulticastBuffer, SymmetricBuffer

__all__ = ["Bucket", "build_layout_buckets", "NativeDDP", "DEFAULT_BUCKET_BYTES"]

DEFAULT_BUCKET_BYTES = 25 * 1024 * 1024


@dataclass
class Bucket:
    lo: int          # first element (flat layout), 64-element aligned
    hi: int          # one past the last element including alignment padding
    numel: int       # parameter elements (no padding): the counted payload
    ready: int       # index of the gradient group that completes this bucket


def group_order(layout: ParamLayout) -> list[str]:
    L = layout.config.n_layer
    return ["root_head"] + [f"h.{i}" for i in reversed(range(L))] + ["root_tail"]


def _spec_group(spec) -> str:
    if spec.group != "root":
        return spec.group
    return "root_head" if spec.name.startswith("ln_f") else "root_tail"


def build_layout_buckets(layout: ParamLayout, bucket_bytes: int = DEFAULT_BUCKET_BYTES,
                         elem_bytes: int = 4) -> list[Bucket]:
    """Greedy buckets over the layout (= backward) order; a tensor larger than
    the cap gets a bucket of its own (reference data_parallel.py:64-95)."""
    order = {g: i for i, g in enumerate(group_order(layout))}
    buckets: list[Bucket] = []
    cur: list = []
    size = 0
    for s in layout.specs:
        nbytes = s.numel * elem_bytes
        if cur and size + nbytes > bucket_bytes:
            buckets.append(_mk(cur, order))
            cur, size = [], 0
        cur.append(s)
        size += nbytes
    if cur:
        buckets.append(_mk(cur, order))
    return buckets


def _mk(specs, order) -> Bucket:
    lo = specs[0].offset
    last = specs[-1]
    hi = last.offset + (last.numel + ALIGN - 1) // ALIGN * ALIGN
    return Bucket(lo, hi, sum(s.numel for s in specs), max(order[_spec_group(s)] for s in specs))


class NativeDDP:
    """Bucketed, backward-overlapped gradient averaging for :class:`Engine`.

    Construct it BEFORE the engine and pass :attr:`grad_buffer` to the engine
    (``Engine(..., grad_buffer=ddp.grad_buffer)``), then :meth:`attach`.
    """

    def __init__(self, layout: ParamLayout, group=None, comm: str = "p2p",
                 bucket_bytes: int = DEFAULT_BUCKET_BYTES, nblocks: int = 128,
                 device: Optional[torch.device] = None, tail_blocks: int = 128,
                 wait_budget_s: float = 30.0, reduce_dtype: str = "fp32") -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.comm = comm if self.world > 1 else "none"
        if self.comm not in ("p2p", "mc", "nccl", "none"):
            raise ValueError(f"unknown comm {comm!r}")
        self.layout = layout
        self.buckets = build_layout_buckets(layout, bucket_bytes)
        self.order = {g: i for i, g in enumerate(group_order(layout))}
        # Buckets completed during backward run with `nblocks` CTAs, those of
        # the last gradient group (nothing left to overlap) with
        # `tail_blocks`; both on the wide kernel (512 threads a CTA) unless
        # the slim one (128 threads, fits beside a resident GEMM) is chosen.
        self.nblocks = nblocks
        self.tail_blocks = tail_blocks
        # Measured on 2 B200s (GPT-2 124M, 16 x 1024 per GPU, same box): the
        # wide kernel for every bucket 21.49 ms / step, slim CTAs during
        # backward 21.87 ms -- sharing SMs with the GEMMs costs them more
        # than the SMs the wide CTAs hold for the short bucket reductions.
        # G2B_COMM_SLIM=1 selects the slim kernel for the overlapped buckets.
        self.slim = os.environ.get("G2B_COMM_SLIM", "0") == "1"
        self.last_group = len(self.order) - 1
        self.symm = None
        self.flags: Optional[SymmetricBuffer] = None
        if self.comm in ("p2p", "mc"):
            self.symm = (MulticastBuffer if self.comm == "mc" else SymmetricBuffer)(
                layout.total * 4, group, self.device)
            self.grad_buffer = self.symm.view(torch.float32, layout.total)
            words = N.lib().comm_flag_words()
            self.flags = SymmetricBuffer(words * 4, group, self.device)
        else:
            self.grad_buffer = torch.zeros(layout.total, dtype=torch.float32, device=self.device)
        # bf16 wire (reference data_parallel.py:136-151: cast the bucket down,
        # reduce, cast up): each bucket is cast into a bf16 copy that the
        # all-reduce works on (fp32 sums in the kernel) and cast back
        if reduce_dtype not in ("fp32", "bf16"):
            raise ValueError(f"reduce_dtype must be fp32 or bf16, not {reduce_dtype!r}")
        if reduce_dtype == "bf16" and self.comm == "mc":
            raise ValueError("the bf16 wire runs on the P2P or NCCL all-reduce")
        self.reduce_dtype = reduce_dtype
        self._wire16 = None
        self.grad16 = None
        if reduce_dtype == "bf16" and self.comm == "p2p":
            self._wire16 = SymmetricBuffer(layout.total * 2, group, self.device)
            self.grad16 = self._wire16.view(torch.bfloat16, layout.total)
        elif reduce_dtype == "bf16" and self.comm == "nccl":
            self.grad16 = torch.zeros(layout.total, dtype=torch.bfloat16, device=self.device)
        # The reduction kernels get a higher stream priority than the compute
        # stream: their CTAs are placed as soon as SMs free up, so each bucket
        # finishes (and hands its SMs back to the backward) as early as possible.
        prio = int(os.environ.get("G2B_COMM_PRIORITY", "-1"))
        self.stream = (torch.cuda.Stream(device=self.device, priority=prio)
                       if self.world > 1 else None)
        self.byte_counter = torch.zeros(1, dtype=torch.int64, device=self.device)
        # Handshake epochs: host-side, strictly increasing (eager steps), or
        # -- set before the first launch for a captured CUDA graph, whose
        # replays repeat their recorded arguments -- read by each launch from
        # a device counter in this rank's flag buffer (epoch argument 0).
        self.device_epochs = False
        self.epoch = 0
        # How long a bucket kernel waits for a peer before it records a
        # timeout and gives up (a rank held up by host work -- a checkpoint
        # write, a collection pause -- must not trip it)
        self.wait_budget_ns = int(wait_budget_s * 1e9)
        self._next = 0
        self.engine = None

    @property
    def grad_scale(self) -> float:
        """Multiplier the optimiser applies to gradients (1/p for NCCL SUM)."""
        return 1.0 / self.world if self.comm == "nccl" else 1.0

    def attach(self, engine) -> None:
        self.engine = engine
        engine.grad_ready_hook = self.on_grads_ready
        engine.grad_scale = self.grad_scale

    # ----------------------------------------------------------- hooks --
    def on_grads_ready(self, group: str) -> None:
        if self.comm == "none":
            return
        idx = self.order[group]
        last = idx == self.last_group
        while self._next < len(self.buckets) and self.buckets[self._next].ready <= idx:
            self._launch(self.buckets[self._next], slim=self.slim and not last, last=last)
            self._next += 1

    def _launch(self, b: Bucket, slim: bool = False, last: bool = False) -> None:
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        wire16 = self.grad16 is not None
        comms.record_external("all_reduce", b.numel, b.numel * (2 if wire16 else 4))
        with torch.cuda.stream(self.stream), nvtx_range(f"allreduce/bucket{self.buckets.index(b)}"):
            if wire16:
                N.cast_f32_bf16(self.grad_buffer[b.lo:b.hi], self.grad16[b.lo:b.hi])
            if self.device_epochs:
                epoch = 0
            else:
                self.epoch += 1
                epoch = self.epoch & 0xFFFFFFFF
            if self.comm == "mc":
                N.lib().allreduce_mc(self.symm.peer_ptrs_dev.data_ptr(), self.flags.peer_ptrs_dev.data_ptr(),
                                     self.symm.mc_ptr, self.rank, self.world, b.lo, b.hi - b.lo, 0,
                                     1.0 / self.world, epoch, self.byte_counter.data_ptr(),
                                     N.error_word().data_ptr(), self.tail_blocks if last else self.nblocks,
                                     self.wait_budget_ns, b.numel, self.stream.cuda_stream)
            elif self.comm == "p2p":
                fn = N.lib().allreduce_p2p_slim if slim else N.lib().allreduce_p2p
                bufs = self._wire16 if wire16 else self.symm
                fn(bufs.peer_ptrs_dev.data_ptr(), self.flags.peer_ptrs_dev.data_ptr(),
                   self.rank, self.world, b.lo, b.hi - b.lo, int(wire16), 1.0 / self.world,
                   epoch, self.byte_counter.data_ptr(), N.error_word().data_ptr(),
                   self.nblocks if slim else self.tail_blocks, self.wait_budget_ns, b.numel,
                   self.stream.cuda_stream)
            else:
                dist.all_reduce((self.grad16 if wire16 else self.grad_buffer)[b.lo:b.hi], group=self.group)
            if wire16:
                N.cast_bf16_f32(self.grad16[b.lo:b.hi], self.grad_buffer[b.lo:b.hi])

    def timeout_record(self) -> Optional[dict]:
        """Where this rank's first bucket handshake gave up (synchronises), or
        None: the phase (0 arrive, 1 done), CTA, peer, the epoch it waited for
        and the flag value it last saw."""
        if self.flags is None:
            return None
        words = N.lib().comm_flag_words()
        rec = [int(x) for x in self.flags.view(torch.int32, words)[words - 8:words - 1].cpu()]
        if not rec[0]:
            return None
        return {"phase": rec[1], "cta": rec[2], "peer": rec[3], "epoch": rec[4] & 0xFFFFFFFF,
                "flag_seen": rec[5] & 0xFFFFFFFF, "rank": rec[6]}

    def finish(self) -> None:
        """Make the compute stream wait for every launched bucket."""
        if self.comm == "none":
            return
        if self._next != len(self.buckets):
            # backward did not announce every group (e.g. a frozen tail):
            # launch the rest now so every rank issues the same sequence.
            while self._next < len(self.buckets):
                self._launch(self.buckets[self._next], last=True)
                self._next += 1
        torch.cuda.current_stream().wait_stream(self.stream)
        self._next = 0

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        if self.symm is not None:
            self.symm.close()
        if self.flags is not None:
            self.flags.close()
        if self._wire16 is not None:
            self._wire16.close()
