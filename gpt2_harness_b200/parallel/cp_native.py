"""Context parallelism (all-gather-KV form) on the native engine.

Reference semantics: src/transformer_internals/parallel/sequence_parallel.py
:60-132 (``all_gather_kv_attention``: every rank holds a contiguous shard of
the sequence, all-gathers K and V along the sequence, attends causally at
absolute positions ``rank * T_local``; backward reduce-scatters dK and dV; the
weight gradients are all-reduced over the group).

B200 design:

* Each rank runs the engine on its T/p tokens of every sequence, with
  positions offset by ``rank * T/p`` (learned position embeddings read at the
  absolute position).
* Attention of layer l: ``cp_kv_gather`` (csrc/tp.cu) copies this rank's k/v
  rows into its block of a per-layer symmetric [B, T, 2C] key/value buffer and
  pulls the blocks of the EARLIER ranks by P2P loads -- a causal query of rank
  r never sees later keys, so rank r moves r/p of the sequence, not all of it.
  The tcgen05 attention then runs with ``q_offset = r*T/p`` over the first
  (r+1)*T/p keys of that buffer.
* Backward: the attention backward writes dK/dV of every key it saw into a
  symmetric partial buffer; ``cp_kv_reduce`` sums this rank's key block over
  the ranks whose queries saw it (r..p-1, in rank order) straight into the
  k/v columns of the local dqkv, which the c_attn backward then consumes.
* Weight gradients: the data-parallel machinery over the same group
  (:class:`~gpt2_harness_b200.parallel.ddp_native.NativeDDP`: bucketed P2P
  all-reduce overlapped with backward, mean over ranks) -- with equal token
  counts per rank the mean of the per-rank mean losses is the global mean.

Load balancing (``balance="zigzag"``, the default): under the contiguous
split rank p-1 attends to p times the keys of rank 0 (causal work grows with
the position), so the step waits for the last rank. The zig-zag split cuts
every sequence into 2p chunks of T/(2p) tokens and gives rank r chunks r and
2p-1-r, stored as the two halves of its local sequence (positions read from
two offsets by the embedding). Every rank then attends over the same area:
half 1 (queries of chunk r) over keys [0, (r+1)T/2p), half 2 (chunk 2p-1-r)
over [0, (2p-r)T/2p) -- two attention calls on strided half views. The K/V
buffer keeps the natural order; the gather pulls every chunk up to 2p-1-r
from its owner, and the reduce sums each own chunk over the two halves'
dK/dV partials of every rank that saw it.

Streaming form (``kv="stream"``): no gathered copy. ``cp_kv_publish``
(csrc/tp.cu) copies this rank's k/v rows, in local order, into its own compact
per-layer symmetric buffer ([B, T/p, 2C]: a p-th of the gathered one) and
stores an epoch into word ``rank`` of every peer's publish buffer (system-scope
release after the rows are fenced). The tensor-core attention kernels
(``N.attention_fwd_peers`` / ``N.attention_bwd_peers``) then take one TMA map
per owner over that owner's buffer: before its first load from rank q a
producer waits (bounded) for rank q's word to reach the epoch, and every
64-key block is loaded straight from its owner's memory over NVLink (plain
tile loads, no cluster multicast), overlapped with the MMAs of the blocks
already in shared memory. The backward reads the same buffers under the
epoch the forward published; the dK/dV partials and their reduction are the
gathered form's. A buffer is rewritten one step later, after the
data-parallel gradient reduction of the same group, which no rank passes
while a peer's backward may still read it.

Payload per rank per layer in the reference convention: the gather is charged
its output (2 x B x T x C x 2 bytes: K and V, bf16), the reduce-scatter its
input (the same), as for ``_GatherSequence``; the streaming form is charged
the same (the reference convention counts the logical collective).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.symm import SymmetricBuffer
from gpt2_harness_b200.utils.nvtx import nvtx_range

__all__ = ["NativeCP"]


class NativeCP:
    """Sequence sharding of attention for :class:`~gpt2_harness_b200.models.engine.Engine`.

    Build it with the full sequence length ``T`` and batch ``B``; the engine
    then runs on ``B x T/p`` tokens per rank (this rank's shard of every
    sequence). Call :meth:`attach` on the engine.

    ``layers`` (default all) names the absolute layer indices whose gathered
    K/V are kept (a pipeline stage's blocks); ``slots`` keeps that many
    independent sets, one per micro-batch in flight: the backward of a
    micro-batch reads the K/V its forward gathered, after the forwards of
    later micro-batches. :attr:`slot` selects the set.
    """

    def __init__(self, config: GPTConfig, B: int, T: int, group=None,
                 device: Optional[torch.device] = None, nblocks: int = 128,
                 layers: Optional[list] = None, slots: int = 1, balance: str = "zigzag",
                 kv: str = "gather") -> None:
        if not dist.is_initialized():
            raise RuntimeError("NativeCP needs an initialised process group")
        if config.kv_heads != config.n_head:
            raise ValueError("NativeCP gathers 2C-wide key/value rows: multi-head attention only")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("NativeCP supports up to 8 ranks (one NVSwitch domain)")
        if T % self.world:
            raise ValueError("the sequence length must split evenly over the group")
        self.device = dev = device or torch.device("cuda", torch.cuda.current_device())
        self.config = config
        self.B, self.T = B, T
        self.Tl = T // self.world
        if balance not in ("zigzag", "contiguous"):
            raise ValueError(f"unknown balance {balance!r}")
        self.zigzag = balance == "zigzag"
        self.balance = balance
        if kv not in ("gather", "stream"):
            raise ValueError(f"unknown kv mode {kv!r} (gather or stream)")
        self.stream = kv == "stream"
        self.kv_mode = kv
        if self.stream and not self.zigzag and self.Tl % 128:
            raise ValueError(f"streamed keys need T / p a multiple of 128, got {self.Tl}")
        if self.zigzag:
            h = self.Tl // 2
            if self.Tl % 2 or h % 128:
                raise ValueError(f"zig-zag needs T / (2p) a multiple of 128, got {self.Tl / 2}")
            self.h = h
            # local sequence = [chunk r ; chunk 2p-1-r]
            self.chunks = (self.rank, 2 * self.world - 1 - self.rank)
            self.pos0, self.pos_split, self.pos1 = self.rank * h, h, self.chunks[1] * h
        else:
            self.pos0, self.pos_split, self.pos1 = self.rank * self.Tl, None, 0
        C, L = config.n_embd, config.n_layer
        self.C = C
        self.nblocks = nblocks
        bf = torch.bfloat16
        rows = B * T
        layers = list(range(L)) if layers is None else list(layers)
        self.layer_index = {l: i for i, l in enumerate(layers)}
        nl = len(layers) * slots
        self.slots = slots
        self.slot = 0
        # per-layer k/v: the gathered sequence, or (streaming) this rank's rows only
        kv_rows = B * self.Tl if self.stream else rows
        self._kv_rows = kv_rows
        self._kv = SymmetricBuffer(nl * kv_rows * 2 * C * 2, group, dev)
        self._dkv = SymmetricBuffer(rows * 2 * C * 2, group, dev)         # dk/dv partials (reused)
        # zig-zag: the second half's queries write their own partials
        self._dkv2 = SymmetricBuffer(rows * 2 * C * 2, group, dev) if self.zigzag else None
        self._flags = SymmetricBuffer(N.lib().tp_flag_words() * 4, group, dev)
        kv = self._kv.view(bf, nl * kv_rows * 2 * C).view(nl, kv_rows, 2 * C)
        self.kv = [kv[i] for i in range(nl)]
        self.dkv = self._dkv.view(bf, rows * 2 * C).view(rows, 2 * C)
        self.dkv2 = self._dkv2.view(bf, rows * 2 * C).view(rows, 2 * C) if self.zigzag else None
        self._kv_ptrs = [torch.tensor([p + i * kv_rows * 2 * C * 2 for p in self._kv.peer_ptrs],
                                      dtype=torch.int64, device=dev) for i in range(nl)]
        self._pub = None
        if self.stream:
            # word q: the last epoch rank q published; then the publish
            # kernel's finished-CTA counter. Starts at zero on every rank.
            self._pub = SymmetricBuffer(N.lib().kv_publish_words() * 4, group, dev)
            self._pub.view(torch.int32).zero_()
            dist.barrier(group=group)
            self.pub_counter = 0
            self.pub_epoch = [0] * nl
        self.byte_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self.epoch = 0

    def attach(self, engine) -> None:
        """Route the engine's (or a pipeline stage engine's) attention here."""
        engine.pos0, engine.pos_split, engine.pos1 = self.pos0, self.pos_split, self.pos1
        engine.attn_fwd_hook = self.attention_fwd
        engine.attn_bwd_hook = self.attention_bwd
        if hasattr(engine, "slot_hook"):
            engine.slot_hook = self.set_slot

    def set_slot(self, slot: int) -> None:
        if not 0 <= slot < self.slots:
            raise ValueError(f"slot {slot} out of range ({self.slots} kept)")
        self.slot = slot

    def local_tokens(self, t: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Copy this rank's tokens of the full [B, T] batch ``t`` into ``out``
        ([B, T/p], any device): its slice, or under zig-zag its two chunks."""
        if not self.zigzag:
            a = self.rank * self.Tl
            src = t[:, a:a + self.Tl]
            if src.device.type == "cpu" and not src.is_contiguous():
                src = src.contiguous()
            return out.copy_(src, non_blocking=True)
        h = self.h
        for half, k in enumerate(self.chunks):
            out[:, half * h:(half + 1) * h].copy_(t[:, k * h:(k + 1) * h], non_blocking=True)
        return out

    def _kv_index(self, l: int) -> int:
        return self.slot * len(self.layer_index) + self.layer_index[l]

    def _args(self, ptrs: int, **kw) -> dict:
        self.epoch += 1
        d = {"peer_bufs": ptrs, "peer_flags": self._flags.peer_ptrs_dev.data_ptr(), "rank": self.rank,
             "world": self.world, "nblocks": self.nblocks, "epoch": self.epoch & 0xFFFFFFFF,
             "err": N.error_word(self.device).data_ptr(), "byte_counter": self.byte_counter.data_ptr(),
             "cols": 2 * self.C, "B": self.B, "Tl": self.Tl}
        d.update(kw)
        return d

    def _peers(self, i: int, epoch: int) -> dict:
        """Owner buffers of layer-slot i for the streaming attention calls."""
        C = self.C
        off = i * self._kv_rows * 2 * C * 2
        return {"bases": [p + off for p in self._kv.peer_ptrs], "sb": self.Tl * 2 * C, "st": 2 * C,
                "v_off": C, "Tl": self.Tl, "zigzag": int(self.zigzag), "flags": self._pub.ptr,
                "epoch": epoch}

    def _publish(self, i: int, qkv) -> int:
        self.pub_counter += 1
        ep = self.pub_counter & 0xFFFFFFFF
        d = {"peer_bufs": self._kv_ptrs[i].data_ptr(), "peer_flags": self._pub.peer_ptrs_dev.data_ptr(),
             "rank": self.rank, "world": self.world, "nblocks": self.nblocks, "epoch": ep,
             "err": N.error_word(self.device).data_ptr(), "byte_counter": self.byte_counter.data_ptr(),
             "cols": 2 * self.C, "B": self.B, "Tl": self.Tl, "src": qkv.data_ptr(),
             "src_ld": qkv.stride(0), "zigzag": int(self.zigzag)}
        with nvtx_range(f"cp/publish/{i}"):
            N.lib().cp_kv_publish(d, torch.cuda.current_stream(self.device).cuda_stream)
        self.pub_epoch[i] = ep
        return ep

    # ------------------------------------------------------------ hooks --
    def attention_fwd(self, l: int, qkv, y, lse, B: int, H: int, Tl: int) -> None:
        C, T = self.C, self.T
        i = self._kv_index(l)
        if self.stream:
            comms.record_external("all_gather", B * T * 2 * C, B * T * 2 * C * 2)
            peers = self._peers(i, self._publish(i, qkv))
            if not self.zigzag:
                N.attention_fwd_peers(qkv[:, :C], y, lse, B, H, Tl, (self.rank + 1) * self.Tl, self.pos0,
                                      peers)
                return
            h = self.h
            lse2 = lse.view(-1)[: 2 * B * H * h].view(2, B, H, h)
            for half, k in enumerate(self.chunks):
                N.attention_fwd_peers(qkv[half * h:, :C], y[half * h:], lse2[half], B, H, h, (k + 1) * h,
                                      k * h, peers, q_rows=Tl)
            return
        kv = self.kv[i]
        nbytes = B * T * 2 * C * 2
        comms.record_external("all_gather", B * T * 2 * C, nbytes)
        d = self._args(self._kv_ptrs[i].data_ptr(), src=qkv.data_ptr(), src_ld=qkv.stride(0),
                       zigzag=int(self.zigzag))
        with nvtx_range(f"cp/gather/{i}"):
            N.lib().cp_kv_gather(d, torch.cuda.current_stream(self.device).cuda_stream)
        if not self.zigzag:
            Tk = (self.rank + 1) * self.Tl
            N.attention_fwd(qkv[:, :C], kv[:, :C], kv[:, C:], y, lse, B, H, Tl, Tk=Tk,
                            q_offset=self.pos0, kv_rows=T)
            return
        h = self.h
        lse2 = lse.view(-1)[: 2 * B * H * h].view(2, B, H, h)
        for half, k in enumerate(self.chunks):
            N.attention_fwd(qkv[half * h:, :C], kv[:, :C], kv[:, C:], y[half * h:], lse2[half],
                            B, H, h, Tk=(k + 1) * h, q_offset=k * h, kv_rows=T, q_rows=Tl)

    def attention_bwd(self, l: int, qkv, y, dy, dqkv, lse, delta, B: int, H: int, Tl: int) -> None:
        C, T = self.C, self.T
        i = self._kv_index(l)
        kv, dkv = self.kv[i], self.dkv
        if self.stream:
            peers = self._peers(i, self.pub_epoch[i])
            if not self.zigzag:
                N.attention_bwd_peers(qkv[:, :C], y, dy, dqkv[:, :C], dkv[:, :C], dkv[:, C:], lse, delta, B, H,
                                      Tl, (self.rank + 1) * self.Tl, self.pos0, peers, kv_rows=T)
                extra = {}
            else:
                h = self.h
                lse2 = lse.view(-1)[: 2 * B * H * h].view(2, B, H, h)
                delta2 = delta.view(-1)[: 2 * B * H * h].view(2, B, H, h)
                for half, (k, part) in enumerate(zip(self.chunks, (self.dkv, self.dkv2))):
                    N.attention_bwd_peers(qkv[half * h:, :C], y[half * h:], dy[half * h:], dqkv[half * h:, :C],
                                          part[:, :C], part[:, C:], lse2[half], delta2[half], B, H, h,
                                          (k + 1) * h, k * h, peers, kv_rows=T, q_rows=Tl)
                extra = {"zigzag": 1, "peer_bufs2": self._dkv2.peer_ptrs_dev.data_ptr()}
            self._reduce(B, T, C, dqkv, extra)
            return
        if not self.zigzag:
            Tk = (self.rank + 1) * self.Tl
            N.attention_bwd(qkv[:, :C], kv[:, :C], kv[:, C:], y, dy, dqkv[:, :C], dkv[:, :C],
                            dkv[:, C:], lse, delta, B, H, Tl, Tk=Tk, q_offset=self.pos0, kv_rows=T)
            extra = {}
        else:
            h = self.h
            lse2 = lse.view(-1)[: 2 * B * H * h].view(2, B, H, h)
            delta2 = delta.view(-1)[: 2 * B * H * h].view(2, B, H, h)
            for half, (k, part) in enumerate(zip(self.chunks, (self.dkv, self.dkv2))):
                N.attention_bwd(qkv[half * h:, :C], kv[:, :C], kv[:, C:], y[half * h:], dy[half * h:],
                                dqkv[half * h:, :C], part[:, :C], part[:, C:], lse2[half], delta2[half],
                                B, H, h, Tk=(k + 1) * h, q_offset=k * h, kv_rows=T, q_rows=Tl)
            extra = {"zigzag": 1, "peer_bufs2": self._dkv2.peer_ptrs_dev.data_ptr()}
        self._reduce(B, T, C, dqkv, extra)

    def _reduce(self, B: int, T: int, C: int, dqkv, extra: dict) -> None:
        nbytes = B * T * 2 * C * 2
        comms.record_external("reduce_scatter", B * T * 2 * C, nbytes)
        d = self._args(self._dkv.peer_ptrs_dev.data_ptr(), out_bf16=dqkv.data_ptr(), src_ld=dqkv.stride(0),
                       **extra)
        with nvtx_range("cp/reduce_scatter"):
            N.lib().cp_kv_reduce(d, torch.cuda.current_stream(self.device).cuda_stream)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for b in (self._kv, self._dkv, self._dkv2, self._flags, self._pub):
            if b is not None:
                b.close()
