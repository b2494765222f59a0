"""ZeRO-3 for the native engine: every transformer block's parameters are
sharded across ranks, gathered over NVLink just before the block runs
(prefetched one block ahead on a communication stream), and its gradients are
reduce-scattered straight out of a peer-mapped buffer as soon as its backward
finishes.

Reference semantics (src/transformer_internals/parallel/zero.py:494-860,
``Zero3Model`` + ``Zero3AdamW``): one flat unit per block, sharded p ways;
forward all-gathers the unit (param dtype), runs it and frees it; backward
all-gathers it again, backpropagates and reduce-scatters the gradient
(reduce dtype), dividing by p; the root (wte, wpe, ln_f) is replicated and
all-reduced per tensor; clipping sums the shard squares with one 4-byte
all-reduce and adds the replicated root's squares after it.

B200 design:

* Units follow the engine's flat layout: unit l is the contiguous range of
  block l's twelve tensors. Rank r owns slice r (64-element aligned) and
  keeps the fp32 master, both AdamW moments and the bf16 copy of that slice
  only. The bf16 shards are symmetric (peer-mapped) memory.
* A step uses the units in the order fwd 0..L-1, bwd L-1..0. Use k gathers
  into buffer k%2 (csrc/zero.cu ``zero_ag_kernel``: P2P loads of each rank's
  slice); the gather of use k+1 is launched when use k begins, on a
  communication stream, after an event that marks use k-1's kernels done.
  The compute stream waits only on the event of the gather it needs.
* Backward writes block l's full gradient into one of two peer-mapped fp32
  buffers; ``zero_rs_kernel`` (with a closing handshake) reduces this rank's
  slice from every peer's buffer into the local gradient shard while the next
  block's backward runs; the buffer is rewritten two blocks later, after that
  reduce-scatter is known complete on every rank.
* Root gradients are averaged with the fused peer-memory all-reduce kernel.
  The optimiser: shard sum of squares -> 4-byte all-reduce (NCCL) -> + root
  squares -> clip -> AdamW on the shard (bf16 written into the local shard)
  and on the replicated root.
* Activations are kept (no recompute): B200 memory holds them at the
  benchmark shapes, so the MFU numerator counts the model FLOPs actually run.
* Nothing full-size stays resident: the engine is built on
  :attr:`storage_layout` (only the root tensors in its fp32 master, bf16 copy
  and fp32 gradient), block parameters exist as bf16 shards plus the two
  gather buffers, block gradients as two max-unit fp32 buffers plus the fp32
  shard. At GPT-2 medium on 8 ranks that leaves ~0.2 GB of root tensors where
  the full-size bf16 copy and fp32 gradient took 2.1 GB.

Payload per rank per step in the reference convention (all-gather = output,
reduce-scatter = input): sum over units of (2 + 2 + e) x span_u bytes for the
two bf16 gathers and the reduce-scatter, e x N_root for the root all-reduces
and 4 bytes for the norm, with e = 4 (fp32 wire, the default) or 2
(``reduce_dtype="bf16"``: the block and root gradients are cast to bf16
copies that the peers read, the sums stay fp32; at GPT-2 medium on 8 ranks
that is the reference's bf16-everywhere 1,918,883,840 B plus the norm).
span_u is the unit's 64-aligned length.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.models.engine import ALIGN, CompactLayout, ParamLayout, init_flat_weights
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.symm import SymmetricBuffer
from gpt2_harness_b200.utils.nvtx import nvtx_range

__all__ = ["NativeZeRO3", "unit_plan"]


def _align(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


def unit_plan(layout: ParamLayout, world: int) -> list[dict]:
    """Per block: flat range, span, slice size and shard offset."""
    L = layout.config.n_layer
    out, off = [], 0
    for l in range(L):
        lo, hi = layout.group_range(f"h.{l}")
        span = hi - lo
        s = _align(-(-span // world))
        out.append({"lo": lo, "hi": hi, "span": span, "slice": s, "off": off})
        off += s
    return out


class NativeZeRO3:
    """Block-parameter sharding for :class:`~gpt2_harness_b200.models.engine.Engine`.

    Build the engine with ``grad_buffer=z.grad_buffer, optimizer_state=False``
    and call :meth:`attach`; call :meth:`finish` after ``engine.backward``.
    """

    def __init__(self, layout: ParamLayout, group=None, device: Optional[torch.device] = None,
                 nblocks: int = 148, wait_budget_ns: int = 2_000_000_000,
                 reduce_dtype: str = "fp32") -> None:
        if not dist.is_initialized():
            raise RuntimeError("NativeZeRO3 needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("NativeZeRO3 supports up to 8 ranks (one NVSwitch domain)")
        self.device = dev = device or torch.device("cuda", torch.cuda.current_device())
        L = N.lib()
        self.layout = layout
        self.L = layout.config.n_layer
        self.units = unit_plan(layout, self.world)
        self.shard_numel = sum(u["slice"] for u in self.units)
        self.max_span = max(u["span"] for u in self.units)
        self.nblocks = nblocks
        # The engine's flat buffers hold the root tensors only (ln_f, then
        # wte and wpe), packed: root_ranges are [0, a) = ln_f (no decay) and
        # [a, n_root) = wte, wpe (decay) in that packed storage.
        self.storage_layout = CompactLayout(layout, lambda s: s.group == "root")
        sto = self.storage_layout
        a = sto.by_name["wte.weight"].offset
        self.root_ranges = [(0, a), (a, sto.total)]
        # symmetric memory
        self._grad_full = SymmetricBuffer(sto.total * 4, group, dev)        # root grads live here
        self._gbuf = SymmetricBuffer(2 * self.max_span * 4, group, dev)     # block grads, 2 slots
        # bf16 reduce wire (reference param_dtype/reduce_dtype, zero.py:594-631):
        # the block gradient and the root gradients are cast to bf16 copies
        # that the peers read; sums stay fp32
        if reduce_dtype not in ("fp32", "bf16"):
            raise ValueError(f"reduce_dtype must be fp32 or bf16, not {reduce_dtype!r}")
        self.reduce_dtype = reduce_dtype
        self._re = 2 if reduce_dtype == "bf16" else 4  # wire bytes per reduced element
        self._gbuf16 = self._root16 = None
        if reduce_dtype == "bf16":
            self._gbuf16 = SymmetricBuffer(2 * self.max_span * 2, group, dev)
            self._root16 = SymmetricBuffer(sto.total * 2, group, dev)
        self._pshard = SymmetricBuffer(self.shard_numel * 2, group, dev)    # bf16 shards
        self._flags = SymmetricBuffer(L.zero_flag_words() * 4, group, dev)
        self._ar_flags = SymmetricBuffer(L.comm_flag_words() * 4, group, dev)
        self.grad_buffer = self._grad_full.view(torch.float32, sto.total)
        self.gbuf = self._gbuf.view(torch.float32, 2 * self.max_span)
        self.gbuf16 = self._gbuf16.view(torch.bfloat16, 2 * self.max_span) if self._gbuf16 else None
        self.root16 = self._root16.view(torch.bfloat16, sto.total) if self._root16 else None
        self.pshard = self._pshard.view(torch.bfloat16, self.shard_numel)
        self.gather = torch.zeros(2, self.max_span, dtype=torch.bfloat16, device=dev)
        S = self.shard_numel
        self.gsh = torch.zeros(S, dtype=torch.float32, device=dev)
        self.master = torch.zeros(S, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(S, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(S, dtype=torch.float32, device=dev)
        nroot = sum(b - a for a, b in self.root_ranges)
        self.root_master = torch.zeros(nroot, dtype=torch.float32, device=dev)
        self.root_m = torch.zeros(nroot, dtype=torch.float32, device=dev)
        self.root_v = torch.zeros(nroot, dtype=torch.float32, device=dev)
        self.root_numel = sum(s.numel for s in layout.specs if s.group == "root")
        # reduce-scatter table: unit l's gradient sits in gbuf slot (L-1-l) % 2
        rows = []
        for l, u in enumerate(self.units):
            base = ((self.L - 1 - l) % 2) * self.max_span
            rows += [base, base + u["span"], u["slice"], u["off"]]
        self.rs_table = torch.tensor(rows, dtype=torch.int64, device=dev)
        self.shard_decay = self._shard_decay_ranges()
        self.byte_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self.sumsq = torch.zeros(4, dtype=torch.float32, device=dev)
        self._norm_ws = torch.empty(1024, dtype=torch.float32, device=dev)
        self.clip = torch.ones(1, dtype=torch.float32, device=dev)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.epoch = 0
        self.uses = [("fwd", l) for l in range(self.L)] + [("bwd", l) for l in reversed(range(self.L))]
        self._use_index = {u: k for k, u in enumerate(self.uses)}
        self._gathered: dict[int, torch.cuda.Event] = {}
        self._rs_done: dict[int, torch.cuda.Event] = {}
        self._cur_unit = -1
        self._cur_slot = 0
        self._names = {}
        for s in layout.specs:
            if s.group != "root":
                l = int(s.group.split(".")[1])
                self._names[s.name] = (l, s.offset - self.units[l]["lo"], s.numel, s.shape)
        self.engine = None
        self._args = {
            "peer_grad": self._gbuf.peer_ptrs_dev.data_ptr(), "peer_shadow": 0,
            "peer_flags": self._flags.peer_ptrs_dev.data_ptr(), "peer_norm": 0,
            "rank": self.rank, "world": self.world, "buckets": self.rs_table.data_ptr(),
            "nb": self.L, "bucket": 0, "rs_blocks": nblocks, "gsh": self.gsh.data_ptr(),
            "master": 0, "exp_avg": 0, "exp_avg_sq": 0, "sumsq_parts": 0, "decay_ranges": 0,
            "nr": 0, "hp": 0, "max_norm": 0.0, "scale": 1.0 / self.world, "epoch": 0,
            "byte_counter": self.byte_counter.data_ptr(), "norm_out": 0,
            "err": N.error_word(dev).data_ptr(), "wait_budget_ns": int(wait_budget_ns),
            "done_handshake": 1, "peer_shard": self._pshard.peer_ptrs_dev.data_ptr(),
            "gather_dst": 0, "ag_span": 0, "ag_slice": 0, "ag_offset": 0,
            "peer_grad16": self._gbuf16.peer_ptrs_dev.data_ptr() if self._gbuf16 else 0,
        }
        self.ar_epoch = 0

    def _shard_decay_ranges(self) -> torch.Tensor:
        """Weight-decay ranges of this rank's shard, in shard coordinates."""
        out = []
        for l, u in enumerate(self.units):
            f0 = u["lo"] + self.rank * u["slice"]
            f1 = min(u["hi"], f0 + u["slice"])
            for s in self.layout.specs:
                if s.group != f"h.{l}" or not s.decay:
                    continue
                a, b = max(f0, s.offset), min(f1, s.offset + _align(s.numel))
                if a < b:
                    lo, hi = u["off"] + a - f0, u["off"] + b - f0
                    if out and out[-1] == lo:
                        out[-1] = hi
                    else:
                        out += [lo, hi]
        if not out:
            out = [0, 0]
        return torch.tensor(out, dtype=torch.int64, device=self.device)

    # -------------------------------------------------------------- setup --
    def attach(self, engine, full_master: Optional[torch.Tensor] = None) -> None:
        """Take over `engine` (built with ``grad_buffer=z.grad_buffer`` and
        ``storage=z.storage_layout``). Block shards come from `full_master`
        (a full fp32 vector in layout order, identical on every rank) or, by
        default, from the engine's init seed (the same values its full-layout
        init gives); the root from the engine's own buffers."""
        if engine.grad.data_ptr() != self.grad_buffer.data_ptr():
            raise ValueError("build the engine with grad_buffer=z.grad_buffer")
        if engine.storage is not self.storage_layout:
            raise ValueError("build the engine with storage=z.storage_layout")
        self.engine = engine
        with torch.no_grad():
            full = full_master
            if full is None:
                full = torch.empty(self.layout.total, dtype=torch.float32, device=self.device)
                init_flat_weights(self.layout, full, engine.init_seed or 0)
            for u in self.units:
                f0 = u["lo"] + self.rank * u["slice"]
                n = max(0, min(u["hi"], f0 + u["slice"]) - f0)
                if n:
                    self.master[u["off"]:u["off"] + n].copy_(full[f0:f0 + n])
            del full
            self.pshard.copy_(self.master)
            self.root_master.copy_(engine.master[:self.storage_layout.total])
        engine.master = None
        engine.param_source = self._param
        engine.grad_source = self._grad
        engine.block_hook = self._block_hook
        engine.fuse_bias_grad_into_ln = False
        engine.grad_ready_hook = self._grads_ready
        engine.optimizer_impl = self._optimizer_step
        engine.grad_scale = 1.0
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    # ------------------------------------------------------ engine sources --
    def _param(self, name: str) -> Optional[torch.Tensor]:
        e = self._names.get(name)
        if e is None:
            return None
        l, off, n, shape = e
        if l != self._cur_unit:
            raise RuntimeError(f"parameter {name} requested while unit {self._cur_unit} is gathered")
        return self.gather[self._cur_slot, off:off + n].view(shape)

    def _grad(self, name: str) -> Optional[torch.Tensor]:
        e = self._names.get(name)
        if e is None:
            return None
        l, off, n, shape = e
        base = ((self.L - 1 - l) % 2) * self.max_span
        return self.gbuf[base + off: base + off + n].view(shape)

    # ------------------------------------------------------------ gathers --
    def _launch_gather(self, k: int, after: torch.cuda.Event) -> None:
        _, l = self.uses[k]
        u = self.units[l]
        self.stream.wait_event(after)
        comms.record_external("all_gather", u["span"], u["span"] * 2)
        self.epoch += 1
        a = self._args
        a["epoch"] = self.epoch & 0xFFFFFFFF
        a["gather_dst"] = self.gather[k % 2].data_ptr()
        a["ag_span"], a["ag_slice"], a["ag_offset"] = u["span"], u["slice"], u["off"]
        with nvtx_range(f"zero3/gather/h.{l}"):
            N.lib().zero_ag(a, self.nblocks, self.stream.cuda_stream)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self._gathered[k] = ev

    def _block_hook(self, phase: str, l: int) -> None:
        k = self._use_index[(phase, l)]
        mark = torch.cuda.Event()
        mark.record()  # every kernel of use k-1 (and before) has been issued
        if k == 0:
            self._gathered.clear()
            self._launch_gather(0, mark)
        if k + 1 < len(self.uses):
            self._launch_gather(k + 1, mark)
        if phase == "bwd":
            m = self.L - 1 - l
            if m >= 2:  # gradient slot m % 2 was last reduce-scattered for use m-2
                torch.cuda.current_stream().wait_event(self._rs_done[m - 2])
        torch.cuda.current_stream().wait_event(self._gathered.pop(k))
        self._cur_unit, self._cur_slot = l, k % 2

    # ---------------------------------------------------- reduce-scatters --
    def _grads_ready(self, group: str) -> None:
        if not group.startswith("h."):
            return
        l = int(group.split(".")[1])
        u = self.units[l]
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        comms.record_external("reduce_scatter", u["span"], u["span"] * self._re)
        self.epoch += 1
        a = self._args
        a["epoch"] = self.epoch & 0xFFFFFFFF
        a["bucket"] = l
        with torch.cuda.stream(self.stream), nvtx_range(f"zero3/reduce_scatter/h.{l}"):
            if self.gbuf16 is not None:
                base = ((self.L - 1 - l) % 2) * self.max_span
                N.cast_f32_bf16(self.gbuf[base:base + u["span"]], self.gbuf16[base:base + u["span"]])
            N.lib().zero_rs(a, self.stream.cuda_stream)
        done = torch.cuda.Event()
        done.record(self.stream)
        self._rs_done[self.L - 1 - l] = done

    def finish(self) -> None:
        """After backward: average the replicated root gradients (fused P2P
        all-reduce, per tensor in the reference's accounting) and make the
        compute stream wait for all communication."""
        ev = torch.cuda.Event()
        ev.record()
        self.stream.wait_event(ev)
        for s in self.layout.specs:
            if s.group == "root":
                comms.record_external("all_reduce", s.numel, s.numel * self._re)
        bf16 = self.root16 is not None
        with torch.cuda.stream(self.stream):
            if bf16:
                N.cast_f32_bf16(self.grad_buffer, self.root16)
            buf = self._root16 if bf16 else self._grad_full
            for a, b in self.root_ranges:
                self.ar_epoch += 1
                count = sum(s.numel for s in self.layout.specs
                            if s.group == "root" and a <= s.offset < b)
                N.lib().allreduce_p2p(
                    buf.peer_ptrs_dev.data_ptr(), self._ar_flags.peer_ptrs_dev.data_ptr(),
                    self.rank, self.world, a, b - a, int(bf16), 1.0 / self.world,
                    self.ar_epoch & 0xFFFFFFFF, self.byte_counter.data_ptr(),
                    N.error_word(self.device).data_ptr(), self.nblocks, self._args["wait_budget_ns"],
                    count, self.stream.cuda_stream)
            if bf16:
                N.cast_bf16_f32(self.root16, self.grad_buffer)
        torch.cuda.current_stream().wait_stream(self.stream)
        self._rs_done.clear()
        self._cur_unit = -1

    # ---------------------------------------------------------- optimiser --
    def _optimizer_step(self, hp: torch.Tensor) -> None:
        eng = self.engine
        o = eng.optim
        clip = None
        if o.grad_clip and o.grad_clip > 0:
            N.grad_sumsq(self.gsh, self._norm_ws, self.sumsq[0:1])
            comms.record_external("all_reduce", 1, 4)
            dist.all_reduce(self.sumsq[0:1], group=self.group)
            for i, (a, b) in enumerate(self.root_ranges):
                N.grad_sumsq(self.grad_buffer[a:b], self._norm_ws, self.sumsq[1 + i:2 + i])
            total = self.sumsq[:3].sum(0, keepdim=True)
            N.clip_coef(total, o.grad_clip, self.clip, self.grad_norm)
            clip = self.clip
        N.adamw_step(self.master, self.gsh, self.exp_avg, self.exp_avg_sq, self.pshard, 0, hp, clip,
                     decay_ranges=self.shard_decay)
        off = 0
        for i, (a, b) in enumerate(self.root_ranges):
            n = b - a
            # ln_f (first range) has no decay; wte and wpe (second) both decay
            N.adamw_step(self.root_master[off:off + n], self.grad_buffer[a:b], self.root_m[off:off + n],
                         self.root_v[off:off + n], eng.shadow[a:b], 0 if i == 0 else n, hp, clip)
            off += n

    # ------------------------------------------------------------- state --
    def _full(self, shard: torch.Tensor, root: torch.Tensor) -> torch.Tensor:
        S = self.shard_numel
        parts = torch.empty(self.world * S, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(parts, shard.contiguous(), group=self.group)
        full = torch.zeros(self.layout.total, dtype=torch.float32, device=self.device)
        for r in range(self.world):
            for u in self.units:
                f0 = u["lo"] + r * u["slice"]
                n = max(0, min(u["hi"], f0 + u["slice"]) - f0)
                if n:
                    full[f0:f0 + n].copy_(parts[r * S + u["off"]: r * S + u["off"] + n])
        self.storage_layout.scatter_to_full(root, full)
        return full

    def full_master(self) -> torch.Tensor:
        """Full fp32 master vector in layout order (collective)."""
        return self._full(self.master, self.root_master)

    def full_moments(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Full exp_avg and exp_avg_sq vectors in layout order (collective)."""
        return self._full(self.exp_avg, self.root_m), self._full(self.exp_avg_sq, self.root_v)

    @torch.no_grad()
    def load_full(self, master: torch.Tensor, exp_avg: Optional[torch.Tensor] = None,
                  exp_avg_sq: Optional[torch.Tensor] = None) -> None:
        """Take this rank's shards (and the replicated root) of full vectors
        that are identical on every rank; refresh the bf16 copies."""
        for u in self.units:
            f0 = u["lo"] + self.rank * u["slice"]
            n = max(0, min(u["hi"], f0 + u["slice"]) - f0)
            if not n:
                continue
            sl = slice(u["off"], u["off"] + n)
            self.master[sl].copy_(master[f0:f0 + n])
            if exp_avg is not None:
                self.exp_avg[sl].copy_(exp_avg[f0:f0 + n])
                self.exp_avg_sq[sl].copy_(exp_avg_sq[f0:f0 + n])
        self.pshard.copy_(self.master)
        sto = self.storage_layout
        sto.gather_from_full(master, self.root_master)
        if exp_avg is not None:
            sto.gather_from_full(exp_avg, self.root_m)
            sto.gather_from_full(exp_avg_sq, self.root_v)
        self.engine.shadow.copy_(self.root_master)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for b in (self._grad_full, self._gbuf, self._pshard, self._flags, self._ar_flags,
                  self._gbuf16, self._root16):
            if b is None:
                continue
            b.close()
