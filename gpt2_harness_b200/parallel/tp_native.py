"""Tensor parallelism with sequence parallelism on the native engine kernels.

Reference semantics: src/transformer_internals/parallel/tensor_parallel.py
(``ColumnParallelLinear`` c_attn/c_fc, ``RowParallelLinear`` c_proj/mlp
c_proj with the bias added once after the reduction, c_attn sliced per q/k/v
section so every rank owns whole heads, replicated LayerNorms) plus what the
reference only models: Megatron sequence parallelism (the residual stream and
the LayerNorms run on this rank's token rows; an all-gather enters each
column-parallel GEMM and a reduce-scatter leaves each row-parallel one) and a
vocabulary-parallel tied embedding / lm_head / cross-entropy over the padded
vocabulary (``padded_vocab``).

B200 design (kernels in csrc/tp.cu, GEMM/attention/LN from the engine):

* Heads are split unevenly when the head count does not divide: rank r gets
  ``H // p`` heads plus one for the first ``H % p`` ranks (GPT-2 XL's 25 heads
  on 8 ranks: 4, 3, 3, 3, 3, 3, 3, 3). The MLP's 4C columns split evenly.
* Every [M, C] activation that crosses ranks lives in a symmetric buffer with
  each rank's token rows at the same offset: the all-gather pulls peers' row
  blocks by P2P loads, the reduce-scatter sums this rank's block of every
  peer's bf16 partial in fp32 and adds the bias and the fp32 residual in the
  same kernel. The LayerNorm outputs gathered for the forward stay resident
  (one buffer per LayerNorm) and are reused by the weight-gradient GEMMs.
* Embedding: each rank looks up the wte rows of its own tokens straight from
  the shard of the rank that owns each token id (P2P loads); backward adds the
  gradient rows into the owner's shard with P2P atomics.
* Cross-entropy: each rank reduces its logit slice to per-row (max, sum exp,
  target logit); one kernel combines every rank's statistics (P2P loads) into
  the loss and overwrites the local slice with softmax - onehot.
* Replicated parameters (LayerNorms, row-parallel biases, wpe, ln_f) sit in
  one contiguous region at the start of the local layout; their per-rank partial
  gradients are summed by the fused peer-memory all-reduce. Clipping sums the
  sharded region's squares across ranks (one 4-byte all-reduce) and adds the
  replicated region once.

Per block and step every rank moves 4 all-gathers and 4 reduce-scatters of
M x C bf16 (forward 2 + 2, backward 2 + 2): in the reference convention
(all-gather = output, reduce-scatter = input) 8 x 2 x M x C bytes, twice the
4 all-reduces of the reference's parity mode with the same ring wire bytes.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.engine import ALIGN, OptimConfig, ParamLayout, choose_splits, init_flat_weights
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.symm import SymmetricBuffer
from gpt2_harness_b200.parallel.tensor_parallel import padded_vocab
from gpt2_harness_b200.utils.nvtx import nvtx_range

__all__ = ["head_partition", "TPLayout", "TPEngine"]

D = 64  # head dim


def _align(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


def head_partition(n_head: int, world: int) -> list[tuple[int, int]]:
    """[h0, h1) of every rank: H // p heads each, one more for the first H % p."""
    base, extra = divmod(n_head, world)
    out, h = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((h, h + n))
        h += n
    return out


class TPLayout:
    """This rank's flat parameter layout: the replicated tensors (one
    contiguous region [0, repl_hi), all-reduced as one), the wte shard, then
    the block shards."""

    def __init__(self, config: GPTConfig, rank: int, world: int) -> None:
        if config.head_dim != D or config.kv_heads != config.n_head or not config.tie_weights:
            raise ValueError("TP engine: head_dim 64, MHA, tied lm_head")
        C, L, H = config.n_embd, config.n_layer, config.n_head
        if world > H:
            raise ValueError("more tensor-parallel ranks than heads")
        if (4 * C) % world or ((4 * C) // world) % 8:
            raise ValueError("4*n_embd must split into multiples of 8 per rank")
        self.config, self.rank, self.world = config, rank, world
        self.heads = head_partition(H, world)
        self.h0, self.h1 = self.heads[rank]
        self.Hl = self.h1 - self.h0
        self.fl = 4 * C // world
        self.f0 = rank * self.fl
        self.Vp = padded_vocab(config.vocab_size, world)
        self.Vl = self.Vp // world
        self.v0 = rank * self.Vl
        self.vocab_valid = max(0, min(self.Vl, config.vocab_size - self.v0))
        hd = self.Hl * D
        sharded = []
        for l in range(L):
            p = f"h.{l}."
            sharded += [
                (p + "attn.c_attn.weight", (3 * hd, C), True),
                (p + "attn.c_attn.bias", (3 * hd,), False),
                (p + "attn.c_proj.weight", (C, hd), True),
                (p + "mlp.c_fc.weight", (self.fl, C), True),
                (p + "mlp.c_fc.bias", (self.fl,), False),
                (p + "mlp.c_proj.weight", (C, self.fl), True),
            ]
        sharded.append(("wte.weight", (self.Vl, C), True))
        repl = []
        for l in range(L):
            p = f"h.{l}."
            repl += [(p + "ln_1.weight", (C,), False), (p + "ln_1.bias", (C,), False),
                     (p + "ln_2.weight", (C,), False), (p + "ln_2.bias", (C,), False),
                     (p + "attn.c_proj.bias", (C,), False), (p + "mlp.c_proj.bias", (C,), False)]
        repl += [("ln_f.weight", (C,), False), ("ln_f.bias", (C,), False),
                 ("wpe.weight", (config.n_positions, C), True)]
        # Replicated tensors first, then the wte shard (equal on every rank),
        # then the block shards (whose sizes differ when heads split
        # unevenly): the replicated region and the wte shard sit at the same
        # offsets on every rank, which the peer-memory kernels rely on.
        wte = sharded.pop()
        self.specs: dict[str, tuple[int, tuple, bool]] = {}
        off = 0
        for name, shape, decay in repl + [wte] + sharded:
            if name == wte[0]:
                self.repl_hi = off
            self.specs[name] = (off, shape, decay)
            off += _align(math.prod(shape))
        self.total = off

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        off, shape, _ = self.specs[name]
        return flat[off:off + math.prod(shape)].view(shape)

    def decay_ranges(self) -> list[int]:
        out = []
        for off, shape, decay in sorted(self.specs.values()):
            if not decay:
                continue
            hi = off + _align(math.prod(shape))
            if out and out[-1] == off:
                out[-1] = hi
            else:
                out += [off, hi]
        return out

    def shard_of(self, name: str, full: torch.Tensor) -> torch.Tensor:
        """This rank's piece of a full (reference-shaped) tensor."""
        C = self.config.n_embd
        a, b = self.h0 * D, self.h1 * D
        if name.endswith("attn.c_attn.weight") or name.endswith("attn.c_attn.bias"):
            return torch.cat([full[a:b], full[C + a:C + b], full[2 * C + a:2 * C + b]], 0)
        if name.endswith("attn.c_proj.weight"):
            return full[:, a:b]
        if name.endswith("mlp.c_fc.weight") or name.endswith("mlp.c_fc.bias"):
            return full[self.f0:self.f0 + self.fl]
        if name.endswith("mlp.c_proj.weight"):
            return full[:, self.f0:self.f0 + self.fl]
        if name == "wte.weight":
            out = torch.zeros(self.Vl, C, dtype=full.dtype, device=full.device)
            out[:self.vocab_valid] = full[self.v0:self.v0 + self.vocab_valid]
            return out
        return full


class TPEngine:
    """GPT-2 training step with tensor + sequence parallelism over the group.

    Every rank passes the same global batch (B, T); rank r computes the
    residual stream of token rows [r*M/p, (r+1)*M/p) (M = B*T, a multiple of
    p). :meth:`train_step` runs forward, backward and AdamW.
    """

    def __init__(self, config: GPTConfig, B: int, T: int, device=None, *,
                 optim: Optional[OptimConfig] = None, group=None, seed: int = 0,
                 nblocks: int = 128, fused: bool = True) -> None:
        if not dist.is_initialized():
            # a single process: a one-rank group over an in-memory store (the
            # peer-memory kernels then run with world 1)
            dev0 = torch.device(device) if device is not None else torch.device(
                "cuda", torch.cuda.current_device())
            dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                    device_id=dev0)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        L = N.lib()
        self.config = cfg = config
        self.optim = optim or OptimConfig()
        self.lay = lay = TPLayout(cfg, self.rank, self.world)
        C, NL = cfg.n_embd, cfg.n_layer
        self.B, self.T = B, T
        self.M = M = B * T
        if M % self.world or T > cfg.n_positions:
            raise ValueError("B*T must be a multiple of the group size and T <= n_positions")
        self.Ms = Ms = M // self.world
        self.nblocks = nblocks
        bf, f32 = torch.bfloat16, torch.float32
        # parameters: bf16 copy and fp32 gradient are symmetric (the wte shard
        # is read and its gradient written by peers)
        self._p16 = SymmetricBuffer(lay.total * 2, group, dev)
        self._g32 = SymmetricBuffer(lay.total * 4, group, dev)
        self.shadow = self._p16.view(bf, lay.total)
        self.grad = self._g32.view(f32, lay.total)
        self.master = torch.zeros(lay.total, dtype=f32, device=dev)
        self.exp_avg = torch.zeros(lay.total, dtype=f32, device=dev)
        self.exp_avg_sq = torch.zeros(lay.total, dtype=f32, device=dev)
        self.decay = torch.tensor(lay.decay_ranges() or [0, 0], dtype=torch.int64, device=dev)
        # cross-rank activation buffers
        nG = 2 * NL + 1
        self._G = SymmetricBuffer(nG * M * C * 2, group, dev)   # gathered LayerNorm outputs
        # Row-parallel partials and the gathered residual gradient are double
        # buffered: use k+2 rewrites a buffer only after every rank has passed
        # the handshake of use k+1, i.e. finished reading use k.
        self._P = SymmetricBuffer(2 * M * C * 2, group, dev)    # row-parallel partials / inboxes
        self._D = SymmetricBuffer(2 * M * C * 2, group, dev)    # gathered residual gradient
        self._stats = SymmetricBuffer(M * 4 * 4, group, dev)
        self._flags = SymmetricBuffer(L.tp_flag_words() * 4, group, dev)
        self._ar_flags = SymmetricBuffer(L.comm_flag_words() * 4, group, dev)
        Gall = self._G.view(bf, nG * M * C).view(nG, M, C)
        self.G1 = [Gall[2 * l] for l in range(NL)]
        self.G2 = [Gall[2 * l + 1] for l in range(NL)]
        self.Gf = Gall[2 * NL]
        Pall = self._P.view(bf, 2 * M * C).view(2, M, C)
        Dall = self._D.view(bf, 2 * M * C).view(2, M, C)
        self.Pbuf = [Pall[0], Pall[1]]
        self.Dbuf = [Dall[0], Dall[1]]
        self._pb = 0  # partial buffer of the next row-parallel GEMM
        self._db = 0  # gradient buffer of the next residual-gradient gather
        # Fused collectives (more than one rank): the LayerNorms store their
        # rows into every rank's gather buffer (the gather kernels only
        # synchronise) and the row-parallel GEMMs store each partial row into
        # its owner's inbox, [p][Ms][C] in the partial buffer (the
        # reduce-scatter kernels sum local memory).
        self.fused = fused and self.world > 1 and os.environ.get("G2B_TP_FUSED", "1") != "0"
        self._push_G = self._push_desc(self._G)
        self._push_D = self._push_desc(self._D)
        self._owner = [torch.tensor([self._P.peer_ptrs[q] + (b * M * C + self.rank * Ms * C) * 2
                                     for q in range(self.world)], dtype=torch.int64, device=dev)
                       for b in (0, 1)]
        self.stats = self._stats.view(f32, M * 4).view(M, 4)
        r0 = self.rank * Ms
        own = slice(r0, r0 + Ms)
        self.own = own
        # local activations
        hd, fl = lay.Hl * D, lay.fl
        self.x = [torch.empty(Ms, C, dtype=f32, device=dev) for _ in range(2 * NL + 1)]
        self.mu = [torch.empty(Ms, dtype=f32, device=dev) for _ in range(2 * NL + 1)]
        self.rs = [torch.empty(Ms, dtype=f32, device=dev) for _ in range(2 * NL + 1)]
        self.qkv = [torch.empty(M, 3 * hd, dtype=bf, device=dev) for _ in range(NL)]
        self.y = [torch.empty(M, hd, dtype=bf, device=dev) for _ in range(NL)]
        self.lse = [torch.empty(B, lay.Hl, T, dtype=f32, device=dev) for _ in range(NL)]
        self.u = [torch.empty(M, fl, dtype=bf, device=dev) for _ in range(NL)]
        self.g = [torch.empty(M, fl, dtype=bf, device=dev) for _ in range(NL)]
        self.ld = _align(lay.Vl)
        self.logits = torch.empty(M, self.ld, dtype=bf, device=dev)
        self.loss_rows = torch.empty(M, dtype=f32, device=dev)
        self.loss_out = torch.zeros(2, dtype=f32, device=dev)
        self.dres = torch.empty(Ms, C, dtype=f32, device=dev)
        self.dh = torch.empty(Ms, C, dtype=bf, device=dev)
        self.du = torch.empty(M, fl, dtype=bf, device=dev)
        self.dy = torch.empty(M, hd, dtype=bf, device=dev)
        self.dqkv = torch.empty(M, 3 * hd, dtype=bf, device=dev)
        self.delta = torch.empty(B, lay.Hl, T, dtype=f32, device=dev)
        self.ln_parts = N.layernorm_bwd_partials(Ms, C, dev)
        self.col_ws = torch.empty(N.colsum_ws_numel(M, max(fl, 3 * hd, C)), dtype=f32, device=dev)
        self.splits = {"c_attn": choose_splits(3 * hd, C, M), "c_proj": choose_splits(C, hd, M),
                       "c_fc": choose_splits(fl, C, M), "mlp_proj": choose_splits(C, fl, M),
                       "wte": 1}
        ws = max(self.splits["c_attn"] * 3 * hd * C, self.splits["c_proj"] * C * hd,
                 self.splits["c_fc"] * fl * C, self.splits["mlp_proj"] * C * fl)
        self.splitk_ws = torch.empty(ws, dtype=f32, device=dev)
        # optimiser scalars
        self.hp = torch.zeros(8, dtype=f32, device=dev)
        self._hp_ring = [torch.zeros(8, dtype=f32).pin_memory() for _ in range(4)]
        self._hp_events: list = [None] * 4
        self._norm_ws = torch.empty(1024, dtype=f32, device=dev)
        self.sumsq = torch.zeros(2, dtype=f32, device=dev)
        self.clip = torch.ones(1, dtype=f32, device=dev)
        self.grad_norm = torch.zeros(1, dtype=f32, device=dev)
        self.byte_counter = torch.zeros(1, dtype=torch.int64, device=dev)
        self.step_count = 0
        self.epoch = 0
        self.ar_epoch = 0
        self.init_weights(seed)

    # ----------------------------------------------------------- weights --
    def set_lr(self, lr: float) -> None:
        self.optim.lr = lr

    def p16(self, name: str) -> torch.Tensor:
        return self.lay.view(self.shadow, name)

    def g32(self, name: str) -> torch.Tensor:
        return self.lay.view(self.grad, name)

    @torch.no_grad()
    def load_full(self, full_layout: ParamLayout, full: torch.Tensor, exp_avg: Optional[torch.Tensor] = None,
                  exp_avg_sq: Optional[torch.Tensor] = None) -> None:
        """Take this rank's pieces of full flat fp32 vectors in the
        single-GPU engine layout (weights, and optionally the AdamW moments)."""
        for dst, src in ((self.master, full), (self.exp_avg, exp_avg), (self.exp_avg_sq, exp_avg_sq)):
            if src is None:
                continue
            for name in self.lay.specs:
                self.lay.view(dst, name).copy_(self.lay.shard_of(name, full_layout.view(src, name)))
        self.shadow.copy_(self.master)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    @torch.no_grad()
    def load_full_grads(self, full_layout: ParamLayout, full_grad: torch.Tensor) -> None:
        """Set this rank's gradient shards from a full flat gradient in the
        single-GPU layout (as if backward plus the replicated all-reduce had
        produced it); used to check the optimiser in isolation."""
        for name in self.lay.specs:
            self.lay.view(self.grad, name).copy_(self.lay.shard_of(name, full_layout.view(full_grad, name)))

    @torch.no_grad()
    def init_weights(self, seed: int = 0) -> None:
        """The single-GPU engine's init (same seed, same weights), sliced."""
        full_layout = ParamLayout(self.config)
        full = torch.empty(full_layout.total, dtype=torch.float32, device=self.device)
        init_flat_weights(full_layout, full, seed)
        self.load_full(full_layout, full)
        del full

    # ---------------------------------------------------- communication --
    def _args(self, sym: SymmetricBuffer, **kw) -> dict:
        self.epoch += 1
        d = {"peer_bufs": sym.peer_ptrs_dev.data_ptr(), "peer_flags": self._flags.peer_ptrs_dev.data_ptr(),
             "rank": self.rank, "world": self.world, "nblocks": self.nblocks,
             "epoch": self.epoch & 0xFFFFFFFF, "err": N.error_word(self.device).data_ptr(),
             "byte_counter": self.byte_counter.data_ptr()}
        d.update(kw)
        return d

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _ag(self, sym: SymmetricBuffer, offset_bytes: int = 0) -> None:
        """All-gather of the row blocks of a [M, C] bf16 buffer."""
        C = self.config.n_embd
        comms.record_external("all_gather", self.M * C, self.M * C * 2)
        d = self._args(sym, rows=self.Ms, cols=C, pushed=int(self.fused))
        if offset_bytes:
            d["peer_bufs"] = self._offset_ptrs(sym, offset_bytes).data_ptr()
        with nvtx_range("tp/all_gather"):
            N.lib().tp_ag_rows(d, self._stream())

    def _offset_ptrs(self, sym: SymmetricBuffer, offset_bytes: int) -> torch.Tensor:
        key = (id(sym), offset_bytes)
        cache = self.__dict__.setdefault("_ptr_cache", {})
        if key not in cache:
            cache[key] = torch.tensor([p + offset_bytes for p in sym.peer_ptrs], dtype=torch.int64,
                                      device=self.device)
        return cache[key]

    def _push_desc(self, sym: SymmetricBuffer) -> tuple:
        """Row-push descriptor of a symmetric buffer: every other rank's base
        address, their count and this rank's base (see N.layernorm_fwd)."""
        others = [ptr for q, ptr in enumerate(sym.peer_ptrs) if q != self.rank]
        return (torch.tensor(others or [0], dtype=torch.int64, device=self.device), len(others),
                sym.peer_ptrs[self.rank])

    def _row_gemm(self, a: torch.Tensor, w: torch.Tensor, **kw) -> None:
        """A row-parallel GEMM into the current partial buffer; fused, every
        row goes straight into its owner's inbox over NVLink."""
        out = self.Pbuf[self._pb]
        if self.fused:
            N.gemm(a, w, out, owner_out=(self._owner[self._pb], self.Ms, self.rank), **kw)
        else:
            N.gemm(a, w, out, **kw)

    def _rs(self, bias=None, resid=None, out_f32=None, out_bf16=None) -> None:
        """Reduce-scatter of the current partial buffer into this rank's rows
        (fused: the local inbox; else peers' partials by P2P loads)."""
        C, b = self.config.n_embd, self._pb
        comms.record_external("reduce_scatter", self.M * C, self.M * C * 2)
        d = self._args(self._P, rows=self.Ms, cols=C,
                       bias=0 if bias is None else bias.data_ptr(),
                       resid=0 if resid is None else resid.data_ptr(),
                       out_f32=0 if out_f32 is None else out_f32.data_ptr(),
                       out_bf16=0 if out_bf16 is None else out_bf16.data_ptr())
        if self.fused:
            d["inbox"] = self.Pbuf[b].data_ptr()
        elif b:
            d["peer_bufs"] = self._offset_ptrs(self._P, b * self.M * C * 2).data_ptr()
        with nvtx_range("tp/reduce_scatter"):
            N.lib().tp_rs_rows(d, self._stream())
        self._pb ^= 1

    def _grad_rows(self) -> torch.Tensor:
        """Where the next LayerNorm backward writes this rank's bf16 rows."""
        return self.Dbuf[self._db][self.own]

    def _gather_grad(self) -> torch.Tensor:
        """All-gather of the residual-gradient rows just written; returns the
        gathered [M, C] buffer (the next writes go to the other buffer)."""
        b = self._db
        self._ag(self._D, b * self.M * self.config.n_embd * 2)
        self._db ^= 1
        return self.Dbuf[b]

    def _g_offset(self, which: str, l: int = 0) -> int:
        C, M, NL = self.config.n_embd, self.M, self.config.n_layer
        k = {"G1": 2 * l, "G2": 2 * l + 1, "Gf": 2 * NL}[which]
        return k * M * C * 2

    # ----------------------------------------------------------- forward --
    def forward(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        cfg, lay = self.config, self.lay
        C, NL, H = cfg.n_embd, cfg.n_layer, lay.Hl
        B, T, own = self.B, self.T, self.own
        eps = cfg.layer_norm_epsilon
        p = self.p16
        idx = idx.contiguous().view(-1)
        self._targets = targets.contiguous().view(-1)
        self._idx = idx
        hd = H * D
        # embedding of this rank's rows (wte rows from their owners' shards)
        wte_off = lay.specs["wte.weight"][0] * 2
        d = self._args(self._p16, rows=self.Ms, cols=C, idx=idx.data_ptr(),
                       wpe=p("wpe.weight").data_ptr(), T=T, vocab_per_rank=lay.Vl,
                       out_f32=self.x[0].data_ptr())
        d["peer_bufs"] = self._offset_ptrs(self._p16, wte_off).data_ptr()
        # each rank receives its rows' token embeddings from their owners
        comms.record_external("all_to_all", self.Ms * C, self.Ms * C * 2)
        N.lib().tp_embed_fwd(d, self._stream())
        for l in range(NL):
            pre = f"h.{l}."
            G1, G2 = self.G1[l], self.G2[l]
            N.layernorm_fwd(self.x[2 * l], p(pre + "ln_1.weight"), p(pre + "ln_1.bias"), G1[own],
                            self.mu[2 * l], self.rs[2 * l], eps, push=self._push_G if self.fused else None)
            self._ag(self._G, self._g_offset("G1", l))
            N.gemm(G1, p(pre + "attn.c_attn.weight"), self.qkv[l], bias=p(pre + "attn.c_attn.bias"))
            qkv = self.qkv[l]
            N.attention_fwd(qkv[:, :hd], qkv[:, hd:2 * hd], qkv[:, 2 * hd:], self.y[l], self.lse[l],
                            B, H, T)
            self._row_gemm(self.y[l], p(pre + "attn.c_proj.weight"))
            self._rs(bias=p(pre + "attn.c_proj.bias"), resid=self.x[2 * l], out_f32=self.x[2 * l + 1])
            N.layernorm_fwd(self.x[2 * l + 1], p(pre + "ln_2.weight"), p(pre + "ln_2.bias"), G2[own],
                            self.mu[2 * l + 1], self.rs[2 * l + 1], eps, push=self._push_G if self.fused else None)
            self._ag(self._G, self._g_offset("G2", l))
            N.gemm(G2, p(pre + "mlp.c_fc.weight"), self.g[l], epilogue=N.EPI_BIAS_GELU,
                   bias=p(pre + "mlp.c_fc.bias"), aux=self.u[l])
            self._row_gemm(self.g[l], p(pre + "mlp.c_proj.weight"))
            self._rs(bias=p(pre + "mlp.c_proj.bias"), resid=self.x[2 * l + 1], out_f32=self.x[2 * l + 2])
        N.layernorm_fwd(self.x[2 * NL], p("ln_f.weight"), p("ln_f.bias"), self.Gf[own],
                        self.mu[2 * NL], self.rs[2 * NL], eps, push=self._push_G if self.fused else None)
        self._ag(self._G, self._g_offset("Gf"))
        N.gemm(self.Gf, p("wte.weight"), self.logits[:, :lay.Vl])
        # vocabulary-parallel cross-entropy
        L = N.lib()
        L.tp_ce_stats({"rows": self.M, "logits": self.logits.data_ptr(), "ld": self.ld,
                       "vocab_valid": lay.vocab_valid, "vocab_start": lay.v0,
                       "idx": self._targets.data_ptr(), "stats": self.stats.data_ptr()}, self._stream())
        d = self._args(self._stats, rows=self.M, logits=self.logits.data_ptr(), ld=self.ld,
                       vocab_valid=lay.vocab_valid, vocab_start=lay.v0, idx=self._targets.data_ptr(),
                       loss_rows=self.loss_rows.data_ptr())
        # every rank reads every peer's [M, 4] row statistics (max, sum, target)
        comms.record_external("all_gather", self.world * self.M * 4, self.world * self.M * 4 * 4)
        L.tp_ce_finish(d, self._stream())
        L.loss_reduce(self.loss_rows.data_ptr(), self._targets.data_ptr(), self.M,
                      self.loss_out.data_ptr(), self._stream())
        return self.loss_out[0]

    # ---------------------------------------------------------- backward --
    def backward(self) -> None:
        cfg, lay = self.config, self.lay
        C, NL, H = cfg.n_embd, cfg.n_layer, lay.Hl
        B, T, own = self.B, self.T, self.own
        p, g = self.p16, self.g32
        hd = H * D
        inv = self.loss_out[1:2]
        dl = self.logits[:, :lay.Vl]
        ws = self.splitk_ws
        # lm_head (tied, vocabulary-parallel)
        self._row_gemm(dl, p("wte.weight"), b_t=True, alpha_ptr=inv)
        N.gemm(dl, self.Gf, g("wte.weight"), a_t=True, b_t=True, epilogue=N.EPI_F32, alpha_ptr=inv)
        self._rs(out_bf16=self.dh)
        Down = self._grad_rows()
        N.layernorm_bwd(self.dh, self.x[2 * NL], self.mu[2 * NL], self.rs[2 * NL], p("ln_f.weight"),
                        self.dres, Down, g("ln_f.weight"), g("ln_f.bias"), self.ln_parts,
                        accumulate_dres=False, accumulate_params=False, push=self._push_D if self.fused else None)
        for l in reversed(range(NL)):
            pre = f"h.{l}."
            # --- MLP
            N.colsum_bf16(Down, g(pre + "mlp.c_proj.bias"), self.col_ws, accumulate=False)
            Dg = self._gather_grad()
            N.gemm(Dg, p(pre + "mlp.c_proj.weight"), self.du, b_t=True, epilogue=N.EPI_GELU_BWD,
                   aux=self.u[l])
            N.gemm(Dg, self.g[l], g(pre + "mlp.c_proj.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, splits=self.splits["mlp_proj"], workspace=ws)
            self._row_gemm(self.du, p(pre + "mlp.c_fc.weight"), b_t=True)
            N.gemm(self.du, self.G2[l], g(pre + "mlp.c_fc.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, splits=self.splits["c_fc"], workspace=ws)
            N.colsum_bf16(self.du, g(pre + "mlp.c_fc.bias"), self.col_ws, accumulate=False)
            self._rs(out_bf16=self.dh)
            Down = self._grad_rows()
            N.layernorm_bwd(self.dh, self.x[2 * l + 1], self.mu[2 * l + 1], self.rs[2 * l + 1],
                            p(pre + "ln_2.weight"), self.dres, Down, g(pre + "ln_2.weight"),
                            g(pre + "ln_2.bias"), self.ln_parts, accumulate_dres=True,
                            accumulate_params=False, push=self._push_D if self.fused else None)
            # --- attention
            N.colsum_bf16(Down, g(pre + "attn.c_proj.bias"), self.col_ws, accumulate=False)
            Dg = self._gather_grad()
            N.gemm(Dg, p(pre + "attn.c_proj.weight"), self.dy, b_t=True)
            N.gemm(Dg, self.y[l], g(pre + "attn.c_proj.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, splits=self.splits["c_proj"], workspace=ws)
            qkv, dqkv = self.qkv[l], self.dqkv
            N.attention_bwd(qkv[:, :hd], qkv[:, hd:2 * hd], qkv[:, 2 * hd:], self.y[l], self.dy,
                            dqkv[:, :hd], dqkv[:, hd:2 * hd], dqkv[:, 2 * hd:], self.lse[l], self.delta,
                            B, H, T)
            self._row_gemm(dqkv, p(pre + "attn.c_attn.weight"), b_t=True)
            N.gemm(dqkv, self.G1[l], g(pre + "attn.c_attn.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, splits=self.splits["c_attn"], workspace=ws)
            N.colsum_bf16(dqkv, g(pre + "attn.c_attn.bias"), self.col_ws, accumulate=False)
            self._rs(out_bf16=self.dh)
            Down = self._grad_rows()
            N.layernorm_bwd(self.dh, self.x[2 * l], self.mu[2 * l], self.rs[2 * l],
                            p(pre + "ln_1.weight"), self.dres, Down, g(pre + "ln_1.weight"),
                            g(pre + "ln_1.bias"), self.ln_parts, accumulate_dres=True,
                            accumulate_params=False, push=self._push_D if self.fused else None)
        # embedding: wte rows into their owners' gradient shards, wpe locally
        wpe_g = g("wpe.weight")
        wpe_g.zero_()
        wte_off = lay.specs["wte.weight"][0] * 4
        d = self._args(self._g32, rows=self.Ms, cols=C, idx=self._idx.data_ptr(), T=T,
                       vocab_per_rank=lay.Vl, resid=self.dres.data_ptr(), out_f32=wpe_g.data_ptr())
        d["peer_bufs"] = self._offset_ptrs(self._g32, wte_off).data_ptr()
        # each rank pushes its rows' fp32 gradients to the embedding owners
        comms.record_external("all_to_all", self.Ms * C, self.Ms * C * 4)
        N.lib().tp_embed_bwd(d, self._stream())
        # replicated parameters: sum the per-rank partial gradients
        n = lay.repl_hi
        count = 0
        for name, (off, shape, _) in lay.specs.items():
            if off < n:
                numel = math.prod(shape)
                count += numel
                comms.record_external("all_reduce", numel, numel * 4)
        self.ar_epoch += 1
        N.lib().allreduce_p2p(self._g32.peer_ptrs_dev.data_ptr(), self._ar_flags.peer_ptrs_dev.data_ptr(),
                              self.rank, self.world, 0, n, 0, 1.0, self.ar_epoch & 0xFFFFFFFF,
                              self.byte_counter.data_ptr(), N.error_word(self.device).data_ptr(),
                              self.nblocks, 2_000_000_000, count, self._stream())

    # --------------------------------------------------------- optimiser --
    def optimizer_step(self) -> None:
        o, lay = self.optim, self.lay
        self.step_count += 1
        t = self.step_count
        slot = t % 4
        if self._hp_events[slot] is not None:
            self._hp_events[slot].synchronize()
        hp = self._hp_ring[slot]
        hp[0], hp[1], hp[2], hp[3], hp[4] = o.lr, o.betas[0], o.betas[1], o.eps, o.weight_decay
        hp[5] = 1.0 - o.betas[0] ** t
        hp[6] = math.sqrt(1.0 - o.betas[1] ** t)
        hp[7] = 1.0
        self.hp.copy_(hp, non_blocking=True)
        ev = self._hp_events[slot] or torch.cuda.Event()
        ev.record()
        self._hp_events[slot] = ev
        clip = None
        if o.grad_clip and o.grad_clip > 0:
            N.grad_sumsq(self.grad[lay.repl_hi:], self._norm_ws, self.sumsq[0:1])
            comms.record_external("all_reduce", 1, 4)
            dist.all_reduce(self.sumsq[0:1], group=self.group)
            N.grad_sumsq(self.grad[:lay.repl_hi], self._norm_ws, self.sumsq[1:2])
            N.clip_coef(self.sumsq.sum(0, keepdim=True), o.grad_clip, self.clip, self.grad_norm)
            clip = self.clip
        N.adamw_step(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.shadow, 0, self.hp,
                     clip, decay_ranges=self.decay)

    def train_step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        loss = self.forward(idx, targets)
        self.backward()
        self.optimizer_step()
        return loss

    # ------------------------------------------------------------- state --
    def full_state(self, which: str = "master") -> dict:
        """Reference-named full tensors rebuilt from every rank's shards (a
        collective). ``which`` is ``master``, ``grad``, ``exp_avg`` or ``exp_avg_sq``."""
        src = {"master": self.master, "grad": self.grad, "exp_avg": self.exp_avg,
               "exp_avg_sq": self.exp_avg_sq}[which]
        lays = [TPLayout(self.config, r, self.world) for r in range(self.world)]
        # ranks' layouts differ in length when heads split unevenly: pad
        n = max(l.total for l in lays)
        buf = torch.zeros(n, dtype=src.dtype, device=src.device)
        buf[:src.numel()].copy_(src)
        parts = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(parts, buf, group=self.group)
        cfg = self.config
        C = cfg.n_embd
        out = {}
        for name in self.lay.specs:
            pieces = [lays[r].view(parts[r], name) for r in range(self.world)]
            if name == "wte.weight":
                out[name] = torch.cat(pieces, 0)[:cfg.vocab_size].clone()
            elif name.endswith("attn.c_attn.weight") or name.endswith("attn.c_attn.bias"):
                secs = []
                for sec in range(3):
                    secs += [pc[sec * lays[r].Hl * D:(sec + 1) * lays[r].Hl * D] for r, pc in enumerate(pieces)]
                # order: q of all ranks, k of all ranks, v of all ranks
                q = torch.cat([secs[r] for r in range(self.world)], 0)
                k = torch.cat([secs[self.world + r] for r in range(self.world)], 0)
                v = torch.cat([secs[2 * self.world + r] for r in range(self.world)], 0)
                out[name] = torch.cat([q, k, v], 0).clone()
            elif name.endswith("attn.c_proj.weight") or name.endswith("mlp.c_proj.weight"):
                out[name] = torch.cat(pieces, 1).clone()
            elif name.endswith("mlp.c_fc.weight") or name.endswith("mlp.c_fc.bias"):
                out[name] = torch.cat(pieces, 0).clone()
            else:
                out[name] = pieces[0].clone()
        return out

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for b in (self._p16, self._g32, self._G, self._P, self._D, self._stats, self._flags, self._ar_flags):
            b.close()
