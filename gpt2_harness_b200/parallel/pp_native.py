"""Pipeline parallelism on the native engine kernels.

Reference semantics (src/transformer_internals/parallel/pipeline_parallel.py
:56-336): a contiguous depth split, stage 0 owning the embeddings and the last
stage ln_f and an lm_head UNTIED from wte; GPipe or 1F1B over m micro-batches
(``schedule_order``); non-blocking sends and blocking receives of the fp32
residual stream and of its gradient; the loss of every micro-batch divided by
m; gradients accumulated over the micro-batches, then one optimiser step.

B200 design:

* :class:`StageEngine` runs this stage's blocks with the engine's sm_100a
  kernels (tcgen05 GEMMs with fused epilogues, flash attention, LayerNorm,
  cross-entropy, AdamW) on per-micro-batch activation slots, so the forwards
  of several micro-batches can be in flight before their backwards (1F1B keeps
  at most p, GPipe m).
* Stage boundaries are NCCL point-to-point transfers (isend / irecv), which
  run on NCCL's own streams: a send overlaps the next micro-batch's compute; a
  receive makes the compute stream wait on the device, not the host.
  Activations and gradients travel on two different communicators. On one
  communicator the two directions would share one NCCL stream per rank pair,
  and 1F1B issues them in different orders on the two sides (stage s sends
  activation p-s-1 before it receives gradient 0; stage s+1 sends gradient 0
  before it receives that activation), so two rendezvous sends would wait for
  each other on the device. Per direction the order is the same on both
  sides.
* Clipping uses the global norm over all stages (one 4-byte all-reduce);
  the attention can be delegated to a context-parallel group through the same
  hooks as the single-GPU engine (``attn_fwd_hook`` / ``attn_bwd_hook`` /
  ``pos0``, plus ``slot_hook`` so that the gathered K/V of every micro-batch
  in flight is kept), which is how the PP x CP mesh composes; the stage's
  weight gradients are then averaged over the context-parallel group by the
  fused peer-memory all-reduce before the norm.
"""

from __future__ import annotations

import math
from typing import Callable, Optional

import torch
import torch.distributed as dist

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.engine import (ALIGN, OptimConfig, ParamLayout, choose_splits, init_flat_weights,
                                            qkv_views, qkv_width)
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.pipeline_parallel import schedule_order
from gpt2_harness_b200.parallel.symm import P2PAllReducer

__all__ = ["StageLayout", "StageEngine", "PipelineMesh", "make_mesh"]


def _align(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


class StageLayout:
    """Flat layout of one stage's parameters (reference names)."""

    def __init__(self, config: GPTConfig, stage: int, n_stages: int) -> None:
        L, C = config.n_layer, config.n_embd
        if L % n_stages:
            raise ValueError(f"n_layer={L} must be divisible by n_stages={n_stages}")
        per = L // n_stages
        self.l0, self.l1 = stage * per, (stage + 1) * per
        self.first, self.last = stage == 0, stage == n_stages - 1
        full = ParamLayout(config)
        specs = []
        if self.first:
            specs += [("wte.weight", (config.vocab_size, C), True), ("wpe.weight", (config.n_positions, C), True)]
        for s in full.specs:
            if s.group.startswith("h.") and self.l0 <= int(s.group.split(".")[1]) < self.l1:
                specs.append((s.name, s.shape, s.decay))
        if self.last:
            specs += [("ln_f.weight", (C,), False), ("ln_f.bias", (C,), False),
                      ("lm_head.weight", (config.vocab_size, C), True)]
        self.specs: dict[str, tuple[int, tuple, bool]] = {}
        off = 0
        for name, shape, decay in specs:
            self.specs[name] = (off, shape, decay)
            off += _align(math.prod(shape))
        self.total = off

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        off, shape, _ = self.specs[name]
        return flat[off:off + math.prod(shape)].view(shape)

    def decay_ranges(self) -> list[int]:
        out = []
        for off, shape, decay in sorted(self.specs.values()):
            if decay:
                hi = off + _align(math.prod(shape))
                if out and out[-1] == off:
                    out[-1] = hi
                else:
                    out += [off, hi]
        return out or [0, 0]


class _Slot:
    """Activations of one micro-batch on this stage."""

    def __init__(self, cfg: GPTConfig, n: int, M: int, B: int, T: int, last: bool, dev) -> None:
        C, H = cfg.n_embd, cfg.n_head
        bf, f32 = torch.bfloat16, torch.float32
        self.x = [torch.empty(M, C, dtype=f32, device=dev) for _ in range(2 * n + 1)]
        self.mu = [torch.empty(M, dtype=f32, device=dev) for _ in range(2 * n + 1)]
        self.rs = [torch.empty(M, dtype=f32, device=dev) for _ in range(2 * n + 1)]
        self.h1 = [torch.empty(M, C, dtype=bf, device=dev) for _ in range(n)]
        self.qkv = [torch.empty(M, qkv_width(cfg), dtype=bf, device=dev) for _ in range(n)]
        self.y = [torch.empty(M, C, dtype=bf, device=dev) for _ in range(n)]
        self.lse = [torch.empty(B, H, T, dtype=f32, device=dev) for _ in range(n)]
        self.h2 = [torch.empty(M, C, dtype=bf, device=dev) for _ in range(n)]
        self.u = [torch.empty(M, 4 * C, dtype=bf, device=dev) for _ in range(n)]
        self.g = [torch.empty(M, 4 * C, dtype=bf, device=dev) for _ in range(n)]
        self.dx_out = torch.empty(M, C, dtype=f32, device=dev)   # gradient sent upstream
        self.send_fwd = None   # in-flight send of x[-1]
        self.send_bwd = None   # in-flight send of dx_out
        if last:
            self.hf = torch.empty(M, C, dtype=bf, device=dev)
            self.logits = torch.empty(M, cfg.padded_vocab_size(), dtype=bf, device=dev)
            self.loss_rows = torch.empty(M, dtype=f32, device=dev)
            self.loss_out = torch.zeros(2, dtype=f32, device=dev)


class StageEngine:
    """One pipeline stage (this rank) of GPT-2 on the native kernels.

    Every rank of the pipeline group calls :meth:`train_step` with the same
    micro-batches (only stage 0 reads the token ids, only the last stage the
    targets); it returns the mean micro-batch loss on the last stage.
    """

    def __init__(self, config: GPTConfig, micro_batch: int, seq_len: int, micro_batches: int, *,
                 schedule: str = "1f1b", optim: Optional[OptimConfig] = None, group=None,
                 p2p_groups: Optional[tuple] = None, dp_group=None, device=None, seed: int = 0,
                 comm_blocks: int = 128) -> None:
        if not dist.is_initialized():
            raise RuntimeError("StageEngine needs an initialised process group")
        # the full-model layout (tied GPT-2, head_dim 64) defines the init;
        # the last stage then unties lm_head from wte
        ParamLayout(config)
        self.group = group
        self.p = dist.get_world_size(group)
        self.stage = dist.get_rank(group)
        self.ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.p))
        # (activation group, gradient group) over the same ranks; creating
        # them is collective over the default group.
        if p2p_groups is None:
            p2p_groups = (dist.new_group(self.ranks), dist.new_group(self.ranks))
        self.fwd_group, self.bwd_group = p2p_groups
        self.device = dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        N.lib()
        self.config = cfg = config
        self.optim = optim or OptimConfig()
        self.lay = lay = StageLayout(cfg, self.stage, self.p)
        self.n = lay.l1 - lay.l0
        self.B, self.T, self.m = micro_batch, seq_len, micro_batches
        self.M = M = micro_batch * seq_len
        self.schedule = schedule
        f32 = torch.float32
        self.master = torch.zeros(lay.total, dtype=f32, device=dev)
        self.shadow = torch.zeros(lay.total, dtype=torch.bfloat16, device=dev)
        # ranks that hold the same stage on different data (a context- or
        # data-parallel group) average gradients through a symmetric buffer
        self.dp = dist.get_world_size(dp_group) if dp_group is not None else 1
        self._reducer = None
        if self.dp > 1:
            self._reducer = P2PAllReducer(lay.total * 4, dp_group, dev, nblocks=comm_blocks)
            self.grad = self._reducer.tensor[:lay.total]
        else:
            self.grad = torch.zeros(lay.total, dtype=f32, device=dev)
        self.exp_avg = torch.zeros(lay.total, dtype=f32, device=dev)
        self.exp_avg_sq = torch.zeros(lay.total, dtype=f32, device=dev)
        self.decay = torch.tensor(lay.decay_ranges(), dtype=torch.int64, device=dev)
        # micro-batches in flight on this stage: all of them under GPipe, at
        # most p - stage under 1F1B (its warm-up depth plus one)
        nslots = micro_batches if schedule == "gpipe" else min(micro_batches, self.p - self.stage)
        self.slots = [_Slot(cfg, self.n, M, micro_batch, seq_len, lay.last, dev) for _ in range(nslots)]
        C = cfg.n_embd
        bf = torch.bfloat16
        self.dres = torch.empty(M, C, dtype=f32, device=dev)
        # the first stage sums its token-embedding gradient deterministically
        self.emb_ws = (N.EmbeddingGradWorkspace(M, C, config.vocab_size, dev)
                       if lay.first else None)
        self.dres16 = torch.empty(M, C, dtype=bf, device=dev)
        self.dh = torch.empty(M, C, dtype=bf, device=dev)
        self.dy = torch.empty(M, C, dtype=bf, device=dev)
        self.du = torch.empty(M, 4 * C, dtype=bf, device=dev)
        W = qkv_width(config)
        self.dqkv = torch.empty(M, W, dtype=bf, device=dev)
        self.delta = torch.empty(micro_batch, cfg.n_head, seq_len, dtype=f32, device=dev)
        self.ln_parts = N.layernorm_bwd_partials(M, C, dev)
        self.col_ws = torch.empty(N.colsum_ws_numel(M, 4 * C), dtype=f32, device=dev)
        self.splits = {"c_attn": choose_splits(W, C, M), "c_proj": choose_splits(C, C, M),
                       "c_fc": choose_splits(4 * C, C, M), "mlp_proj": choose_splits(C, 4 * C, M)}
        ws = max(self.splits["c_attn"] * W * C, self.splits["c_proj"] * C * C,
                 self.splits["c_fc"] * 4 * C * C, self.splits["mlp_proj"] * 4 * C * C)
        self.splitk_ws = torch.empty(ws, dtype=f32, device=dev)
        self.hp = torch.zeros(8, dtype=f32, device=dev)
        self._hp_ring = [torch.zeros(8, dtype=f32).pin_memory() for _ in range(4)]
        self._hp_events: list = [None] * 4
        self._norm_ws = torch.empty(1024, dtype=f32, device=dev)
        self.sumsq = torch.zeros(1, dtype=f32, device=dev)
        self.clip = torch.ones(1, dtype=f32, device=dev)
        self.grad_norm = torch.zeros(1, dtype=f32, device=dev)
        self.loss_sum = torch.zeros(1, dtype=f32, device=dev)
        self.step_count = 0
        # context-parallel composition (same hooks as the single-GPU engine)
        self.pos0 = 0
        self.pos_split: Optional[int] = None
        self.pos1 = 0
        self.attn_fwd_hook: Optional[Callable] = None
        self.attn_bwd_hook: Optional[Callable] = None
        self.slot_hook: Optional[Callable[[int], None]] = None
        self.init_weights(seed)
        self._connect()

    def _connect(self) -> None:
        """One tiny transfer along each direction of the pipeline, so every
        point-to-point communicator exists before the first step (a rank that
        creates one mid-step delays its context-parallel peers' kernels)."""
        if self.p == 1:
            return
        t = torch.zeros(1, dtype=torch.float32, device=self.device)
        for group, src, dst in ((self.fwd_group, -1, 1), (self.bwd_group, 1, -1)):
            has_src = 0 <= self.stage + src < self.p
            has_dst = 0 <= self.stage + dst < self.p
            if has_src:
                dist.irecv(t, self._peer(src), group=group).wait()
            if has_dst:
                dist.isend(t, self._peer(dst), group=group).wait()
        torch.cuda.synchronize(self.device)

    # ----------------------------------------------------------- weights --
    def p16(self, name: str) -> torch.Tensor:
        return self.lay.view(self.shadow, name)

    def g32(self, name: str) -> torch.Tensor:
        return self.lay.view(self.grad, name)

    @torch.no_grad()
    def init_weights(self, seed: int = 0) -> None:
        """The single-GPU engine's init (same seed, same weights) for this
        stage's tensors; the untied lm_head starts as a copy of wte."""
        full_layout = ParamLayout(self.config)
        full = torch.empty(full_layout.total, dtype=torch.float32, device=self.device)
        init_flat_weights(full_layout, full, seed)
        for name in self.lay.specs:
            src = full_layout.view(full, "wte.weight" if name == "lm_head.weight" else name)
            self.lay.view(self.master, name).copy_(src)
        self.shadow.copy_(self.master)
        del full

    # ------------------------------------------------------ point-to-point --
    def _peer(self, delta: int) -> int:
        return self.ranks[self.stage + delta]

    # ----------------------------------------------------------- forward --
    def _forward(self, S: _Slot, idx: Optional[torch.Tensor], targets: Optional[torch.Tensor]) -> None:
        cfg, lay = self.config, self.lay
        C, H, B, T = cfg.n_embd, cfg.n_head, self.B, self.T
        eps = cfg.layer_norm_epsilon
        p = self.p16
        if lay.first:
            N.embedding_fwd(idx, p("wte.weight"), p("wpe.weight"), S.x[0], pos0=self.pos0,
                            pos_split=self.pos_split, pos1=self.pos1)
        for j in range(self.n):
            pre = f"h.{lay.l0 + j}."
            N.layernorm_fwd(S.x[2 * j], p(pre + "ln_1.weight"), p(pre + "ln_1.bias"), S.h1[j],
                            S.mu[2 * j], S.rs[2 * j], eps)
            N.gemm(S.h1[j], p(pre + "attn.c_attn.weight"), S.qkv[j], bias=p(pre + "attn.c_attn.bias"))
            qkv = S.qkv[j]
            if self.attn_fwd_hook is not None:
                self.attn_fwd_hook(lay.l0 + j, qkv, S.y[j], S.lse[j], B, H, T)
            else:
                N.attention_fwd(*qkv_views(qkv, cfg), S.y[j], S.lse[j], B, H, T, kv_heads=cfg.kv_heads)
            N.gemm(S.y[j], p(pre + "attn.c_proj.weight"), S.x[2 * j + 1], epilogue=N.EPI_RESID_F32,
                   bias=p(pre + "attn.c_proj.bias"), aux=S.x[2 * j])
            N.layernorm_fwd(S.x[2 * j + 1], p(pre + "ln_2.weight"), p(pre + "ln_2.bias"), S.h2[j],
                            S.mu[2 * j + 1], S.rs[2 * j + 1], eps)
            N.gemm(S.h2[j], p(pre + "mlp.c_fc.weight"), S.g[j], epilogue=N.EPI_BIAS_GELU,
                   bias=p(pre + "mlp.c_fc.bias"), aux=S.u[j])
            N.gemm(S.g[j], p(pre + "mlp.c_proj.weight"), S.x[2 * j + 2], epilogue=N.EPI_RESID_F32,
                   bias=p(pre + "mlp.c_proj.bias"), aux=S.x[2 * j + 1])
        if lay.last:
            n, V = self.n, cfg.vocab_size
            N.layernorm_fwd(S.x[2 * n], p("ln_f.weight"), p("ln_f.bias"), S.hf, S.mu[2 * n], S.rs[2 * n], eps)
            N.gemm(S.hf, p("lm_head.weight"), S.logits[:, :V])
            N.cross_entropy_fwd_bwd(S.logits, targets.contiguous().view(-1), S.loss_rows, S.loss_out, V)
            self.loss_sum.add_(S.loss_out[0:1])

    # ---------------------------------------------------------- backward --
    def _backward(self, S: _Slot, idx: Optional[torch.Tensor], acc: bool) -> None:
        cfg, lay = self.config, self.lay
        C, H, B, T, V = cfg.n_embd, cfg.n_head, self.B, self.T, cfg.vocab_size
        p, g = self.p16, self.g32
        ws = self.splitk_ws
        n, l0 = self.n, lay.l0
        top_bias = g(f"h.{l0 + n - 1}.mlp.c_proj.bias")
        if lay.last:
            # each micro-batch's loss is divided by m: alpha = 1/m x 1/count
            inv = S.loss_out[1:2]
            logits = S.logits[:, :V]
            N.gemm(logits, p("lm_head.weight"), self.dh, b_t=True, alpha=1.0 / self.m, alpha_ptr=inv)
            N.gemm(logits, S.hf, g("lm_head.weight"), a_t=True, b_t=True, epilogue=N.EPI_F32,
                   alpha=1.0 / self.m, alpha_ptr=inv, accumulate=acc)
            N.layernorm_bwd(self.dh, S.x[2 * n], S.mu[2 * n], S.rs[2 * n], p("ln_f.weight"), self.dres,
                            self.dres16, g("ln_f.weight"), g("ln_f.bias"), self.ln_parts,
                            accumulate_dres=False, accumulate_params=acc, dsum=top_bias,
                            accumulate_dsum=acc)
        else:
            # self.dres holds the gradient received from the next stage; its
            # column sum is the bias gradient of this stage's last projection,
            # summed in fp32 as the single-GPU engine's LayerNorm backward does
            N.cast_f32_bf16(self.dres, self.dres16)
            N.colsum_f32(self.dres, top_bias, accumulate=acc)
        for j in reversed(range(n)):
            pre = f"h.{l0 + j}."
            N.gemm(self.dres16, p(pre + "mlp.c_proj.weight"), self.du, b_t=True, epilogue=N.EPI_GELU_BWD,
                   aux=S.u[j])
            N.gemm(self.dres16, S.g[j], g(pre + "mlp.c_proj.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=self.splits["mlp_proj"], workspace=ws)
            N.gemm(self.du, p(pre + "mlp.c_fc.weight"), self.dh, b_t=True)
            N.gemm(self.du, S.h2[j], g(pre + "mlp.c_fc.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=self.splits["c_fc"], workspace=ws)
            N.colsum_bf16(self.du, g(pre + "mlp.c_fc.bias"), self.col_ws, accumulate=acc)
            N.layernorm_bwd(self.dh, S.x[2 * j + 1], S.mu[2 * j + 1], S.rs[2 * j + 1],
                            p(pre + "ln_2.weight"), self.dres, self.dres16, g(pre + "ln_2.weight"),
                            g(pre + "ln_2.bias"), self.ln_parts, accumulate_dres=True,
                            accumulate_params=acc, dsum=g(pre + "attn.c_proj.bias"), accumulate_dsum=acc)
            N.gemm(self.dres16, p(pre + "attn.c_proj.weight"), self.dy, b_t=True)
            N.gemm(self.dres16, S.y[j], g(pre + "attn.c_proj.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=self.splits["c_proj"], workspace=ws)
            qkv, dqkv = S.qkv[j], self.dqkv
            if self.attn_bwd_hook is not None:
                self.attn_bwd_hook(l0 + j, qkv, S.y[j], self.dy, dqkv, S.lse[j], self.delta, B, H, T)
            else:
                N.attention_bwd(*qkv_views(qkv, cfg), S.y[j], self.dy, *qkv_views(dqkv, cfg), S.lse[j],
                                self.delta, B, H, T, kv_heads=cfg.kv_heads)
            N.gemm(dqkv, p(pre + "attn.c_attn.weight"), self.dh, b_t=True)
            N.gemm(dqkv, S.h1[j], g(pre + "attn.c_attn.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=self.splits["c_attn"], workspace=ws)
            N.colsum_bf16(dqkv, g(pre + "attn.c_attn.bias"), self.col_ws, accumulate=acc)
            # ln_1's residual gradient also gives the bias gradient of the
            # previous block's mlp.c_proj (on this stage)
            N.layernorm_bwd(self.dh, S.x[2 * j], S.mu[2 * j], S.rs[2 * j], p(pre + "ln_1.weight"),
                            self.dres, self.dres16, g(pre + "ln_1.weight"), g(pre + "ln_1.bias"),
                            self.ln_parts, accumulate_dres=True, accumulate_params=acc,
                            dsum=g(f"h.{l0 + j - 1}.mlp.c_proj.bias") if j > 0 else None,
                            accumulate_dsum=acc)
        if lay.first:
            wpe_g = g("wpe.weight")
            if not acc:
                g("wte.weight").zero_()
                wpe_g.zero_()
            N.embedding_bwd(idx, self.dres, g("wte.weight"), wpe_g, V, pos0=self.pos0,
                            pos_split=self.pos_split, pos1=self.pos1, det=self.emb_ws)

    # -------------------------------------------------------------- step --
    def train_step(self, micro_idx: list, micro_tgt: list) -> torch.Tensor:
        """One optimiser step over m micro-batches (lists of [B, T] device
        tensors; stage 0 reads the ids, the last stage the targets). Returns
        the mean micro-batch loss (a device scalar, meaningful on the last
        stage)."""
        lay, n = self.lay, self.n
        if len(micro_idx) != self.m or len(micro_tgt) != self.m:
            raise ValueError(f"expected {self.m} micro-batches")
        self.loss_sum.zero_()
        first_bwd = True
        nslot = len(self.slots)
        act_bytes = self.M * self.config.n_embd * 4
        for op, i in schedule_order(self.stage, self.p, self.m, self.schedule):
            S = self.slots[i % nslot]
            if self.slot_hook is not None:
                self.slot_hook(i % nslot)
            idx = micro_idx[i].contiguous() if lay.first else None
            if op == "F":
                if S.send_fwd is not None:     # the slot's previous output has left
                    S.send_fwd.wait()
                    S.send_fwd = None
                if not lay.first:
                    comms.record_external("recv", self.M * self.config.n_embd, act_bytes)
                    dist.irecv(S.x[0], self._peer(-1), group=self.fwd_group).wait()
                self._forward(S, idx, micro_tgt[i] if lay.last else None)
                if not lay.last:
                    comms.record_external("send", self.M * self.config.n_embd, act_bytes)
                    S.send_fwd = dist.isend(S.x[2 * n], self._peer(1), group=self.fwd_group)
            else:
                if not lay.last:
                    comms.record_external("recv", self.M * self.config.n_embd, act_bytes)
                    dist.irecv(self.dres, self._peer(1), group=self.bwd_group).wait()
                self._backward(S, idx, acc=not first_bwd)
                first_bwd = False
                if not lay.first:
                    if S.send_bwd is not None:
                        S.send_bwd.wait()
                    S.dx_out.copy_(self.dres)
                    comms.record_external("send", self.M * self.config.n_embd, act_bytes)
                    S.send_bwd = dist.isend(S.dx_out, self._peer(-1), group=self.bwd_group)
        for S in self.slots:
            for h in (S.send_fwd, S.send_bwd):
                if h is not None:
                    h.wait()
            S.send_fwd = S.send_bwd = None
        if self._reducer is not None:
            n_el = self.lay.total
            comms.record_external("all_reduce", n_el, n_el * 4)
            self._reducer.all_reduce(n_el, scale=1.0 / self.dp)
        self.optimizer_step()
        return self.loss_sum[0] / self.m

    def loss_of_last_step(self) -> Optional[float]:
        """Host value of the last step's mean loss on the last stage, else None."""
        return float(self.loss_sum[0]) / self.m if self.lay.last else None

    def optimizer_step(self) -> None:
        o = self.optim
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
            N.grad_sumsq(self.grad, self._norm_ws, self.sumsq)
            comms.record_external("all_reduce", 1, 4)
            dist.all_reduce(self.sumsq, group=self.group)
            N.clip_coef(self.sumsq, o.grad_clip, self.clip, self.grad_norm)
            clip = self.clip
        N.adamw_step(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.shadow, 0, self.hp,
                     clip, decay_ranges=self.decay)

    def check(self) -> None:
        N.check_errors(self.device)

    def state_dict(self) -> dict:
        """This stage's parameters (fp32 master, reference names; the last
        stage's untied ``lm_head.weight`` included)."""
        return {name: self.lay.view(self.master, name).clone() for name in self.lay.specs}

    def optimizer_state(self) -> dict:
        """AdamW moments of this stage (reference names) and the step count."""
        return {"step": self.step_count,
                "exp_avg": {n: self.lay.view(self.exp_avg, n).clone() for n in self.lay.specs},
                "exp_avg_sq": {n: self.lay.view(self.exp_avg_sq, n).clone() for n in self.lay.specs}}

    @torch.no_grad()
    def load_state_dict(self, sd: dict, optim: Optional[dict] = None) -> None:
        """Load this stage's tensors from a dict keyed by reference names (a
        full-model state dict works: only this stage's names are read; a
        missing ``lm_head.weight`` is taken from ``wte.weight``)."""
        for name in self.lay.specs:
            src = sd.get(name)
            if src is None and name == "lm_head.weight":
                src = sd["wte.weight"]
            self.lay.view(self.master, name).copy_(src)
        self.shadow.copy_(self.master)
        if optim is not None:
            self.step_count = int(optim["step"])
            for n in self.lay.specs:
                self.lay.view(self.exp_avg, n).copy_(optim["exp_avg"][n])
                self.lay.view(self.exp_avg_sq, n).copy_(optim["exp_avg_sq"][n])

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        if self._reducer is not None:
            self._reducer.close()
            self._reducer = None


class PipelineMesh:
    """Process groups of a pp x cp mesh (global rank = stage * cp + c): the
    pipeline line of this rank with one extra communicator per transfer
    direction, and the context-parallel group of its stage."""

    def __init__(self, pp: int, cp: int, stage: int, cp_rank: int, pp_group, fwd_group, bwd_group,
                 cp_group) -> None:
        self.pp, self.cp, self.stage, self.cp_rank = pp, cp, stage, cp_rank
        self.pp_group, self.fwd_group, self.bwd_group, self.cp_group = pp_group, fwd_group, bwd_group, cp_group


def make_mesh(pp: int, cp: int = 1) -> PipelineMesh:
    """Create the mesh's groups. Collective over the default group: every
    rank calls it with the same arguments (``pp * cp`` = world size)."""
    from gpt2_harness_b200.parallel.mesh import Mesh

    mesh = Mesh({"pp": pp, "cp": cp})
    # the activation and gradient communicators of every pipeline line, made
    # in the same order on every rank
    p2p = None
    for c in range(cp):
        ranks = [mesh.rank_of({"pp": s, "cp": c}) for s in range(pp)]
        gs = (dist.new_group(ranks), dist.new_group(ranks))
        if c == mesh.coord("cp"):
            p2p = gs
    return PipelineMesh(pp, cp, mesh.coord("pp"), mesh.coord("cp"), mesh.group("pp"), p2p[0], p2p[1],
                        mesh.group("cp") if cp > 1 else None)
