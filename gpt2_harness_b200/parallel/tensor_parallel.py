"""Megatron tensor parallelism, with sequence parallelism and a vocab-parallel
head.

Reference semantics (src/transformer_internals/parallel/tensor_parallel.py:
69-425): conjugate operators f (identity forward / all-reduce backward) and g
(all-reduce forward / identity backward); column-parallel c_attn (sliced per
q/k/v SECTION so each rank gets whole heads) and c_fc; row-parallel c_proj
(bias added once, after the reduction); replicated pre-LN LayerNorms; 4
all-reduces of B*T*C per block per step ("parity mode").

Added for the B200 configs (absent in the reference):

* ``sequence_parallel=True``: activations outside the tensor-parallel region
  are sharded along the sequence. The f/g pair becomes all-gather (forward)
  / reduce-scatter (backward) before a column-parallel GEMM and reduce-scatter
  (forward) / all-gather (backward) after a row-parallel GEMM. Per block and
  step that is 8 collectives of B*T*C elements in the counting convention
  (all-gather charged its output, reduce-scatter its input): twice the raw
  payload of parity mode for the same ring wire bytes, 2(p-1)/p*S either way.
  :func:`tp_payload_bytes` gives both and the "AR-equivalent" figure.
  LayerNorm parameter gradients become partial (each rank saw T/p tokens) and
  are all-reduced across the group.
* :class:`VocabParallelEmbedding` and :func:`vocab_parallel_cross_entropy`:
  the token table (padded to a multiple of 64*p rows, 50304 for GPT-2) is
  row-sharded; embedding lookups are masked and summed with one all-reduce;
  the loss needs three (B*T,)-vector all-reduces (row max, sum of exp, target
  logit) and never materialises the full-vocabulary logits on any rank.
"""

from __future__ import annotations

import math
from typing import Any, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.gpt import Block, gelu_tanh
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.common import current_device, identical_block, parallel_config

__all__ = [
    "CopyToTensorParallel",
    "ReduceFromTensorParallel",
    "GatherFromSequenceParallel",
    "ReduceScatterToSequenceParallel",
    "ColumnParallelLinear",
    "RowParallelLinear",
    "TensorParallelBlock",
    "VocabParallelEmbedding",
    "vocab_parallel_cross_entropy",
    "padded_vocab",
    "tp_payload_bytes",
    "tp_equivalence_worker",
    "vocab_parallel_worker",
]


# ------------------------------------------------------------- conjugates --
class CopyToTensorParallel(torch.autograd.Function):
    """f: identity forward, all-reduce backward."""

    @staticmethod
    def forward(ctx, x, group=None):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        comms.all_reduce(g, group=ctx.group)
        return g, None


class ReduceFromTensorParallel(torch.autograd.Function):
    """g: all-reduce forward, identity backward."""

    @staticmethod
    def forward(ctx, x, group=None):
        y = x.contiguous().clone()
        comms.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


def _seq_gather(x: torch.Tensor, world: int, group) -> torch.Tensor:
    """[B, T/p, C] shards -> [B, T, C] (rank order along the sequence)."""
    B, tp, C = x.shape
    out = torch.empty(world * B * tp * C, dtype=x.dtype, device=x.device)
    comms.all_gather_into(out, x.contiguous().view(-1), group=group)
    return out.view(world, B, tp, C).permute(1, 0, 2, 3).reshape(B, world * tp, C)


def _seq_reduce_scatter(x: torch.Tensor, world: int, group) -> torch.Tensor:
    """[B, T, C] partial sums -> this rank's [B, T/p, C] slice of the sum."""
    B, T, C = x.shape
    tp = T // world
    src = x.reshape(B, world, tp, C).permute(1, 0, 2, 3).contiguous().view(-1)
    out = torch.empty(B * tp * C, dtype=x.dtype, device=x.device)
    comms.reduce_scatter_into(out, src, group=group)
    return out.view(B, tp, C)


class GatherFromSequenceParallel(torch.autograd.Function):
    """SP entry to a column-parallel GEMM: all-gather forward, reduce-scatter backward."""

    @staticmethod
    def forward(ctx, x, world, group=None):
        ctx.world, ctx.group = world, group
        return _seq_gather(x, world, group)

    @staticmethod
    def backward(ctx, g):
        return _seq_reduce_scatter(g, ctx.world, ctx.group), None, None


class ReduceScatterToSequenceParallel(torch.autograd.Function):
    """SP exit of a row-parallel GEMM: reduce-scatter forward, all-gather backward."""

    @staticmethod
    def forward(ctx, x, world, group=None):
        ctx.world, ctx.group = world, group
        return _seq_reduce_scatter(x, world, group)

    @staticmethod
    def backward(ctx, g):
        return _seq_gather(g, ctx.world, ctx.group), None, None


# ------------------------------------------------------------- linear layers --
class ColumnParallelLinear(nn.Module):
    """Output features split: rank r keeps rows [r*out/p, (r+1)*out/p)."""

    def __init__(self, linear: nn.Linear, rank: int, world_size: int, group=None) -> None:
        super().__init__()
        out_f = linear.out_features
        if out_f % world_size:
            raise ValueError(f"out_features={out_f} not divisible by {world_size}")
        per = out_f // world_size
        self.weight = nn.Parameter(linear.weight.data[rank * per:(rank + 1) * per].clone())
        self.bias = (nn.Parameter(linear.bias.data[rank * per:(rank + 1) * per].clone())
                     if linear.bias is not None else None)
        self.group = group

    def forward(self, x: torch.Tensor, already_gathered: bool = False) -> torch.Tensor:
        if not already_gathered:
            x = CopyToTensorParallel.apply(x, self.group)
        return F.linear(x, self.weight, self.bias)


class RowParallelLinear(nn.Module):
    """Input features split; partial outputs summed across ranks, bias added
    once after the sum (adding it per rank would count it p times)."""

    def __init__(self, linear: nn.Linear, rank: int, world_size: int, group=None,
                 sequence_parallel: bool = False) -> None:
        super().__init__()
        in_f = linear.in_features
        if in_f % world_size:
            raise ValueError(f"in_features={in_f} not divisible by {world_size}")
        per = in_f // world_size
        self.weight = nn.Parameter(linear.weight.data[:, rank * per:(rank + 1) * per].clone())
        self.bias = nn.Parameter(linear.bias.data.clone()) if linear.bias is not None else None
        self.group, self.world = group, world_size
        self.sequence_parallel = sequence_parallel

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.weight)
        if self.sequence_parallel:
            y = ReduceScatterToSequenceParallel.apply(y, self.world, self.group)
        else:
            y = ReduceFromTensorParallel.apply(y, self.group)
        return y + self.bias if self.bias is not None else y


def _section_rows(t: torch.Tensor, sizes, rank: int, local) -> torch.Tensor:
    parts = t.split(list(sizes), dim=0)
    return torch.cat([p[rank * n:(rank + 1) * n] for p, n in zip(parts, local)], dim=0)


class TensorParallelBlock(nn.Module):
    """A pre-LN GPT-2 block with head-parallel attention and a split MLP.

    The fused c_attn weight [q; k; v] is sliced per section so every rank owns
    whole heads. With ``sequence_parallel`` the block's input/output are the
    rank's sequence shard [B, T/p, C]; otherwise they are replicated [B, T, C].
    """

    def __init__(self, block: Block, rank: int, world_size: int, group=None,
                 sequence_parallel: bool = False) -> None:
        super().__init__()
        cfg: GPTConfig = block.config
        if cfg.norm_position != "pre":
            raise ValueError("TensorParallelBlock implements the pre-LN block only")
        if cfg.n_head % world_size or cfg.kv_heads % world_size:
            raise ValueError(f"n_head={cfg.n_head} and kv_heads={cfg.kv_heads} must be divisible "
                             f"by world_size={world_size}")
        self.config, self.rank, self.world_size, self.group = cfg, rank, world_size, group
        self.sequence_parallel = sequence_parallel
        self.nh = cfg.n_head // world_size
        self.nkv = cfg.kv_heads // world_size
        self.hd = cfg.head_dim
        self.ln_1 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_epsilon)
        self.ln_2 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_epsilon)
        self.ln_1.load_state_dict(block.ln_1.state_dict())
        self.ln_2.load_state_dict(block.ln_2.state_dict())
        kv = cfg.kv_heads * cfg.head_dim
        sizes = (cfg.n_embd, kv, kv)
        local = (self.nh * self.hd, self.nkv * self.hd, self.nkv * self.hd)
        ca = block.attn.c_attn
        self.c_attn_weight = nn.Parameter(_section_rows(ca.weight.data, sizes, rank, local).clone())
        self.c_attn_bias = (nn.Parameter(_section_rows(ca.bias.data, sizes, rank, local).clone())
                            if ca.bias is not None else None)
        self.attn_proj = RowParallelLinear(block.attn.c_proj, rank, world_size, group, sequence_parallel)
        self.mlp_fc = ColumnParallelLinear(block.mlp.c_fc, rank, world_size, group)
        self.mlp_proj = RowParallelLinear(block.mlp.c_proj, rank, world_size, group, sequence_parallel)

    def _enter(self, h: torch.Tensor) -> torch.Tensor:
        if self.sequence_parallel:
            return GatherFromSequenceParallel.apply(h, self.world_size, self.group)
        return CopyToTensorParallel.apply(h, self.group)

    def _attention(self, h: torch.Tensor) -> torch.Tensor:
        x = self._enter(h)
        b, t, _ = x.shape
        qkv = F.linear(x, self.c_attn_weight, self.c_attn_bias)
        qd, kd = self.nh * self.hd, self.nkv * self.hd
        q, k, v = qkv.split([qd, kd, kd], dim=2)
        q = q.view(b, t, self.nh, self.hd).transpose(1, 2)
        k = k.view(b, t, self.nkv, self.hd).transpose(1, 2)
        v = v.view(b, t, self.nkv, self.hd).transpose(1, 2)
        if self.nkv != self.nh:
            k = k.repeat_interleave(self.nh // self.nkv, dim=1)
            v = v.repeat_interleave(self.nh // self.nkv, dim=1)
        att = (q @ k.transpose(-2, -1)) / math.sqrt(self.hd)
        mask = torch.ones(t, t, dtype=torch.bool, device=x.device).tril()
        att = F.softmax(att.masked_fill(~mask.view(1, 1, t, t), float("-inf")), dim=-1)
        y = (att @ v).transpose(1, 2).contiguous().view(b, t, qd)
        return self.attn_proj(y)

    def _act(self, h: torch.Tensor) -> torch.Tensor:
        a = self.config.activation
        return gelu_tanh(h) if a == "gelu_tanh" else (F.gelu(h) if a == "gelu_exact" else F.relu(h))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self._attention(self.ln_1(x))
        h = self.mlp_fc(self._enter(self.ln_2(x)), already_gathered=True)
        return x + self.mlp_proj(self._act(h))

    def replicated_parameters(self) -> list:
        """Parameters every rank holds in full: the LayerNorms and the biases
        of the row-parallel projections (added after the reduction)."""
        out = [self.ln_1.weight, self.ln_1.bias, self.ln_2.weight, self.ln_2.bias]
        out += [p for p in (self.attn_proj.bias, self.mlp_proj.bias) if p is not None]
        return out

    def allreduce_replicated_grads(self) -> None:
        """Under SP every replicated parameter acts on this rank's T/p tokens
        only, so its gradient is partial: sum it across the group."""
        for p in self.replicated_parameters():
            if p.grad is not None:
                comms.all_reduce(p.grad, group=self.group)


# ----------------------------------------------------------- vocab parallel --
def padded_vocab(vocab: int, world_size: int, multiple: int = 64, per_rank: int = 16) -> int:
    """Vocabulary rounded up to a multiple of `multiple` that also splits into
    equal per-rank blocks of a multiple of `per_rank` rows: 50257 -> 50304
    for p in 1, 2, 4 and 8 (the padded GPT-2 vocabulary)."""
    step = math.lcm(multiple, per_rank * world_size)
    return (vocab + step - 1) // step * step


class _MaskedEmbeddingSum(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local, group):
        out = local.contiguous().clone()
        comms.all_reduce(out, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        return g, None


class VocabParallelEmbedding(nn.Module):
    """Token table row-sharded over the padded vocabulary."""

    def __init__(self, weight: torch.Tensor, vocab: int, rank: int, world_size: int, group=None) -> None:
        super().__init__()
        vp = padded_vocab(vocab, world_size)
        per = vp // world_size
        full = torch.zeros(vp, weight.shape[1], dtype=weight.dtype, device=weight.device)
        full[:vocab] = weight.data
        self.weight = nn.Parameter(full[rank * per:(rank + 1) * per].clone())
        self.vocab, self.vp, self.per = vocab, vp, per
        self.start = rank * per
        self.group = group

    def forward(self, idx: torch.Tensor) -> torch.Tensor:
        local = idx - self.start
        inside = (local >= 0) & (local < self.per)
        emb = F.embedding(local.clamp(0, self.per - 1), self.weight) * inside.unsqueeze(-1)
        return _MaskedEmbeddingSum.apply(emb, self.group)


class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, start, vocab, group):
        # logits: [N, per] this rank's vocab slice; padded columns >= vocab masked
        n, per = logits.shape
        cols = torch.arange(start, start + per, device=logits.device)
        logits = logits.float().masked_fill((cols >= vocab).unsqueeze(0), float("-inf"))
        mx = logits.max(dim=1).values
        comms.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(logits - mx.unsqueeze(1))
        se = ex.sum(dim=1)
        comms.all_reduce(se, group=group)
        local_t = targets - start
        inside = (local_t >= 0) & (local_t < per) & (targets != -100)
        tl = torch.zeros(n, device=logits.device, dtype=torch.float32)
        rows = torch.nonzero(inside).squeeze(1)
        tl[rows] = logits[rows, local_t[rows]]
        comms.all_reduce(tl, group=group)
        valid = targets != -100
        count = valid.sum().clamp(min=1).to(torch.float32)
        loss_rows = (torch.log(se) + mx - tl) * valid
        ctx.save_for_backward(ex, se, local_t, inside, valid, count)
        return loss_rows.sum() / count

    @staticmethod
    def backward(ctx, g):
        ex, se, local_t, inside, valid, count = ctx.saved_tensors
        grad = ex / se.unsqueeze(1)
        rows = torch.nonzero(inside).squeeze(1)
        grad[rows, local_t[rows]] -= 1.0
        grad = grad * (valid.unsqueeze(1).to(grad.dtype) * (g / count))
        return grad, None, None, None, None


def vocab_parallel_cross_entropy(local_logits: torch.Tensor, targets: torch.Tensor, start: int,
                                 vocab: int, group=None) -> torch.Tensor:
    """Mean cross-entropy (ignore_index -100) from vocab-sharded logits."""
    return _VocabParallelCE.apply(local_logits.reshape(-1, local_logits.shape[-1]),
                                  targets.reshape(-1), start, vocab, group)


# ---------------------------------------------------------------- closed forms --
def tp_payload_bytes(B: int, T: int, C: int, L: int, sequence_parallel: bool = False,
                     elem_bytes: int = 4) -> dict[str, int]:
    """Per-rank payload per step of the block collectives. Parity mode: 4
    all-reduces of B*T*C per block; SP: 8 gathers/scatters of B*T*C per block
    (2x raw payload, same ring wire bytes)."""
    per = B * T * C * elem_bytes
    raw = (8 if sequence_parallel else 4) * per * L
    return {"raw": raw, "allreduce_equivalent": 4 * per * L}


# ------------------------------------------------------------------ workers --
def _grad_errors(tp: TensorParallelBlock, ref: Block, rank: int, world: int) -> dict[str, float]:
    cfg = ref.config
    per = cfg.n_embd // world
    kv = cfg.kv_heads * cfg.head_dim
    sizes = (cfg.n_embd, kv, kv)
    local = ((cfg.n_head // world) * cfg.head_dim, (cfg.kv_heads // world) * cfg.head_dim,
             (cfg.kv_heads // world) * cfg.head_dim)
    want_attn = _section_rows(ref.attn.c_attn.weight.grad, sizes, rank, local)

    def err(a, b):
        return float((a - b).abs().max())

    return {
        "c_attn_weight": err(tp.c_attn_weight.grad, want_attn),
        "attn_c_proj_weight": err(tp.attn_proj.weight.grad, ref.attn.c_proj.weight.grad[:, rank * per:(rank + 1) * per]),
        "mlp_c_fc_weight": err(tp.mlp_fc.weight.grad, ref.mlp.c_fc.weight.grad[rank * 4 * per:(rank + 1) * 4 * per]),
        "mlp_c_proj_weight": err(tp.mlp_proj.weight.grad, ref.mlp.c_proj.weight.grad[:, rank * 4 * per:(rank + 1) * 4 * per]),
        "ln_1_weight": err(tp.ln_1.weight.grad, ref.ln_1.weight.grad),
        "ln_2_weight": err(tp.ln_2.weight.grad, ref.ln_2.weight.grad),
        "attn_c_proj_bias": err(tp.attn_proj.bias.grad, ref.attn.c_proj.bias.grad),
        "mlp_c_proj_bias": err(tp.mlp_proj.bias.grad, ref.mlp.c_proj.bias.grad),
    }


def tp_equivalence_worker(rank: int, world_size: int, batch: int = 4, seq: int = 12,
                          sequence_parallel: bool = False,
                          config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """A TP block vs the unsharded block: forward output, input gradient,
    replicated LayerNorm gradients and this rank's weight-gradient slices."""
    cfg = parallel_config(**(config_kwargs or {}))
    ref = identical_block(cfg, seed=7).train()
    tp = TensorParallelBlock(ref, rank, world_size, sequence_parallel=sequence_parallel)
    torch.manual_seed(99)
    x = torch.randn(batch, seq, cfg.n_embd).to(current_device())
    x_ref = x.clone().requires_grad_(True)
    ref_out, _ = ref(x_ref)
    if sequence_parallel:
        tp_seq = seq // world_size
        x_tp = x[:, rank * tp_seq:(rank + 1) * tp_seq].clone().requires_grad_(True)
    else:
        x_tp = x.clone().requires_grad_(True)
    tp_out = tp(x_tp)
    want = ref_out[:, rank * (seq // world_size):(rank + 1) * (seq // world_size)] if sequence_parallel else ref_out
    fwd_err = float((tp_out - want).detach().abs().max())
    torch.manual_seed(100)
    gout = torch.randn(ref_out.shape, dtype=ref_out.dtype).to(ref_out.device)
    ref_out.backward(gout)
    gslice = gout[:, rank * (seq // world_size):(rank + 1) * (seq // world_size)] if sequence_parallel else gout
    tp_out.backward(gslice.clone())
    if sequence_parallel:
        with comms.counter_scope(world_size):  # LN grad sync counted separately
            tp.allreduce_replicated_grads()
        want_gx = x_ref.grad[:, rank * (seq // world_size):(rank + 1) * (seq // world_size)]
    else:
        want_gx = x_ref.grad
    errors = _grad_errors(tp, ref, rank, world_size)
    errors["input"] = float((x_tp.grad - want_gx).abs().max())
    comms.get_counter().steps += 1
    return {"rank": rank, "sequence_parallel": sequence_parallel, "forward_error": fwd_err,
            "grad_errors": errors, "max_grad_error": max(errors.values()),
            "closed_form": tp_payload_bytes(batch, seq, cfg.n_embd, 1, sequence_parallel)}


def vocab_parallel_worker(rank: int, world_size: int, batch: int = 4, seq: int = 16,
                          config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """Vocab-parallel embedding + cross-entropy vs the full-vocabulary ones
    (tied table; padded vocab), forward loss and table gradient."""
    cfg = parallel_config(**(config_kwargs or {}))
    torch.manual_seed(3)
    dev = current_device()
    wte = (torch.randn(cfg.vocab_size, cfg.n_embd) * 0.02).to(dev)
    idx = torch.randint(0, cfg.vocab_size, (batch, seq)).to(dev)
    tgt = torch.randint(0, cfg.vocab_size, (batch, seq)).to(dev)
    tgt[0, :3] = -100
    ref_w = wte.clone().requires_grad_(True)
    h_ref = F.embedding(idx, ref_w)
    logits = h_ref @ ref_w.t()
    ref_loss = F.cross_entropy(logits.view(-1, cfg.vocab_size), tgt.view(-1), ignore_index=-100)
    ref_loss.backward()
    emb = VocabParallelEmbedding(wte, cfg.vocab_size, rank, world_size)
    h = emb(idx)
    # f before the vocab-parallel head: each rank's dL/dh covers only its
    # vocabulary slice, so the head input's gradient is all-reduced.
    local_logits = CopyToTensorParallel.apply(h, None) @ emb.weight.t()
    loss = vocab_parallel_cross_entropy(local_logits, tgt, emb.start, cfg.vocab_size)
    loss.backward()
    comms.get_counter().steps += 1
    want = torch.zeros(emb.vp, cfg.n_embd, device=dev)
    want[:cfg.vocab_size] = ref_w.grad
    gerr = float((emb.weight.grad - want[emb.start:emb.start + emb.per]).abs().max())
    return {"rank": rank, "loss_error": abs(float(loss) - float(ref_loss)), "grad_error": gerr,
            "padded_vocab": emb.vp, "tokens": batch * seq}
