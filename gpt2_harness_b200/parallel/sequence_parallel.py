"""Context parallelism: attention over a sequence sharded across ranks.

Module name kept from the reference (src/transformer_internals/parallel/
sequence_parallel.py:60-311), whose two paths this reproduces:

* **all-gather KV** (:func:`all_gather_kv_attention`): each rank keeps its
  T/p queries, all-gathers K and V along the sequence, and attends with the
  causal mask sliced at absolute positions rank*T/p. The gather is
  differentiable: all-gather forward, REDUCE-SCATTER backward (every rank
  produces a gradient for every key position; slicing would drop (p-1)/p of
  it). The c_attn weight gradient is a partial sum per rank and is all-reduced.
* **ring attention** (:func:`ring_attention`): K/V blocks rotate p-1 hops with
  an online softmax (running max / denominator / numerator); blocks entirely
  in the future are skipped, the diagonal block is triangular-masked. Unlike
  the reference (forward only) this one is differentiable: the backward runs a
  second ring in which each K/V block travels with its accumulating dK/dV and
  returns home after p hops, recomputing probabilities from the saved
  log-sum-exp.

Closed forms (fp32, per rank per step): all-gather KV 2*4*B*T*C charged as
gather outputs (and the same again as reduce-scatter inputs in backward);
ring forward 2*(p-1)/p*4*B*T*C of sends.
"""

from __future__ import annotations

import math
from typing import Any, Optional

import torch
import torch.nn.functional as F

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.common import current_device, identical_block, parallel_config

__all__ = [
    "gather_sequence",
    "all_gather_kv_attention",
    "ring_attention",
    "cp_payload_bytes",
    "sequence_parallel_worker",
]


class _GatherSequence(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim: int, world_size: int, group=None):
        ctx.dim, ctx.world, ctx.group = dim, world_size, group
        moved = x.movedim(dim, 0).contiguous()
        out = torch.empty((moved.shape[0] * world_size, *moved.shape[1:]), dtype=moved.dtype,
                          device=moved.device)
        comms.all_gather_into(out, moved, group=group)
        return out.movedim(0, dim).contiguous()

    @staticmethod
    def backward(ctx, g):
        moved = g.movedim(ctx.dim, 0).contiguous()
        shard = torch.empty((moved.shape[0] // ctx.world, *moved.shape[1:]), dtype=moved.dtype,
                            device=moved.device)
        comms.reduce_scatter_into(shard, moved, group=ctx.group)
        return shard.movedim(0, ctx.dim).contiguous(), None, None, None


def gather_sequence(x: torch.Tensor, dim: int, world_size: int, group=None) -> torch.Tensor:
    """All-gather along `dim` (rank order); reduce-scatter in backward."""
    return _GatherSequence.apply(x, dim, world_size, group)


def all_gather_kv_attention(q_local, k_local, v_local, rank: int, world_size: int,
                            causal_mask: Optional[torch.Tensor] = None, group=None) -> torch.Tensor:
    """This rank's rows of causal attention, from gathered K/V.
    q/k/v_local: (B, H, T/p, d). Returns (B, H, T/p, d)."""
    tl, d = q_local.shape[-2], q_local.shape[-1]
    k = gather_sequence(k_local, 2, world_size, group)
    v = gather_sequence(v_local, 2, world_size, group)
    T = k.shape[-2]
    if causal_mask is None:
        causal_mask = torch.ones(T, T, dtype=torch.bool, device=q_local.device).tril()
    mask = causal_mask[rank * tl:(rank + 1) * tl, :T]
    att = (q_local @ k.transpose(-2, -1)) / math.sqrt(d)
    att = att.masked_fill(~mask.view(1, 1, tl, T), float("-inf"))
    return F.softmax(att, dim=-1) @ v


def _rotate(tensors, rank: int, world: int, group=None):
    """Send tensors to rank+1 and receive the same shapes from rank-1."""
    dst, src = (rank + 1) % world, (rank - 1) % world
    handles = [comms.isend(t, dst=dst, group=group) for t in tensors]
    got = []
    for t in tensors:
        buf = torch.empty_like(t)
        comms.recv(buf, src=src, group=group)
        got.append(buf)
    for h in handles:
        h.wait()
    return got


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, rank: int, world: int, group=None):
        B, H, tl, d = q.shape
        scale = 1.0 / math.sqrt(d)
        m = torch.full((B, H, tl, 1), float("-inf"), device=q.device, dtype=q.dtype)
        l = torch.zeros((B, H, tl, 1), device=q.device, dtype=q.dtype)
        acc = torch.zeros_like(q)
        kc, vc = k.contiguous(), v.contiguous()
        blk = rank
        tri = torch.ones(tl, tl, dtype=torch.bool, device=q.device).tril().view(1, 1, tl, tl)
        for step in range(world):
            if blk <= rank:
                s = (q @ kc.transpose(-2, -1)) * scale
                if blk == rank:
                    s = s.masked_fill(~tri, float("-inf"))
                mn = torch.maximum(m, s.amax(dim=-1, keepdim=True))
                r = torch.exp(m - mn)
                w = torch.exp(s - mn)
                l = l * r + w.sum(dim=-1, keepdim=True)
                acc = acc * r + w @ vc
                m = mn
            if step < world - 1:
                kc, vc = _rotate([kc, vc], rank, world, group)
                blk = (blk - 1) % world
        out = acc / l
        lse = m + torch.log(l)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.rank, ctx.world, ctx.group, ctx.scale = rank, world, group, scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        rank, world, group, scale = ctx.rank, ctx.world, ctx.group, ctx.scale
        tl = q.shape[-2]
        delta = (dout * out).sum(dim=-1, keepdim=True)
        dq = torch.zeros_like(q)
        kc, vc = k.contiguous(), v.contiguous()
        dkc, dvc = torch.zeros_like(kc), torch.zeros_like(vc)
        blk = rank
        tri = torch.ones(tl, tl, dtype=torch.bool, device=q.device).tril().view(1, 1, tl, tl)
        for step in range(world):
            if blk <= rank:
                s = (q @ kc.transpose(-2, -1)) * scale
                if blk == rank:
                    s = s.masked_fill(~tri, float("-inf"))
                p = torch.exp(s - lse)
                dvc = dvc + p.transpose(-2, -1) @ dout
                dp = dout @ vc.transpose(-2, -1)
                ds = p * (dp - delta) * scale
                dq = dq + ds @ kc
                dkc = dkc + ds.transpose(-2, -1) @ q
            # every block (with its gradient) moves on; after `world` hops it is home
            if step < world - 1:
                kc, vc, dkc, dvc = _rotate([kc, vc, dkc, dvc], rank, world, group)
            else:
                dkc, dvc = _rotate([dkc, dvc], rank, world, group)
            blk = (blk - 1) % world
        return dq, dkc, dvc, None, None, None


def ring_attention(q_local, k_local, v_local, rank: int, world_size: int, group=None) -> torch.Tensor:
    """Causal ring attention over (B, H, T/p, d) shards (differentiable)."""
    return _RingAttention.apply(q_local, k_local, v_local, rank, world_size, group)


def cp_payload_bytes(B: int, T: int, C: int, world: int, elem_bytes: int = 4) -> dict[str, float]:
    """Closed forms per rank per attention layer and step."""
    fwd = 2 * (world - 1) / world * elem_bytes * B * T * C
    # backward: K, V travel p-1 hops again; dK, dV travel p hops (back to their owner)
    bwd = (2 * (world - 1) + 2 * world) / world * elem_bytes * B * T * C
    return {"all_gather_kv_forward": 2 * elem_bytes * B * T * C,
            "all_gather_kv_backward_reduce_scatter": 2 * elem_bytes * B * T * C,
            "ring_forward_send": fwd, "ring_backward_send": bwd, "ring_send_total": fwd + bwd}


def _project(attn, x):
    b, t, _ = x.shape
    q, k, v = attn.c_attn(x).split([attn.n_embd, attn.kv_dim, attn.kv_dim], dim=2)
    q = q.view(b, t, attn.n_head, attn.head_dim).transpose(1, 2)
    k = k.view(b, t, attn.n_kv_head, attn.head_dim).transpose(1, 2)
    v = v.view(b, t, attn.n_kv_head, attn.head_dim).transpose(1, 2)
    return q, k, v


def sequence_parallel_worker(rank: int, world_size: int, batch: int = 2, seq: int = 32,
                             path: str = "all_gather", config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """One CP path vs the full-sequence attention of the oracle: forward rows,
    this rank's input gradient and the (all-reduced) c_attn weight gradient."""
    cfg = parallel_config(**(config_kwargs or {}))
    if seq % world_size:
        raise ValueError(f"seq={seq} must be divisible by world_size={world_size}")
    tl = seq // world_size
    ref_attn = identical_block(cfg, seed=11).attn
    cp_attn = identical_block(cfg, seed=11).attn
    torch.manual_seed(21)
    x = torch.randn(batch, seq, cfg.n_embd).to(current_device())
    x_ref = x.clone().requires_grad_(True)
    x_loc = x[:, rank * tl:(rank + 1) * tl].clone().requires_grad_(True)
    qr, kr, vr = _project(ref_attn, x_ref)
    mask = ref_attn.causal_mask[:seq, :seq]
    att = (qr @ kr.transpose(-2, -1)) / math.sqrt(cfg.head_dim)
    ref_out = F.softmax(att.masked_fill(~mask.view(1, 1, seq, seq), float("-inf")), dim=-1) @ vr
    ref_slice = ref_out[:, :, rank * tl:(rank + 1) * tl]
    ql, kl, vl = _project(cp_attn, x_loc)
    if path == "all_gather":
        out = all_gather_kv_attention(ql, kl, vl, rank, world_size, ref_attn.causal_mask)
    elif path == "ring":
        out = ring_attention(ql, kl, vl, rank, world_size)
    else:
        raise ValueError(f"unknown path {path!r}")
    fwd_err = float((out - ref_slice).detach().abs().max())
    torch.manual_seed(22)
    g = torch.randn(ref_out.shape).to(ref_out.device)
    ref_out.backward(g)
    out.backward(g[:, :, rank * tl:(rank + 1) * tl].contiguous())
    in_err = float((x_loc.grad - x_ref.grad[:, rank * tl:(rank + 1) * tl]).abs().max())
    wg = cp_attn.c_attn.weight.grad.clone()
    with comms.counter_scope(world_size):  # DP-style weight-grad sync, counted apart
        comms.all_reduce(wg)
    w_err = float((wg - ref_attn.c_attn.weight.grad).abs().max())
    comms.get_counter().steps += 1
    return {"rank": rank, "path": path, "forward_error": fwd_err, "input_grad_error": in_err,
            "weight_grad_error": w_err, "weight_grad_scale": float(ref_attn.c_attn.weight.grad.abs().max()),
            "closed_form": cp_payload_bytes(batch, seq, cfg.n_embd, world_size)}
