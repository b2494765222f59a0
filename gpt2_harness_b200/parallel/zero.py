"""ZeRO-1/2 sharded AdamW and ZeRO-3 (FSDP-style) parameter sharding.

Reference semantics: src/transformer_internals/parallel/zero.py:118-1161.

* Flat parameter vector padded to a multiple of p; rank r owns slice r.
* ZeRO-1: all-reduce the flat gradient, keep the owned slice; ZeRO-2:
  reduce-scatter it. Divide by p, AdamW on the slice (torch single-tensor
  order, per-element decay mask so a shard boundary may cut a tensor),
  all-gather the updated slices. Optional fp32 master shard when the gathered
  parameters are narrower (``param_dtype``).
* Sharded global-norm clipping: ZeRO-1 already holds the full averaged
  gradient (no extra collective); ZeRO-2/3 sum the owned squares with one
  4-byte all-reduce, and ZeRO-3's replicated root is added AFTER it (inside it
  would be counted p times).
* ZeRO-3: one flat shard per transformer block. Forward all-gathers the unit,
  runs it with torch.func.functional_call under no_grad, frees it; backward
  all-gathers again, recomputes, backpropagates, reduce-scatters the gradient
  and divides by p. Root parameters (wte, wpe, ln_f) stay replicated and are
  all-reduced per tensor.

Closed form at p ranks (fp32 wire): ZeRO-1 4N + 4N_pad, ZeRO-2 4N_pad + 4N_pad
(+4 B with clipping), ZeRO-3 sum_u 12 P_u + 4 N_root per step.
"""

from __future__ import annotations

import math
from typing import Any, Optional, Sequence

import torch
import torch.nn as nn
from torch.func import functional_call

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.common import identical_batch, identical_model, parallel_config, state_bytes
from gpt2_harness_b200.parallel.data_parallel import average_gradients, local_shard
from gpt2_harness_b200.precision import reduce_dtype_of

__all__ = [
    "ShardedAdamW",
    "Zero3AdamW",
    "Zero3Model",
    "adamw_update_",
    "clip_coefficient",
    "decay_mask",
    "global_grad_norm",
    "padded_numel",
    "zero3_equivalence_worker",
    "zero3_payload_bytes",
    "zero_equivalence_worker",
]


def padded_numel(total: int, world_size: int) -> int:
    """`total` rounded up to a multiple of `world_size` (equal shards)."""
    return int(math.ceil(total / world_size) * world_size)


def _flatten(tensors: Sequence[torch.Tensor], numel: int) -> torch.Tensor:
    flat = torch.zeros(numel, dtype=tensors[0].dtype, device=tensors[0].device)
    off = 0
    for t in tensors:
        n = t.numel()
        flat[off:off + n] = t.reshape(-1)
        off += n
    return flat


def decay_mask(params: Sequence[torch.Tensor]) -> torch.Tensor:
    """Flat 0/1 per-element mask: 1 for rank>=2 tensors (matmul weights)."""
    return torch.cat([torch.full((p.numel(),), float(p.dim() >= 2), device=p.device) for p in params])


def adamw_update_(param, grad, exp_avg, exp_avg_sq, step: int, lr: float, beta1: float,
                  beta2: float, eps: float, weight_decay) -> None:
    """One decoupled AdamW update in place, in torch's _single_tensor_adamw
    order: decay, first/second moments, bias-corrected step."""
    if isinstance(weight_decay, torch.Tensor) or weight_decay != 0.0:
        param.mul_(1.0 - lr * weight_decay)
    exp_avg.lerp_(grad, 1.0 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1.0 - beta2)
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    denom = (exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
    param.addcdiv_(exp_avg, denom, value=-lr / bc1)


def global_grad_norm(shard_sumsq: torch.Tensor, replicated_sumsq=0.0, *, reduce: bool,
                     group: Any = None) -> torch.Tensor:
    """Global L2 norm from owned squares (summed across ranks when `reduce`)
    plus squares already identical on every rank (added after the reduce)."""
    total = shard_sumsq.clone().reshape(1)
    if reduce:
        comms.all_reduce(total, group=group)
    return (total + replicated_sumsq).sqrt().reshape(())


def clip_coefficient(total_norm: torch.Tensor, max_norm: float) -> torch.Tensor:
    """torch.nn.utils.clip_grad_norm_'s factor: min(1, max/(norm + 1e-6))."""
    return torch.clamp(max_norm / (total_norm + 1e-6), max=1.0)


class ShardedAdamW:
    """AdamW with sharded moments (stage 1) and sharded gradients (stage 2).

    Parameters stay replicated; rank r updates slice r of the flat padded
    parameter vector and the slices are all-gathered at the end of the step.
    """

    def __init__(self, params, rank: int, world_size: int, stage: int = 2, lr: float = 1e-3,
                 betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.1,
                 decay_matmul_only: bool = True, grad_clip: Optional[float] = None,
                 reduce_dtype=None, param_dtype=None, group: Any = None) -> None:
        if stage not in (1, 2):
            raise ValueError(f"ShardedAdamW implements stages 1 and 2, got {stage}")
        self.params = list(params)
        self.rank, self.world_size, self.stage = rank, world_size, stage
        self.lr, (self.beta1, self.beta2), self.eps = lr, betas, eps
        self.grad_clip = grad_clip
        self.reduce_dtype = reduce_dtype_of(reduce_dtype)
        self.param_dtype = reduce_dtype_of(param_dtype)
        self.group = group
        self.step_count = 0
        self.last_grad_norm = float("nan")
        self.numel = sum(p.numel() for p in self.params)
        self.padded = padded_numel(self.numel, world_size)
        self.shard_size = self.padded // world_size
        self.shard_start = rank * self.shard_size
        dev = self.params[0].device
        full = decay_mask(self.params) * weight_decay if decay_matmul_only else torch.full(
            (self.numel,), weight_decay, device=dev)
        padded = torch.zeros(self.padded, device=dev)
        padded[:self.numel] = full
        self.decay = padded[self.shard_start:self.shard_start + self.shard_size].clone()
        self.exp_avg = torch.zeros(self.shard_size, device=dev)
        self.exp_avg_sq = torch.zeros(self.shard_size, device=dev)
        self.grad_shard = torch.zeros(self.shard_size, device=dev)
        self.master_shard: Optional[torch.Tensor] = None
        if self.param_dtype != torch.float32:
            self.master_shard = _flatten([p.detach() for p in self.params], self.padded)[
                self.shard_start:self.shard_start + self.shard_size].clone().float()

    def state_bytes(self) -> int:
        """Adam moment bytes on this rank (the 8N/p of the ZeRO table)."""
        return state_bytes([self.exp_avg, self.exp_avg_sq])

    def resident_bytes(self) -> dict[str, int]:
        params = state_bytes(self.params)
        grads = (state_bytes([self.grad_shard]) if self.stage >= 2
                 else state_bytes([p.grad for p in self.params if p.grad is not None]))
        opt = self.state_bytes()
        decay = state_bytes([self.decay])
        master = state_bytes([self.master_shard]) if self.master_shard is not None else 0
        return {"params": params, "grads": grads, "optimizer": opt, "master_shard": master,
                "decay_mask": decay, "total": params + grads + opt + master + decay}

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None

    @torch.no_grad()
    def step(self) -> None:
        self.step_count += 1
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in self.params]
        flat = _flatten(grads, self.padded)
        lo, hi = self.shard_start, self.shard_start + self.shard_size
        if self.stage == 1:
            if self.reduce_dtype != flat.dtype:
                wire = flat.to(self.reduce_dtype)
                comms.all_reduce(wire, group=self.group)
                flat = wire.to(torch.float32)
            else:
                comms.all_reduce(flat, group=self.group)
            flat.div_(self.world_size)
            self.grad_shard.copy_(flat[lo:hi])
            local_sumsq = flat.pow(2).sum() if self.grad_clip is not None else None
            reduce_norm = False
        else:
            if self.reduce_dtype != flat.dtype:
                wire_in = flat.to(self.reduce_dtype)
                wire_out = torch.empty(self.shard_size, dtype=self.reduce_dtype, device=flat.device)
                comms.reduce_scatter_into(wire_out, wire_in, group=self.group)
                self.grad_shard.copy_(wire_out.to(torch.float32))
            else:
                comms.reduce_scatter_into(self.grad_shard, flat, group=self.group)
            self.grad_shard.div_(self.world_size)
            self.zero_grad()
            local_sumsq = self.grad_shard.pow(2).sum() if self.grad_clip is not None else None
            reduce_norm = True
        del flat
        if self.grad_clip is not None:
            norm = global_grad_norm(local_sumsq, reduce=reduce_norm, group=self.group)
            self.last_grad_norm = float(norm)
            self.grad_shard.mul_(clip_coefficient(norm, self.grad_clip))
        if self.master_shard is not None:
            shard = self.master_shard
        else:
            shard = _flatten([p.detach() for p in self.params], self.padded)[lo:hi].clone()
        adamw_update_(shard, self.grad_shard, self.exp_avg, self.exp_avg_sq, self.step_count,
                      self.lr, self.beta1, self.beta2, self.eps, self.decay)
        gathered = torch.empty(self.padded, dtype=self.param_dtype, device=shard.device)
        comms.all_gather_into(gathered, shard.to(self.param_dtype), group=self.group)
        off = 0
        for p in self.params:
            n = p.numel()
            p.copy_(gathered[off:off + n].view_as(p))
            off += n


def _run_unit(module: nn.Module, full: torch.Tensor, meta, x: torch.Tensor) -> torch.Tensor:
    params, off = {}, 0
    for name, shape, numel in meta:
        params[name] = full[off:off + numel].view(shape)
        off += numel
    out = functional_call(module, params, (x,))
    return out[0] if isinstance(out, tuple) else out


class _GatherRunFree(torch.autograd.Function):
    """Gather a unit's parameters, run it, free them; backward gathers again,
    recomputes, backpropagates and reduce-scatters the unit gradient (/p)."""

    @staticmethod
    def forward(ctx, x, shard, module, meta, world_size, param_dtype, reduce_dtype, group):
        ctx.module, ctx.meta, ctx.world_size = module, meta, world_size
        ctx.param_dtype, ctx.reduce_dtype, ctx.group = param_dtype, reduce_dtype, group
        ctx.in_dtype = x.dtype
        ctx.save_for_backward(x, shard)
        with torch.no_grad():
            full = torch.empty(shard.numel() * world_size, dtype=param_dtype, device=shard.device)
            comms.all_gather_into(full, shard.to(param_dtype), group=group)
            out = _run_unit(module, full, meta, x.to(param_dtype))
            del full
        return out.to(ctx.in_dtype)

    @staticmethod
    def backward(ctx, grad_out):
        x, shard = ctx.saved_tensors
        full = torch.empty(shard.numel() * ctx.world_size, dtype=ctx.param_dtype, device=shard.device)
        comms.all_gather_into(full, shard.to(ctx.param_dtype), group=ctx.group)
        full.requires_grad_(True)
        x_in = x.detach().to(ctx.param_dtype).requires_grad_(True)
        with torch.enable_grad():
            out = _run_unit(ctx.module, full, ctx.meta, x_in)
        gx, gfull = torch.autograd.grad(out, [x_in, full], grad_outputs=grad_out.to(ctx.param_dtype))
        wire = gfull.contiguous().to(ctx.reduce_dtype)
        wshard = torch.empty(shard.numel(), dtype=ctx.reduce_dtype, device=shard.device)
        comms.reduce_scatter_into(wshard, wire, group=ctx.group)
        gshard = wshard.to(shard.dtype).div_(ctx.world_size)
        return gx.to(ctx.in_dtype), gshard, None, None, None, None, None, None


class Zero3Model(nn.Module):
    """A GPT whose blocks are parameter-sharded units (one flat shard each);
    root parameters (wte, wpe, ln_f, tied head) stay replicated. Consumes
    `model`: the blocks' own parameter storages are released."""

    def __init__(self, model: nn.Module, rank: int, world_size: int, param_dtype=None,
                 reduce_dtype=None, group: Any = None) -> None:
        super().__init__()
        self.model = model
        self.rank, self.world_size, self.group = rank, world_size, group
        self.param_dtype = reduce_dtype_of(param_dtype)
        self.reduce_dtype = reduce_dtype_of(reduce_dtype)
        self.unit_meta = []
        self.shards = nn.ParameterList()
        for block in model.h:
            named = list(block.named_parameters())
            meta = tuple((n, p.shape, p.numel()) for n, p in named)
            numel = sum(m[2] for m in meta)
            padded = padded_numel(numel, world_size)
            flat = _flatten([p.detach() for _, p in named], padded)
            sz = padded // world_size
            self.unit_meta.append(meta)
            self.shards.append(nn.Parameter(flat[rank * sz:(rank + 1) * sz].clone()))
            for _, p in named:
                p.data = torch.empty(0, device=p.device)
                p.requires_grad_(False)
        self.root_params = [p for n, p in model.named_parameters()
                            if not n.startswith("h.") and p.requires_grad and p.numel() > 0]

    def unit_decay_mask(self, unit: int, weight_decay: float) -> torch.Tensor:
        meta = self.unit_meta[unit]
        dev = self.shards[unit].device
        full = torch.cat([torch.full((n,), float(len(s) >= 2), device=dev) for _, s, n in meta])
        sz = self.shards[unit].numel()
        padded = torch.zeros(sz * self.world_size, device=dev)
        padded[:full.numel()] = full
        return padded[self.rank * sz:(self.rank + 1) * sz] * weight_decay

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None) -> dict:
        m = self.model
        _, t = idx.shape
        pos = torch.arange(0, t, dtype=torch.long, device=idx.device)
        x = m.drop(m.wte(idx) + m.position_embeddings(pos))
        for u, block in enumerate(m.h):
            x = _GatherRunFree.apply(x, self.shards[u], block, self.unit_meta[u], self.world_size,
                                     self.param_dtype, self.reduce_dtype, self.group)
        logits = m.lm_head(m.ln_f(x))
        out = {"logits": logits}
        if targets is not None:
            out["loss"] = nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)),
                                                      targets.reshape(-1))
        return out

    def resident_bytes(self, optimizer_state=(), constants=()) -> dict[str, int]:
        params = list(self.shards) + self.root_params
        out = {"params": state_bytes(params),
               "grads": state_bytes([p.grad for p in params if p.grad is not None]),
               "optimizer": state_bytes(optimizer_state), "decay_mask": state_bytes(constants)}
        out["total"] = sum(out.values())
        return out


class Zero3AdamW:
    """AdamW for Zero3Model: shard-local updates for the units (their gradient
    was reduce-scattered in backward), per-tensor all-reduce for the root."""

    def __init__(self, model: Zero3Model, lr: float = 1e-3, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1, grad_clip: Optional[float] = None, reduce_dtype=None) -> None:
        self.model = model
        self.lr, (self.beta1, self.beta2), self.eps = lr, betas, eps
        self.weight_decay = weight_decay
        self.grad_clip = grad_clip
        self.reduce_dtype = reduce_dtype_of(reduce_dtype)
        self.last_grad_norm = float("nan")
        self.step_count = 0
        self.state: dict[int, tuple] = {}
        self.decay: dict[int, torch.Tensor] = {}
        for i, sh in enumerate(model.shards):
            self.state[id(sh)] = (torch.zeros_like(sh), torch.zeros_like(sh))
            self.decay[id(sh)] = model.unit_decay_mask(i, weight_decay)
        for p in model.root_params:
            self.state[id(p)] = (torch.zeros_like(p), torch.zeros_like(p))

    def zero_grad(self) -> None:
        for p in list(self.model.shards) + self.model.root_params:
            p.grad = None

    def optimizer_tensors(self) -> list:
        return [t for pair in self.state.values() for t in pair]

    def constant_tensors(self) -> list:
        return list(self.decay.values())

    def step(self) -> None:
        self.step_count += 1
        m = self.model
        average_gradients(m.root_params, m.world_size, bucket_bytes=0, reduce_dtype=self.reduce_dtype,
                          group=m.group)
        coef = None
        if self.grad_clip is not None:
            dev = m.shards[0].device
            ss = torch.zeros((), device=dev)
            for sh in m.shards:
                if sh.grad is not None:
                    ss = ss + sh.grad.pow(2).sum()
            root = sum((p.grad.pow(2).sum() for p in m.root_params if p.grad is not None),
                       torch.zeros((), device=dev))
            norm = global_grad_norm(ss, root, reduce=True, group=m.group)
            self.last_grad_norm = float(norm)
            coef = clip_coefficient(norm, self.grad_clip)
        with torch.no_grad():
            if coef is not None:
                for p in list(m.shards) + m.root_params:
                    if p.grad is not None:
                        p.grad.mul_(coef)
            for sh in m.shards:
                if sh.grad is None:
                    continue
                mm, vv = self.state[id(sh)]
                adamw_update_(sh.data, sh.grad, mm, vv, self.step_count, self.lr, self.beta1,
                              self.beta2, self.eps, self.decay[id(sh)])
            for p in m.root_params:
                if p.grad is None:
                    continue
                mm, vv = self.state[id(p)]
                adamw_update_(p.data, p.grad, mm, vv, self.step_count, self.lr, self.beta1,
                              self.beta2, self.eps, self.weight_decay if p.dim() >= 2 else 0.0)

    def gathered_block_params(self, unit: int) -> torch.Tensor:
        sh = self.model.shards[unit]
        full = torch.empty(sh.numel() * self.model.world_size, dtype=sh.dtype, device=sh.device)
        comms.all_gather_into(full, sh.detach(), group=self.model.group)
        return full


def zero3_payload_bytes(unit_numels: Sequence[int], root_numel: int, world_size: int,
                        param_bytes: int = 4, reduce_bytes: int = 4, root_bytes: int = 4) -> int:
    """Closed-form ZeRO-3 per-rank payload per step: per unit two parameter
    all-gathers (output = padded unit) and one gradient reduce-scatter (input
    = padded unit), plus the root all-reduce."""
    total = 0
    for n in unit_numels:
        pu = padded_numel(n, world_size)
        total += 2 * param_bytes * pu + reduce_bytes * pu
    return total + root_bytes * root_numel


def _reference_adamw(model: nn.Module, lr: float, betas, eps: float, weight_decay: float):
    decay = [p for p in model.parameters() if p.dim() >= 2]
    rest = [p for p in model.parameters() if p.dim() < 2]
    return torch.optim.AdamW([{"params": decay, "weight_decay": weight_decay},
                              {"params": rest, "weight_decay": 0.0}], lr=lr, betas=betas, eps=eps)


def zero_equivalence_worker(rank: int, world_size: int, stage: int = 2, steps: int = 4, batch: int = 8,
                            seq: int = 16, lr: float = 1e-3, weight_decay: float = 0.1,
                            grad_clip: Optional[float] = None, reduce_dtype=None, param_dtype=None,
                            config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """ShardedAdamW vs single-process torch AdamW on the full batch, several
    steps, comparing parameters after every step (and grad norms if clipped)."""
    from gpt2_harness_b200.perf.activation_memory import ActivationMeter

    cfg = parallel_config(**(config_kwargs or {}))
    inputs, targets = identical_batch(cfg, batch, seq)
    x, y = local_shard(inputs, rank, world_size), local_shard(targets, rank, world_size)
    model = identical_model(cfg, seed=0)
    ref = identical_model(cfg, seed=0)
    betas = (0.9, 0.95)
    opt = ShardedAdamW(list(model.parameters()), rank, world_size, stage, lr, betas,
                       weight_decay=weight_decay, grad_clip=grad_clip, reduce_dtype=reduce_dtype,
                       param_dtype=param_dtype)
    ref_opt = _reference_adamw(ref, lr, betas, 1e-8, weight_decay)
    base = identical_model(cfg, seed=0)
    base_opt = _reference_adamw(base, lr, betas, 1e-8, weight_decay)
    errors, norms = [], []
    acts: dict = {}
    for step in range(steps):
        opt.zero_grad()
        if step == 0:
            meter = ActivationMeter(exclude=[*model.parameters(), *model.buffers()])
            with meter:
                out = model(x, targets=y)
            acts = meter.snapshot()
        else:
            out = model(x, targets=y)
        out["loss"].backward()
        opt.step()
        comms.get_counter().steps += 1
        ref_opt.zero_grad(set_to_none=True)
        ref(inputs, targets=targets)["loss"].backward()
        if grad_clip is not None:
            rn = float(torch.nn.utils.clip_grad_norm_(ref.parameters(), grad_clip))
            norms.append({"sharded": opt.last_grad_norm, "reference": rn})
        ref_opt.step()
        with comms.counter_scope(world_size):  # replicated baseline, not counted
            base_opt.zero_grad(set_to_none=True)
            base(x, targets=y)["loss"].backward()
            average_gradients(base.parameters(), world_size, bucket_bytes=0)
            base_opt.step()
        errors.append(max(float((a - b).abs().max()) for a, b in zip(model.parameters(), ref.parameters())))
    base_state = [t for st in base_opt.state.values() for t in (st.get("exp_avg"), st.get("exp_avg_sq"))
                  if t is not None]
    base_bytes = {"params": state_bytes(base),
                  "grads": state_bytes([p.grad for p in base.parameters() if p.grad is not None]),
                  "optimizer": state_bytes(base_state), "decay_mask": 0}
    base_bytes["total"] = sum(base_bytes.values())
    return {
        "rank": rank, "stage": stage, "grad_clip": grad_clip,
        "reduce_dtype": reduce_dtype or "fp32", "param_dtype": param_dtype or "fp32",
        "max_param_error": max(errors), "param_errors": errors, "grad_norms": norms,
        "max_grad_norm_error": max(abs(n["sharded"] - n["reference"]) for n in norms) if norms else None,
        "n_params": sum(p.numel() for p in model.parameters()),
        "reference_param_scale": max(float(p.detach().abs().max()) for p in ref.parameters()),
        "shard_numel": opt.shard_size, "padded_numel": opt.padded,
        "sharded_bytes": opt.resident_bytes(), "replicated_bytes": base_bytes,
        "activation_bytes": acts.get("activation_bytes", 0), "activation_detail": acts,
    }


def zero3_equivalence_worker(rank: int, world_size: int, steps: int = 3, batch: int = 8, seq: int = 16,
                             lr: float = 1e-3, weight_decay: float = 0.1, grad_clip: Optional[float] = None,
                             reduce_dtype=None, param_dtype=None,
                             config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """Zero3Model + Zero3AdamW vs single-process AdamW; the comparison
    all-gathers every unit (in an uncounted scope) so shards this rank does
    not own are checked too."""
    from gpt2_harness_b200.perf.activation_memory import ActivationMeter

    cfg = parallel_config(**(config_kwargs or {}))
    inputs, targets = identical_batch(cfg, batch, seq)
    x, y = local_shard(inputs, rank, world_size), local_shard(targets, rank, world_size)
    betas = (0.9, 0.95)
    model = Zero3Model(identical_model(cfg, seed=0), rank, world_size, param_dtype, reduce_dtype)
    opt = Zero3AdamW(model, lr, betas, weight_decay=weight_decay, grad_clip=grad_clip,
                     reduce_dtype=reduce_dtype)
    ref = identical_model(cfg, seed=0)
    ref_opt = _reference_adamw(ref, lr, betas, 1e-8, weight_decay)
    errors, losses, norms = [], [], []
    acts: dict = {}
    for step in range(steps):
        opt.zero_grad()
        if step == 0:
            meter = ActivationMeter(exclude=[*model.parameters(), *model.buffers()])
            with meter:
                out = model(x, targets=y)
            acts = meter.snapshot()
        else:
            out = model(x, targets=y)
        out["loss"].backward()
        opt.step()
        comms.get_counter().steps += 1
        losses.append(float(out["loss"]))
        ref_opt.zero_grad(set_to_none=True)
        ref(inputs, targets=targets)["loss"].backward()
        if grad_clip is not None:
            norms.append({"sharded": opt.last_grad_norm,
                          "reference": float(torch.nn.utils.clip_grad_norm_(ref.parameters(), grad_clip))})
        ref_opt.step()
        worst = 0.0
        with comms.counter_scope(world_size):
            gathered = [opt.gathered_block_params(u) for u in range(len(model.shards))]
        for u, block in enumerate(ref.h):
            want = torch.cat([p.detach().reshape(-1) for p in block.parameters()])
            worst = max(worst, float((gathered[u][:want.numel()] - want).abs().max()))
        for got, want in zip(model.root_params, [p for n, p in ref.named_parameters() if not n.startswith("h.")]):
            worst = max(worst, float((got.detach() - want.detach()).abs().max()))
        errors.append(worst)
    unit_numels = [sum(m[2] for m in meta) for meta in model.unit_meta]
    root_numel = sum(p.numel() for p in model.root_params)
    return {
        "rank": rank, "grad_clip": grad_clip,
        "reduce_dtype": reduce_dtype or "fp32", "param_dtype": param_dtype or "fp32",
        "max_param_error": max(errors), "param_errors": errors, "losses": losses, "grad_norms": norms,
        "max_grad_norm_error": max(abs(n["sharded"] - n["reference"]) for n in norms) if norms else None,
        "unit_numels": unit_numels, "root_numel": root_numel,
        "closed_form_payload_bytes": zero3_payload_bytes(unit_numels, root_numel, world_size),
        "resident_bytes": model.resident_bytes(opt.optimizer_tensors(), opt.constant_tensors()),
        "activation_bytes": acts.get("activation_bytes", 0),
    }
