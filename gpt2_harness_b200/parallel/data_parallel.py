"""Data parallelism: bucketed gradient averaging and its equivalence worker.

Reference: src/transformer_internals/parallel/data_parallel.py:45-277. The
gradient of the full batch equals the mean over ranks of each rank's gradient
on its slice, so DDP is: SUM all-reduce of reverse-order buckets (25 MiB cap,
torch DDP's default), then divide by p. An optional bf16 wire casts each
bucket down before the reduction and back up after it (division in fp32).

This module is the reference-semantics (torch.distributed) path used by the
CPU/gloo oracle tests and by any torch model; the B200 engine's overlapped,
peer-memory version of the same algorithm is
:mod:`gpt2_harness_b200.parallel.ddp_native`.
"""

from __future__ import annotations

from typing import Any, Iterable, Optional, Sequence

import torch
import torch.nn as nn

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.common import identical_batch, identical_model, parallel_config
from gpt2_harness_b200.precision import reduce_dtype_of

__all__ = [
    "DEFAULT_BUCKET_BYTES",
    "average_gradients",
    "build_buckets",
    "ddp_equivalence_worker",
    "local_shard",
]

DEFAULT_BUCKET_BYTES = 25 * 1024 * 1024


def local_shard(tensor: torch.Tensor, rank: int, world_size: int, dim: int = 0) -> torch.Tensor:
    """This rank's contiguous slice along `dim`; uneven splits are refused
    (they would make a plain gradient average differ from the full batch)."""
    n = tensor.shape[dim]
    if n % world_size:
        raise ValueError(f"axis {dim} of length {n} does not split across {world_size} ranks")
    per = n // world_size
    return tensor.narrow(dim, rank * per, per).contiguous()


def build_buckets(params: Sequence[nn.Parameter], bucket_bytes: int = DEFAULT_BUCKET_BYTES):
    """Greedy buckets in REVERSE parameter order (backward produces the last
    layers' gradients first); a tensor larger than the cap gets its own."""
    buckets, cur, size = [], [], 0
    for p in reversed(list(params)):
        nbytes = p.numel() * p.element_size()
        if cur and size + nbytes > bucket_bytes:
            buckets.append(cur)
            cur, size = [], 0
        cur.append(p)
        size += nbytes
    if cur:
        buckets.append(cur)
    return buckets


def average_gradients(params: Iterable[nn.Parameter], world_size: int,
                      bucket_bytes: int = DEFAULT_BUCKET_BYTES, reduce_dtype=None,
                      group: Any = None) -> int:
    """All-reduce every gradient and divide by `world_size`, in place.

    Parameters without a gradient are skipped. ``bucket_bytes <= 0`` issues one
    collective per tensor. Returns the number of collectives issued.
    """
    dtype = reduce_dtype_of(reduce_dtype) if reduce_dtype is not None else None
    live = [p for p in params if p.grad is not None]
    if not live:
        return 0
    buckets = [[p] for p in reversed(live)] if bucket_bytes <= 0 else build_buckets(live, bucket_bytes)
    for bucket in buckets:
        flat = torch.cat([p.grad.reshape(-1) for p in bucket])
        if dtype is not None and dtype != flat.dtype:
            wire = flat.to(dtype)
            comms.all_reduce(wire, group=group)
            flat = wire.to(flat.dtype)
        else:
            comms.all_reduce(flat, group=group)
        flat.div_(world_size)
        off = 0
        for p in bucket:
            n = p.grad.numel()
            p.grad.copy_(flat[off:off + n].view_as(p.grad))
            off += n
    return len(buckets)


def _grad_vector(model: nn.Module) -> torch.Tensor:
    return torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1)
                      for p in model.parameters()])


def ddp_equivalence_worker(rank: int, world_size: int, batch: int = 8, seq: int = 16, steps: int = 3,
                           bucket_bytes: int = DEFAULT_BUCKET_BYTES, reduce_dtype: Optional[str] = None,
                           config_kwargs: Optional[dict] = None, optimizer: str = "sgd",
                           lr: float = 0.1) -> dict[str, Any]:
    """DDP vs single-process full-batch training, in one process per rank.

    The local model sees batch/p rows and averages gradients; the reference
    model sees the whole batch with no collectives. Gradients and parameters
    are compared after every step (SGD lr 0.1 as in the reference, or AdamW
    with ``optimizer="adamw"``).
    """
    from gpt2_harness_b200.perf.activation_memory import ActivationMeter

    cfg = parallel_config(**(config_kwargs or {}))
    inputs, targets = identical_batch(cfg, batch, seq)
    model = identical_model(cfg, seed=0)
    ref = identical_model(cfg, seed=0)
    if optimizer == "adamw":
        opt = model.configure_optimizers(0.1, lr, (0.9, 0.95))
        ref_opt = ref.configure_optimizers(0.1, lr, (0.9, 0.95))
    else:
        opt = torch.optim.SGD(model.parameters(), lr=lr)
        ref_opt = torch.optim.SGD(ref.parameters(), lr=lr)
    x, y = local_shard(inputs, rank, world_size), local_shard(targets, rank, world_size)
    grad_err, param_err, losses, ref_losses = [], [], [], []
    buckets = 0
    act_local: dict = {}
    act_ref: dict = {}
    for step in range(steps):
        opt.zero_grad(set_to_none=True)
        if step == 0:
            meter = ActivationMeter(exclude=[*model.parameters(), *model.buffers()])
            with meter:
                out = model(x, targets=y)
            act_local = meter.snapshot()
        else:
            out = model(x, targets=y)
        out["loss"].backward()
        buckets = average_gradients(model.parameters(), world_size, bucket_bytes, reduce_dtype)
        comms.get_counter().steps += 1
        ref_opt.zero_grad(set_to_none=True)
        if step == 0:
            meter = ActivationMeter(exclude=[*ref.parameters(), *ref.buffers()])
            with meter:
                ref_out = ref(inputs, targets=targets)
            act_ref = meter.snapshot()
        else:
            ref_out = ref(inputs, targets=targets)
        ref_out["loss"].backward()
        grad_err.append(float((_grad_vector(model) - _grad_vector(ref)).abs().max()))
        opt.step()
        ref_opt.step()
        param_err.append(max(float((a - b).abs().max()) for a, b in zip(model.parameters(), ref.parameters())))
        losses.append(float(out["loss"]))
        ref_losses.append(float(ref_out["loss"]))
    return {
        "rank": rank,
        "reduce_dtype": reduce_dtype or "fp32",
        "max_grad_error": max(grad_err),
        "max_param_error": max(param_err),
        "grad_errors": grad_err,
        "local_losses": losses,
        "reference_losses": ref_losses,
        "buckets": buckets,
        "n_params": sum(p.numel() for p in model.parameters()),
        "grad_bytes": sum(p.numel() * p.element_size() for p in model.parameters()),
        "activation_bytes": act_local.get("activation_bytes", 0),
        "reference_activation_bytes": act_ref.get("activation_bytes", 0),
        "activation_detail": act_local,
    }
