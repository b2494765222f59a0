"""Pipeline parallelism: stage split, GPipe / 1F1B schedules, a dependency
simulator and the point-to-point runtime.

Reference semantics (src/transformer_internals/parallel/pipeline_parallel.py:
56-499): contiguous depth split; stage 0 owns the embeddings, the last stage
ln_f and the head (untied from wte in the pipelined model, and so in its
single-process reference); sends are non-blocking and receives blocking (time
blocked in a receive IS the bubble); the loss of each micro-batch is divided
by m; the bubble is measured as 1 - sum(compute)/(p * makespan) and compared
with (p-1)/(m+p-1).

The 2-D PP x CP composition of the 16k-context config lives in
:mod:`gpt2_harness_b200.parallel.mesh`; this module's runtime takes explicit
process groups so it runs unchanged inside one pipeline row of that mesh.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Optional

import torch
import torch.nn as nn

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.common import current_device, identical_batch, identical_model, parallel_config

__all__ = [
    "analytic_bubble",
    "PipelineStage",
    "schedule_order",
    "SimResult",
    "simulate",
    "run_pipeline_step",
    "pipeline_worker",
    "bubble_scan_worker",
    "pipeline_payload_bytes",
]


def analytic_bubble(n_stages: int, micro_batches: int) -> float:
    """(p-1)/(m+p-1): idle fraction of an ideal GPipe/1F1B step."""
    return (n_stages - 1) / (micro_batches + n_stages - 1)


class PipelineStage(nn.Module):
    """One contiguous depth slice of a GPT (consumes `model`; unowned pieces
    are dropped so per-rank parameter counts are real)."""

    def __init__(self, model: nn.Module, stage: int, n_stages: int) -> None:
        super().__init__()
        L = len(model.h)
        if L % n_stages:
            raise ValueError(f"n_layer={L} must be divisible by n_stages={n_stages}")
        per = L // n_stages
        self.stage, self.n_stages = stage, n_stages
        self.is_first, self.is_last = stage == 0, stage == n_stages - 1
        self.blocks = nn.ModuleList(list(model.h)[stage * per:(stage + 1) * per])
        self.config = model.config
        if self.is_first:
            self.wte, self.wpe, self.drop = model.wte, model.wpe, model.drop
        if self.is_last:
            self.ln_f, self.lm_head = model.ln_f, model.lm_head

    def forward(self, x: torch.Tensor, pos_offset: int = 0) -> torch.Tensor:
        if self.is_first:
            t = x.shape[1]
            pos = torch.arange(pos_offset, pos_offset + t, dtype=torch.long, device=x.device)
            h = self.drop(self.wte(x) + self.wpe(pos))
        else:
            h = x
        for blk in self.blocks:
            h, _ = blk(h)
        return self.lm_head(self.ln_f(h)) if self.is_last else h


def untied_reference_model(config) -> nn.Module:
    """The single-process oracle with the head untied (as the pipeline places
    it), so a mismatch is a pipeline bug, not a tying difference."""
    model = identical_model(config, seed=0)
    model.lm_head = nn.Linear(config.n_embd, config.vocab_size, bias=False).to(current_device())
    model.lm_head.weight = nn.Parameter(model.wte.weight.detach().clone())
    return model


def schedule_order(rank: int, n_stages: int, micro_batches: int, kind: str) -> list:
    """Ops of one rank as ("F"|"B", micro_batch). GPipe: all forwards then all
    backwards in reverse; 1F1B: p-1-r warm-up forwards, then alternate, then
    drain."""
    m = micro_batches
    if kind == "gpipe":
        return [("F", i) for i in range(m)] + [("B", i) for i in reversed(range(m))]
    if kind != "1f1b":
        raise ValueError(f"unknown schedule {kind!r}")
    warm = min(n_stages - 1 - rank, m)
    ops = [("F", i) for i in range(warm)]
    for i in range(m - warm):
        ops.append(("F", warm + i))
        ops.append(("B", i))
    ops += [("B", i) for i in range(m - warm, m)]
    return ops


@dataclass
class SimResult:
    makespan: float
    bubble: float
    peak_stash: int


def simulate(n_stages: int, micro_batches: int, t_f: float, t_b: float, kind: str = "gpipe") -> SimResult:
    """Event simulation of a schedule under its true dependencies: F(r,i)
    after F(r-1,i); B(r,i) after B(r+1,i) (the last stage after its own
    F). Returns makespan, bubble fraction and peak live micro-batch stash."""
    orders = [schedule_order(r, n_stages, micro_batches, kind) for r in range(n_stages)]
    done: dict = {}
    free = [0.0] * n_stages
    cur = [0] * n_stages
    live = [0] * n_stages
    peak = 0
    left = sum(len(o) for o in orders)
    while left:
        moved = False
        for r in range(n_stages):
            if cur[r] >= len(orders[r]):
                continue
            op, i = orders[r][cur[r]]
            if op == "F":
                dep = 0.0 if r == 0 else done.get((r - 1, "F", i))
            elif r == n_stages - 1:
                dep = done.get((r, "F", i))
            else:
                dep = done.get((r + 1, "B", i))
            if dep is None:
                continue
            end = max(free[r], dep) + (t_f if op == "F" else t_b)
            done[(r, op, i)] = end
            free[r] = end
            cur[r] += 1
            left -= 1
            moved = True
            live[r] += 1 if op == "F" else -1
            peak = max(peak, live[r])
        if not moved:
            raise RuntimeError("schedule deadlocked in simulation")
    span = max(free)
    return SimResult(span, 1.0 - micro_batches * (t_f + t_b) / span, peak)


class _Timer:
    """Splits a rank's wall clock into compute and blocked-on-a-peer time."""

    def __init__(self) -> None:
        self.compute = 0.0
        self.comm = 0.0

    def __call__(self, kind: str):
        timer = self

        class _Ctx:
            def __enter__(self_inner):
                self_inner.t0 = time.perf_counter()

            def __exit__(self_inner, *exc):
                dt = time.perf_counter() - self_inner.t0
                if kind == "compute":
                    timer.compute += dt
                else:
                    timer.comm += dt

        return _Ctx()


def run_pipeline_step(stage: PipelineStage, rank: int, world: int, micro_inputs: list,
                      micro_targets: list, hidden_shape: tuple, kind: str, timer: _Timer,
                      group: Any = None, prev_rank: Optional[int] = None,
                      next_rank: Optional[int] = None, dtype=torch.float32) -> tuple:
    """One optimiser step of pipeline work. `prev_rank`/`next_rank` are global
    ranks of the neighbouring stages (default rank-1 / rank+1). Returns
    (loss_sum, peak_stash)."""
    m = len(micro_inputs)
    dev = micro_inputs[0].device
    prev_rank = rank - 1 if prev_rank is None else prev_rank
    next_rank = rank + 1 if next_rank is None else next_rank
    ins: dict = {}
    outs: dict = {}
    pending: list = []
    loss_sum = 0.0
    peak = 0
    for op, i in schedule_order(stage.stage, stage.n_stages, m, kind):
        if op == "F":
            if stage.is_first:
                x = micro_inputs[i]
            else:
                buf = torch.empty(hidden_shape, device=dev, dtype=dtype)
                with timer("comm"):
                    comms.recv(buf, src=prev_rank, group=group)
                x = buf.requires_grad_(True)
            with timer("compute"):
                out = stage(x)
            ins[i], outs[i] = x, out
            peak = max(peak, len(outs))
            if not stage.is_last:
                with timer("comm"):
                    pending.append((comms.isend(out.detach(), dst=next_rank, group=group), out))
            else:
                with timer("compute"):
                    loss = nn.functional.cross_entropy(out.reshape(-1, out.size(-1)),
                                                       micro_targets[i].reshape(-1)) / m
                outs[i] = loss
                loss_sum += float(loss.detach())
        else:
            out = outs.pop(i)
            x = ins.pop(i)
            if stage.is_last:
                with timer("compute"):
                    out.backward()
            else:
                g = torch.empty(out.shape, device=dev, dtype=out.dtype)
                with timer("comm"):
                    comms.recv(g, src=next_rank, group=group)
                with timer("compute"):
                    out.backward(g)
            if not stage.is_first:
                with timer("comm"):
                    pending.append((comms.isend(x.grad.detach(), dst=prev_rank, group=group), x))
    for h, _ in pending:
        h.wait()
    return loss_sum, peak


def pipeline_payload_bytes(micro_batches: int, micro_batch: int, seq: int, n_embd: int,
                           elem_bytes: int = 4) -> int:
    """Per-boundary, per-direction bytes of one step: m activations (or
    gradients) of micro x seq x C."""
    return micro_batches * micro_batch * seq * n_embd * elem_bytes


def pipeline_worker(rank: int, world_size: int, micro_batches: int = 4, batch: int = 8, seq: int = 16,
                    kind: str = "gpipe", check_grads: bool = True,
                    config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """One pipelined step; this rank's stage gradients vs the same stage of a
    model that saw the whole batch at once (a missing 1/m shows as x m)."""
    from gpt2_harness_b200.perf.activation_memory import ActivationMeter

    cfg = parallel_config(**(config_kwargs or {}))
    inputs, targets = identical_batch(cfg, batch, seq)
    if batch % micro_batches:
        raise ValueError(f"batch={batch} must be divisible by micro_batches={micro_batches}")
    micro = batch // micro_batches
    mi, mt = list(inputs.split(micro)), list(targets.split(micro))
    stage = PipelineStage(untied_reference_model(cfg), rank, world_size)
    timer = _Timer()
    meter = ActivationMeter(exclude=[*stage.parameters(), *stage.buffers()])
    comms.barrier()
    t0 = time.perf_counter()
    with meter:
        loss_sum, peak = run_pipeline_step(stage, rank, world_size, mi, mt, (micro, seq, cfg.n_embd),
                                           kind, timer)
    wall = time.perf_counter() - t0
    comms.get_counter().steps += 1
    res: dict[str, Any] = {
        "rank": rank, "kind": kind, "micro_batches": micro_batches, "loss": loss_sum,
        "peak_stash": peak, "compute_seconds": timer.compute, "comm_seconds": timer.comm,
        "wall_seconds": wall, "stage_params": sum(p.numel() for p in stage.parameters()),
        "activation_peak_bytes": meter.peak_bytes,
        "closed_form_send_bytes": pipeline_payload_bytes(micro_batches, micro, seq, cfg.n_embd),
    }
    if check_grads:
        ref = untied_reference_model(cfg)
        ref(inputs, targets=targets)["loss"].backward()
        ref_stage = PipelineStage(ref, rank, world_size)
        errs = [float((a.grad - b.grad).abs().max()) for a, b in zip(stage.parameters(), ref_stage.parameters())
                if a.grad is not None and b.grad is not None]
        res["max_grad_error"] = max(errs) if errs else 0.0
        res["reference_grad_scale"] = max(float(b.grad.abs().max()) for b in ref_stage.parameters()
                                          if b.grad is not None)
        res["compared_tensors"] = len(errs)
    return res


def bubble_scan_worker(rank: int, world_size: int, micro_batch_counts: tuple = (1, 2, 4, 8),
                       batch: int = 8, seq: int = 32, repeats: int = 3, warmup: int = 1,
                       config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """Measured bubble (1 - sum compute / (p * makespan)) vs micro-batch count
    for both schedules, batch held fixed (more micro-batches = smaller ones)."""
    cfg = parallel_config(**(config_kwargs or {}))
    inputs, targets = identical_batch(cfg, batch, seq)
    stage = PipelineStage(untied_reference_model(cfg), rank, world_size)
    rows = []
    for kind in ("gpipe", "1f1b"):
        for m in micro_batch_counts:
            if batch % m:
                continue
            micro = batch // m
            mi, mt = list(inputs.split(micro)), list(targets.split(micro))
            best = None
            for rep in range(warmup + repeats):
                for prm in stage.parameters():
                    prm.grad = None
                timer = _Timer()
                comms.barrier()
                t0 = time.perf_counter()
                _, peak = run_pipeline_step(stage, rank, world_size, mi, mt, (micro, seq, cfg.n_embd),
                                            kind, timer)
                wall = time.perf_counter() - t0
                if rep < warmup:
                    continue
                row = {"compute_seconds": timer.compute, "comm_seconds": timer.comm,
                       "wall_seconds": wall, "peak_stash": peak}
                if best is None or row["wall_seconds"] < best["wall_seconds"]:
                    best = row
            rows.append({"kind": kind, "micro_batches": m, "micro_batch_size": micro,
                         "analytic_bubble": analytic_bubble(world_size, m), **best})
    return {"rank": rank, "world_size": world_size, "rows": rows}
