"""Pipeline parallelism, torch tier: stage split, GPipe / 1F1B orders, a
critical-path schedule model and a point-to-point runtime over any backend.

What it reproduces (reference: src/transformer_internals/parallel/
pipeline_parallel.py:56-499): a contiguous split of the blocks over the
stages, stage 0 holding the embeddings and the last stage ln_f and an lm_head
untied from wte; non-blocking sends and blocking receives of the residual
stream forward and of its gradient backward; each micro-batch's loss divided
by m; the measured bubble 1 - sum(compute) / (p * makespan) against
(p - 1) / (m + p - 1).

How it is built here:

* **Schedules as a stash discipline.** A stage holds the micro-batches whose
  forward has run and whose backward has not (its stash). GPipe lets the
  stash grow to m and drains it last-in-first-out; 1F1B caps it at p - r on
  stage r and drains it first-in-first-out, running a forward whenever the cap
  allows and a backward otherwise. :func:`schedule_order` derives a stage's op
  list from that rule alone.
* **Schedule model as a recurrence.** The finish time of op k of stage r is
  max(finish of op k-1 of r, finish of the op it depends on) + its duration;
  :func:`simulate` evaluates it by memoised recursion over the (stage, op)
  graph, and a cycle in that graph is a schedule that deadlocks.
* **Runtime.** :class:`StageRunner` executes a stage's op list on explicit
  peers and process groups (so it runs unchanged inside one pipeline row of
  the PP x CP mesh in :mod:`gpt2_harness_b200.parallel.mesh`), charging every
  transfer to the counted-collective layer.

The native pipeline (:mod:`gpt2_harness_b200.parallel.pp_native`) walks the
same op lists with the sm_100a kernels.
"""

from __future__ import annotations

import collections
import contextlib
import time
from dataclasses import dataclass, field
from typing import Any, Optional

import torch
import torch.nn as nn

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.common import current_device, identical_batch, identical_model, parallel_config

__all__ = [
    "analytic_bubble",
    "stage_bounds",
    "PipelineStage",
    "schedule_order",
    "stash_limit",
    "SimResult",
    "simulate",
    "StageRunner",
    "run_pipeline_step",
    "pipeline_worker",
    "bubble_scan_worker",
    "pipeline_payload_bytes",
]

SCHEDULES = ("gpipe", "1f1b")


def analytic_bubble(n_stages: int, micro_batches: int) -> float:
    """Idle fraction of an ideal GPipe or 1F1B step: (p - 1) / (m + p - 1)."""
    return (n_stages - 1) / (micro_batches + n_stages - 1)


def stage_bounds(n_layer: int, n_stages: int, stage: int) -> tuple[int, int]:
    """Half-open block range [lo, hi) of `stage` in an even contiguous split."""
    if n_layer % n_stages:
        raise ValueError(f"n_layer={n_layer} must be divisible by n_stages={n_stages}")
    if not 0 <= stage < n_stages:
        raise ValueError(f"stage {stage} outside 0..{n_stages - 1}")
    width = n_layer // n_stages
    return stage * width, (stage + 1) * width


# ------------------------------------------------------------------ stages --
class PipelineStage(nn.Module):
    """The blocks [lo, hi) of a GPT plus, on the first stage, its embeddings
    and, on the last, its final LayerNorm and head.

    The modules are taken over from `model` (not copied); what this stage does
    not own is left behind, so a stage's parameter count is what its rank
    really holds."""

    def __init__(self, model: nn.Module, stage: int, n_stages: int) -> None:
        super().__init__()
        lo, hi = stage_bounds(len(model.h), n_stages, stage)
        self.stage, self.n_stages = stage, n_stages
        self.is_first = stage == 0
        self.is_last = stage == n_stages - 1
        self.config = model.config
        self.blocks = nn.ModuleList(model.h[j] for j in range(lo, hi))
        # Optional ends. Registered as attributes only when owned, so
        # parameters() lists exactly this stage's tensors.
        owned = []
        if self.is_first:
            owned += ["wte", "wpe", "drop"]
        if self.is_last:
            owned += ["ln_f", "lm_head"]
        for name in owned:
            setattr(self, name, getattr(model, name))

    def _embed(self, tokens: torch.Tensor, pos_offset: int) -> torch.Tensor:
        pos = torch.arange(tokens.shape[1], device=tokens.device) + pos_offset
        return self.drop(self.wte(tokens) + self.wpe(pos))

    def forward(self, x: torch.Tensor, pos_offset: int = 0) -> torch.Tensor:
        h = self._embed(x, pos_offset) if self.is_first else x
        for block in self.blocks:
            h = block(h)[0]
        if not self.is_last:
            return h
        return self.lm_head(self.ln_f(h))


def untied_reference_model(config) -> nn.Module:
    """The single-process oracle with its head untied from wte (initialised to
    the same values), which is how the pipeline places it: a mismatch against
    it is then a pipeline bug, not a weight-tying difference."""
    model = identical_model(config, seed=0)
    head = nn.Linear(config.n_embd, config.vocab_size, bias=False).to(current_device())
    with torch.no_grad():
        head.weight.copy_(model.wte.weight)
    model.lm_head = head
    return model


# --------------------------------------------------------------- schedules --
def stash_limit(rank: int, n_stages: int, micro_batches: int, kind: str) -> int:
    """Most micro-batches stage `rank` keeps between forward and backward."""
    if kind == "gpipe":
        return micro_batches
    if kind == "1f1b":
        return max(1, n_stages - rank)
    raise ValueError(f"unknown schedule {kind!r}; expected one of {SCHEDULES}")


def schedule_order(rank: int, n_stages: int, micro_batches: int, kind: str) -> list:
    """Op list ("F" | "B", micro-batch) of stage `rank`.

    Rule: run the next forward while the stash is below its limit
    (:func:`stash_limit`), otherwise a backward; GPipe takes the newest
    stashed micro-batch (LIFO), 1F1B the oldest (FIFO)."""
    limit = stash_limit(rank, n_stages, micro_batches, kind)
    lifo = kind == "gpipe"
    stash: collections.deque = collections.deque()
    next_fwd = 0
    ops = []
    while next_fwd < micro_batches or stash:
        if next_fwd < micro_batches and len(stash) < limit:
            ops.append(("F", next_fwd))
            stash.append(next_fwd)
            next_fwd += 1
        else:
            ops.append(("B", stash.pop() if lifo else stash.popleft()))
    return ops


@dataclass
class SimResult:
    makespan: float
    bubble: float
    peak_stash: int
    finish: dict = field(default_factory=dict, repr=False)  # (stage, op, i) -> finish time


def simulate(n_stages: int, micro_batches: int, t_f: float, t_b: float, kind: str = "gpipe") -> SimResult:
    """Makespan, bubble and peak stash of a schedule with op times t_f / t_b
    and zero-cost transfers.

    Dependencies: F(r, i) needs F(r-1, i); B(r, i) needs B(r+1, i), and on the
    last stage its own F(r, i); every op also follows the previous op of its
    stage. finish(op) = max(finish of its predecessors) + duration, evaluated
    by memoised recursion; a cycle means the orders deadlock."""
    p, m = n_stages, micro_batches
    orders = [schedule_order(r, p, m, kind) for r in range(p)]
    position = {(r, op, i): k for r in range(p) for k, (op, i) in enumerate(orders[r])}
    finish: dict = {}
    on_path: set = set()

    def cross_dep(r: int, op: str, i: int):
        if op == "F":
            return (r - 1, "F", i) if r > 0 else None
        return (r + 1, "B", i) if r < p - 1 else (r, "F", i)

    def preds(node) -> list:
        r, op, i = node
        k = position[node]
        out = [(r, *orders[r][k - 1])] if k > 0 else []
        dep = cross_dep(r, op, i)
        return out + [dep] if dep is not None else out

    def end(root) -> float:
        # the recurrence, memoised, with an explicit stack instead of Python
        # recursion (the dependency chains are 2pm ops long)
        stack = [root]
        while stack:
            node = stack[-1]
            if node in finish:
                stack.pop()
                continue
            todo = [d for d in preds(node) if d not in finish]
            if todo:
                if node in on_path:
                    raise RuntimeError(f"schedule {kind!r} deadlocks: cycle through {node}")
                on_path.add(node)
                stack.extend(todo)
                continue
            on_path.discard(node)
            ready = max((finish[d] for d in preds(node)), default=0.0)
            finish[node] = ready + (t_f if node[1] == "F" else t_b)
            stack.pop()
        return finish[root]

    makespan = max(end((r, *orders[r][-1])) for r in range(p))
    peak = 0
    for order in orders:
        depth = 0
        for op, _ in order:
            depth += 1 if op == "F" else -1
            peak = max(peak, depth)
    bubble = 1.0 - m * (t_f + t_b) / makespan
    return SimResult(makespan, bubble, peak, finish)


# ----------------------------------------------------------------- runtime --
class _Clock:
    """Wall-clock split of a rank's step into compute and waiting on peers."""

    def __init__(self) -> None:
        self.seconds = {"compute": 0.0, "comm": 0.0}

    @contextlib.contextmanager
    def __call__(self, kind: str):
        t0 = time.perf_counter()
        try:
            yield
        finally:
            self.seconds[kind] += time.perf_counter() - t0

    @property
    def compute(self) -> float:
        return self.seconds["compute"]

    @property
    def comm(self) -> float:
        return self.seconds["comm"]


class StageRunner:
    """Runs one stage's op list for one optimiser step.

    Args:
        stage: this rank's :class:`PipelineStage`.
        hidden_shape: shape of the tensor crossing a stage boundary.
        prev_rank / next_rank: global ranks of the neighbouring stages.
        group: process group of the transfers (None: the default group).
        clock: a :class:`_Clock` that the step's time is charged to.
    """

    def __init__(self, stage: PipelineStage, hidden_shape: tuple, prev_rank: int, next_rank: int,
                 group: Any = None, dtype=torch.float32, clock: Optional[_Clock] = None) -> None:
        self.stage = stage
        self.hidden_shape = hidden_shape
        self.prev_rank, self.next_rank = prev_rank, next_rank
        self.group = group
        self.dtype = dtype
        self.clock = clock or _Clock()
        self.inputs: dict = {}      # micro-batch -> stage input (grad-tracked off stage 0)
        self.outputs: dict = {}     # micro-batch -> stage output, or its scaled loss on the last stage
        self.in_flight: list = []   # (send handle, tensor kept alive until it completes)
        self.loss_sum = 0.0
        self.peak = 0

    def _send(self, tensor: torch.Tensor, dst: int) -> None:
        with self.clock("comm"):
            self.in_flight.append((comms.isend(tensor, dst=dst, group=self.group), tensor))

    def _recv(self, shape: tuple, src: int, device) -> torch.Tensor:
        buf = torch.empty(shape, device=device, dtype=self.dtype)
        with self.clock("comm"):
            comms.recv(buf, src=src, group=self.group)
        return buf

    def forward(self, i: int, tokens: torch.Tensor, targets: torch.Tensor, m: int) -> None:
        st = self.stage
        x = tokens if st.is_first else self._recv(self.hidden_shape, self.prev_rank,
                                                  tokens.device).requires_grad_(True)
        with self.clock("compute"):
            y = st(x)
        self.inputs[i] = x
        if st.is_last:
            with self.clock("compute"):
                flat = y.reshape(-1, y.size(-1))
                y = nn.functional.cross_entropy(flat, targets.reshape(-1)) / m
            self.loss_sum += float(y.detach())
        else:
            self._send(y.detach(), self.next_rank)
        self.outputs[i] = y
        self.peak = max(self.peak, len(self.outputs))

    def backward(self, i: int) -> None:
        st = self.stage
        y, x = self.outputs.pop(i), self.inputs.pop(i)
        if st.is_last:
            with self.clock("compute"):
                y.backward()
        else:
            dy = self._recv(tuple(y.shape), self.next_rank, y.device)
            with self.clock("compute"):
                y.backward(dy)
        if not st.is_first:
            self._send(x.grad.detach(), self.prev_rank)

    def run(self, micro_inputs: list, micro_targets: list, kind: str) -> tuple:
        m = len(micro_inputs)
        for op, i in schedule_order(self.stage.stage, self.stage.n_stages, m, kind):
            if op == "F":
                self.forward(i, micro_inputs[i], micro_targets[i], m)
            else:
                self.backward(i)
        for handle, _ in self.in_flight:
            handle.wait()
        self.in_flight.clear()
        return self.loss_sum, self.peak


def run_pipeline_step(stage: PipelineStage, rank: int, world: int, micro_inputs: list,
                      micro_targets: list, hidden_shape: tuple, kind: str, timer: _Clock,
                      group: Any = None, prev_rank: Optional[int] = None,
                      next_rank: Optional[int] = None, dtype=torch.float32) -> tuple:
    """One optimiser step of pipeline work on this rank (neighbours default to
    rank -/+ 1); returns (sum of the micro-batch losses / m, peak stash)."""
    runner = StageRunner(stage, hidden_shape,
                         rank - 1 if prev_rank is None else prev_rank,
                         rank + 1 if next_rank is None else next_rank,
                         group=group, dtype=dtype, clock=timer)
    return runner.run(micro_inputs, micro_targets, kind)


def pipeline_payload_bytes(micro_batches: int, micro_batch: int, seq: int, n_embd: int,
                           elem_bytes: int = 4) -> int:
    """Bytes one stage boundary carries in one direction per step: an
    activation (forward) or its gradient (backward) of micro x seq x C for
    each of the m micro-batches."""
    return micro_batches * micro_batch * seq * n_embd * elem_bytes


def _split_batch(cfg, batch: int, seq: int, micro_batches: int):
    if batch % micro_batches:
        raise ValueError(f"batch={batch} must be divisible by micro_batches={micro_batches}")
    inputs, targets = identical_batch(cfg, batch, seq)
    micro = batch // micro_batches
    return inputs, targets, micro, list(inputs.split(micro)), list(targets.split(micro))


def _grad_gap(stage: nn.Module, ref_stage: nn.Module) -> tuple[float, float, int]:
    """(max |grad - reference grad|, max |reference grad|, tensors compared)."""
    gap = scale = 0.0
    n = 0
    for a, b in zip(stage.parameters(), ref_stage.parameters()):
        if a.grad is None or b.grad is None:
            continue
        gap = max(gap, float((a.grad - b.grad).abs().max()))
        scale = max(scale, float(b.grad.abs().max()))
        n += 1
    return gap, scale, n


def pipeline_worker(rank: int, world_size: int, micro_batches: int = 4, batch: int = 8, seq: int = 16,
                    kind: str = "gpipe", check_grads: bool = True,
                    config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """One pipelined step on `world_size` stages. This rank's gradients are
    compared with the same stage of an identical model that took the whole
    batch in one pass (a missing 1/m would show as a factor m)."""
    from gpt2_harness_b200.perf.activation_memory import ActivationMeter

    cfg = parallel_config(**(config_kwargs or {}))
    inputs, targets, micro, mi, mt = _split_batch(cfg, batch, seq, micro_batches)
    stage = PipelineStage(untied_reference_model(cfg), rank, world_size)
    clock = _Clock()
    meter = ActivationMeter(exclude=[*stage.parameters(), *stage.buffers()])
    comms.barrier()
    start = time.perf_counter()
    with meter:
        loss_sum, peak = run_pipeline_step(stage, rank, world_size, mi, mt, (micro, seq, cfg.n_embd),
                                           kind, clock)
    wall = time.perf_counter() - start
    comms.get_counter().steps += 1
    out: dict[str, Any] = dict(
        rank=rank, kind=kind, micro_batches=micro_batches, loss=loss_sum, peak_stash=peak,
        compute_seconds=clock.compute, comm_seconds=clock.comm, wall_seconds=wall,
        stage_params=sum(t.numel() for t in stage.parameters()),
        activation_peak_bytes=meter.peak_bytes,
        closed_form_send_bytes=pipeline_payload_bytes(micro_batches, micro, seq, cfg.n_embd),
    )
    if check_grads:
        whole = untied_reference_model(cfg)
        whole(inputs, targets=targets)["loss"].backward()
        gap, scale, n = _grad_gap(stage, PipelineStage(whole, rank, world_size))
        out.update(max_grad_error=gap, reference_grad_scale=scale, compared_tensors=n)
    return out


def bubble_scan_worker(rank: int, world_size: int, micro_batch_counts: tuple = (1, 2, 4, 8),
                       batch: int = 8, seq: int = 32, repeats: int = 3, warmup: int = 1,
                       config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    """Measured bubble (1 - sum compute / (p * makespan)) against the
    micro-batch count for both schedules at a fixed batch (more micro-batches
    means smaller ones); each point keeps its fastest repeat."""
    cfg = parallel_config(**(config_kwargs or {}))
    stage = PipelineStage(untied_reference_model(cfg), rank, world_size)
    rows = []
    for kind in SCHEDULES:
        for m in micro_batch_counts:
            if batch % m:
                continue
            _, _, micro, mi, mt = _split_batch(cfg, batch, seq, m)
            trials = []
            for _ in range(warmup + repeats):
                stage.zero_grad(set_to_none=True)
                clock = _Clock()
                comms.barrier()
                start = time.perf_counter()
                _, peak = run_pipeline_step(stage, rank, world_size, mi, mt, (micro, seq, cfg.n_embd),
                                            kind, clock)
                trials.append(dict(compute_seconds=clock.compute, comm_seconds=clock.comm,
                                   wall_seconds=time.perf_counter() - start, peak_stash=peak))
            best = min(trials[warmup:], key=lambda t: t["wall_seconds"])
            rows.append(dict(kind=kind, micro_batches=m, micro_batch_size=micro,
                             analytic_bubble=analytic_bubble(world_size, m), **best))
    return {"rank": rank, "world_size": world_size, "rows": rows}
