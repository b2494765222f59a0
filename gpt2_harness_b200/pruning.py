"""Structured pruning of attention heads and MLP neurons by gradient-of-mask
importance (Michel et al., 2019, "Are Sixteen Heads Really Better than One?").

Reference: src/transformer_internals/pruning.py:57-349.

A multiplicative mask of ones is attached to each head's output (resp. each
hidden unit of the MLP); the importance of a unit is the accumulated
|d loss / d mask| over deterministic calibration batches, optionally
normalised per layer (L2) so scores compare across depth. Pruning keeps the
globally highest-scoring ``1 - sparsity`` fraction. Masks are applied
temporarily (``pruned`` context manager) so every sparsity is evaluated on
the same weights, and the parameters a real pruning would delete are counted
exactly (head: 4 * head_dim * n_embd weights + 3 * head_dim biases; neuron:
2 * n_embd weights + 1 bias).
"""

from __future__ import annotations

import math
from contextlib import contextmanager
from dataclasses import asdict, dataclass
from typing import Callable, Optional

import torch
import torch.nn.functional as F

from .models.gpt import GPT

__all__ = ["head_importance", "neuron_importance", "pruned", "keep_mask", "params_removed_by_head_pruning",
           "params_removed_by_neuron_pruning", "PruneResult", "prune_sweep"]


def _importance(model: GPT, dataset, n_batches: int, batch_size: int, device, normalize: bool, kind: str):
    model = model.to(device).eval()
    cfg = model.config
    width = cfg.n_head if kind == "heads" else 4 * cfg.n_embd
    masks = []
    for blk in model.h:
        m = torch.ones(width, device=device, requires_grad=True)
        if kind == "heads":
            blk.attn.head_mask = m
        else:
            blk.mlp.neuron_mask = m
        masks.append(m)
    scores = torch.zeros(cfg.n_layer, width)
    try:
        for x, y in dataset.sequential_batches("train", batch_size=batch_size, limit=n_batches):
            model.zero_grad(set_to_none=True)
            grads = torch.autograd.grad(model(x.to(device), targets=y.to(device))["loss"], masks,
                                        allow_unused=True)
            for l, g in enumerate(grads):
                if g is not None:
                    scores[l] += g.detach().abs().cpu()
    finally:
        for blk in model.h:
            if kind == "heads":
                blk.attn.head_mask = None
            else:
                blk.mlp.neuron_mask = None
        model.zero_grad(set_to_none=True)
    if normalize:
        scores = scores / scores.norm(dim=1, keepdim=True).clamp_min(1e-12)
    return scores


def head_importance(model: GPT, dataset, n_batches: int = 4, batch_size: int = 4, device="cpu",
                    normalize_per_layer: bool = True) -> torch.Tensor:
    """(n_layer, n_head) importance, higher = more important."""
    return _importance(model, dataset, n_batches, batch_size, device, normalize_per_layer, "heads")


def neuron_importance(model: GPT, dataset, n_batches: int = 4, batch_size: int = 4, device="cpu",
                      normalize_per_layer: bool = True) -> torch.Tensor:
    """(n_layer, 4 * n_embd) importance."""
    return _importance(model, dataset, n_batches, batch_size, device, normalize_per_layer, "neurons")


@contextmanager
def pruned(model: GPT, head_mask: Optional[torch.Tensor] = None, neuron_mask: Optional[torch.Tensor] = None):
    old = [(b.attn.head_mask, b.mlp.neuron_mask) for b in model.h]
    try:
        for i, b in enumerate(model.h):
            if head_mask is not None:
                b.attn.head_mask = head_mask[i]
            if neuron_mask is not None:
                b.mlp.neuron_mask = neuron_mask[i]
        yield model
    finally:
        for b, (h, n) in zip(model.h, old):
            b.attn.head_mask, b.mlp.neuron_mask = h, n


def keep_mask(scores: torch.Tensor, sparsity: float) -> torch.Tensor:
    """0/1 mask removing the ``round(sparsity * numel)`` lowest scores
    (ranked globally across layers)."""
    flat = scores.reshape(-1)
    m = torch.ones_like(flat)
    k = round(sparsity * flat.numel())
    if k > 0:
        m[flat.argsort()[:k]] = 0.0
    return m.view_as(scores)


def params_removed_by_head_pruning(model: GPT, mask: torch.Tensor) -> int:
    c = model.config
    per = 4 * c.head_dim * c.n_embd + (3 * c.head_dim if c.attn_bias else 0)
    return int((mask == 0).sum()) * per


def params_removed_by_neuron_pruning(model: GPT, mask: torch.Tensor) -> int:
    c = model.config
    return int((mask == 0).sum()) * (2 * c.n_embd + (1 if c.mlp_bias else 0))


@dataclass
class PruneResult:
    kind: str
    sparsity: float
    val_loss: float
    val_ppl: float
    params_removed: int
    params_total: int
    induction_second_copy_loss: Optional[float] = None

    def to_dict(self) -> dict:
        d = asdict(self)
        d["fraction_removed"] = self.params_removed / self.params_total
        return d


@torch.no_grad()
def _loss(model, batches, device) -> float:
    tot, n = 0.0, 0
    for x, y in batches:
        lo = model(x.to(device))["logits"].float().cpu()
        tot += F.cross_entropy(lo.reshape(-1, lo.size(-1)), y.reshape(-1), reduction="sum").item()
        n += y.numel()
    return tot / n


def prune_sweep(model: GPT, dataset, sparsities, kind: str = "heads", n_eval_batches: int = 6,
                batch_size: int = 4, device="cpu", importance: Optional[torch.Tensor] = None,
                induction_probe: Optional[Callable] = None):
    """Quality at each sparsity; returns (results, importance)."""
    if kind not in ("heads", "neurons"):
        raise ValueError(f"kind must be 'heads' or 'neurons', got {kind!r}")
    model = model.to(device).eval()
    if importance is None:
        importance = (head_importance if kind == "heads" else neuron_importance)(model, dataset, device=device)
    evals = dataset.sequential_batches("val", batch_size=batch_size, limit=n_eval_batches)
    total = sum(p.numel() for p in {id(p): p for p in model.parameters()}.values())
    out = []
    for s in sparsities:
        m = keep_mask(importance, s)
        with pruned(model, **({"head_mask": m} if kind == "heads" else {"neuron_mask": m})):
            loss = _loss(model, evals, device)
            probe = float(induction_probe(model)) if induction_probe is not None else None
        removed = (params_removed_by_head_pruning if kind == "heads" else params_removed_by_neuron_pruning)(model, m)
        out.append(PruneResult(kind, s, loss, math.exp(min(loss, 20.0)), removed, total, probe))
    return out, importance
