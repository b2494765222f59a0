"""Induction heads: where heads look, what they write, whether they are used.

Reference: src/transformer_internals/induction.py:75-572 (after Olsson et al.,
2022). On ``[BOS] X X`` with X random tokens (unpredictable from n-gram
statistics, so any skill on the second copy is copying):

* prefix-matching score: mean attention from second-copy position ``i`` to
  ``i - (T - 1)`` (the token after the previous occurrence); chance is
  1 / context;
* previous-token score: attention to ``i - 1`` (the other half of the
  circuit, which must sit in an earlier layer);
* copying score: how often the head's OV circuit ``W_U W_O W_V W_E`` maps a
  token to itself (top-1), optionally with the ln_1 / ln_f gains folded in;
* ablation score: rise in second-copy loss when the head's output is zeroed
  (the causal test);
* Spearman rank correlation with averaged ties, for comparing score maps.

B200 addition: the ablation sweep (n_layer * n_head forwards in the
reference) runs as batched forwards in which every sequence carries its own
head mask, so on a GPU the whole sweep is a handful of large batches.
"""

from __future__ import annotations

import math
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any, Optional

import torch
import torch.nn.functional as F

from .models.gpt import GPT

__all__ = ["rank_correlation", "InductionScores", "make_repeated_sequence", "prefix_matching_scores",
           "copying_scores", "ablated_head", "second_copy_loss", "ablation_scores",
           "in_context_learning_curve", "score_heads"]


def _avg_ranks(v: torch.Tensor) -> torch.Tensor:
    order = torch.argsort(v, stable=True)
    sv = v[order]
    ranks = torch.empty_like(v)
    i = 0
    n = len(sv)
    while i < n:
        j = i
        while j + 1 < n and sv[j + 1] == sv[i]:
            j += 1
        ranks[order[i:j + 1]] = (i + j) / 2.0 + 1.0
        i = j + 1
    return ranks


def rank_correlation(a: torch.Tensor, b: torch.Tensor) -> float:
    """Spearman correlation of two score maps (flattened; ties share the
    mean rank of the positions they span)."""
    if a.shape != b.shape:
        raise ValueError(f"shapes differ: {tuple(a.shape)} vs {tuple(b.shape)}")
    x = _avg_ranks(a.reshape(-1).double())
    y = _avg_ranks(b.reshape(-1).double())
    x, y = x - x.mean(), y - y.mean()
    den = torch.sqrt((x * x).sum() * (y * y).sum())
    return float((x * y).sum() / den) if den > 0 else 0.0


@dataclass
class InductionScores:
    prefix_matching: torch.Tensor
    previous_token: torch.Tensor
    copying: torch.Tensor
    copying_ln_folded: Optional[torch.Tensor] = None
    chance_level: float = 0.0
    ablation: Optional[torch.Tensor] = None
    baseline_second_copy_loss: float = float("nan")
    meta: dict = field(default_factory=dict)

    def top_heads(self, k: int = 10, key: str = "prefix_matching") -> list[dict]:
        s = getattr(self, key)
        nh = s.shape[1]
        out = []
        for i in torch.argsort(s.reshape(-1), descending=True)[:k].tolist():
            L, H = divmod(i, nh)
            out.append({"layer": L, "head": H, "name": f"L{L}H{H}",
                        "prefix_matching": float(self.prefix_matching[L, H]),
                        "previous_token": float(self.previous_token[L, H]), "copying": float(self.copying[L, H]),
                        "ablation": float(self.ablation[L, H]) if self.ablation is not None else None})
        return out

    def to_dict(self) -> dict:
        f = self.copying_ln_folded
        return {"prefix_matching": self.prefix_matching.tolist(), "previous_token": self.previous_token.tolist(),
                "copying": self.copying.tolist(), "copying_ln_folded": f.tolist() if f is not None else None,
                "copying_ln_fold_rank_correlation": rank_correlation(self.copying, f) if f is not None else None,
                "chance_level": self.chance_level,
                "ablation": self.ablation.tolist() if self.ablation is not None else None,
                "baseline_second_copy_loss": self.baseline_second_copy_loss, "meta": self.meta}


def _band(vocab: int, low: Optional[int], high: Optional[int]) -> tuple[int, int]:
    if low is None:
        low = 1000 if vocab > 20000 else max(1, vocab // 10)
    if high is None:
        high = 20000 if vocab > 20000 else vocab
    if high > vocab or low >= high:
        raise ValueError(f"token band [{low}, {high}) does not fit vocab {vocab}")
    return low, high


def make_repeated_sequence(batch_size: int, seq_len: int, vocab_size: int, bos_token_id: int,
                           generator: Optional[torch.Generator] = None, low: Optional[int] = None,
                           high: Optional[int] = None) -> torch.Tensor:
    """(B, 2T + 1): BOS then a random block twice. Tokens come from a band of
    ordinary ids (GPT-2: [1000, 20000)) so unigram priors cannot help."""
    lo, hi = _band(vocab_size, low, high)
    block = torch.randint(lo, hi, (batch_size, seq_len), generator=generator)
    return torch.cat([torch.full((batch_size, 1), bos_token_id, dtype=torch.long), block, block], dim=1)


def _bos(model: GPT) -> int:
    return 50256 if model.config.vocab_size > 50256 else 0


def _probe(model: GPT, seq_len: int, batch_size: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return make_repeated_sequence(batch_size, seq_len, model.config.vocab_size, _bos(model), g).to(device)


@torch.no_grad()
def prefix_matching_scores(model: GPT, seq_len: int = 60, batch_size: int = 8, seed: int = 0, device="cpu"):
    """(prefix_matching, previous_token, chance_level, sequences)."""
    seqs = _probe(model, seq_len, batch_size, seed, device)
    atts = model(seqs, need_weights=True)["attentions"]
    q = 1 + seq_len + torch.arange(seq_len - 1)

    def mean_at(offset):
        return torch.stack([a[:, :, q, q - offset].mean(dim=(0, 2)) for a in atts]).cpu()

    chance = float((1.0 / (q.float() + 1.0)).mean())
    return mean_at(seq_len - 1), mean_at(1), chance, seqs.cpu()


@torch.no_grad()
def copying_scores(model: GPT, n_tokens: int = 2000, seed: int = 0, top_k: int = 1, device="cpu",
                   fold_ln: bool = False) -> torch.Tensor:
    """(n_layer, n_head) fraction of sampled tokens each OV circuit maps to
    itself (within top-k)."""
    cfg = model.config
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, cfg.vocab_size, (n_tokens,), generator=g)
    wte = model.wte.weight.detach().to(device)
    E = wte[toks.to(device)]
    U = wte.t()
    if fold_ln:
        U = U * model.ln_f.weight.detach().to(device)[:, None]
    hd, C = cfg.head_dim, cfg.n_embd
    kv = cfg.kv_heads * hd
    out = torch.zeros(cfg.n_layer, cfg.n_head)
    for L, blk in enumerate(model.h):
        Wv = blk.attn.c_attn.weight.detach().to(device)[C + kv:C + 2 * kv]
        bv = blk.attn.c_attn.bias.detach().to(device)[C + kv:C + 2 * kv] if blk.attn.c_attn.bias is not None \
            else torch.zeros(kv, device=device)
        Wo = blk.attn.c_proj.weight.detach().to(device)
        e = E * blk.ln_1.weight.detach().to(device) if fold_ln else E
        rep = cfg.n_head // cfg.kv_heads
        for H in range(cfg.n_head):
            vs = slice((H // rep) * hd, (H // rep + 1) * hd)
            logits = ((e @ Wv[vs].t() + bv[vs]) @ Wo[:, H * hd:(H + 1) * hd].t()) @ U
            top = logits.topk(top_k, dim=-1).indices.cpu()
            out[L, H] = (top == toks[:, None]).any(dim=1).float().mean()
    return out


@contextmanager
def ablated_head(model: GPT, layer: int, head: int):
    """Zero one head's output into the residual stream (its pattern unchanged)."""
    attn = model.h[layer].attn
    prev = attn.head_mask
    m = torch.ones(model.config.n_head) if prev is None else prev.detach().clone().float()
    m[..., head] = 0.0
    attn.head_mask = m
    try:
        yield model
    finally:
        attn.head_mask = prev


def _second_copy_losses(logits: torch.Tensor, seqs: torch.Tensor, seq_len: int) -> torch.Tensor:
    """Per-sequence mean loss over the second copy."""
    x, y = logits[:, :-1], seqs[:, 1:]
    l = F.cross_entropy(x.reshape(-1, x.size(-1)).float(), y.reshape(-1), reduction="none").view(y.shape)
    return l[:, seq_len:2 * seq_len - 1].mean(dim=1)


@torch.no_grad()
def second_copy_loss(model: GPT, seqs: torch.Tensor, seq_len: int) -> float:
    return float(_second_copy_losses(model(seqs)["logits"], seqs, seq_len).mean())


@torch.no_grad()
def ablation_scores(model: GPT, seq_len: int = 60, batch_size: int = 8, seed: int = 0, device="cpu",
                    heads_per_forward: Optional[int] = None):
    """(delta second-copy loss per head, baseline loss). Every head is
    scored on the same sequences; ``heads_per_forward`` ablations share one
    batched forward via per-sequence head masks (default: all on CUDA, one
    at a time on CPU)."""
    cfg = model.config
    seqs = _probe(model, seq_len, batch_size, seed, device)
    base = second_copy_loss(model, seqs, seq_len)
    heads = [(L, H) for L in range(cfg.n_layer) for H in range(cfg.n_head)]
    if heads_per_forward is None:
        heads_per_forward = len(heads) if torch.device(device).type == "cuda" else 1
    deltas = torch.zeros(cfg.n_layer, cfg.n_head)
    prev = [b.attn.head_mask for b in model.h]
    try:
        for s in range(0, len(heads), heads_per_forward):
            group = heads[s:s + heads_per_forward]
            n = len(group)
            for L, blk in enumerate(model.h):
                m = torch.ones(n, batch_size, cfg.n_head, device=device)
                for i, (l2, h2) in enumerate(group):
                    if l2 == L:
                        m[i, :, h2] = 0.0
                blk.attn.head_mask = m.reshape(n * batch_size, cfg.n_head)
            big = seqs.repeat(n, 1)
            per = _second_copy_losses(model(big)["logits"], big, seq_len).view(n, batch_size).mean(dim=1)
            for i, (L, H) in enumerate(group):
                deltas[L, H] = float(per[i]) - base
    finally:
        for b, p in zip(model.h, prev):
            b.attn.head_mask = p
    return deltas, base


@torch.no_grad()
def in_context_learning_curve(model: GPT, seq_len: int = 60, batch_size: int = 16, seed: int = 0,
                              device="cpu") -> dict[str, Any]:
    """Per-position loss on [BOS] X X; the induction bump is first-copy
    minus second-copy loss (nats)."""
    seqs = _probe(model, seq_len, batch_size, seed, device)
    logits = model(seqs)["logits"]
    x, y = logits[:, :-1], seqs[:, 1:]
    l = F.cross_entropy(x.reshape(-1, x.size(-1)).float(), y.reshape(-1), reduction="none").view(y.shape)
    per = l.mean(0).cpu()
    first, second = per[:seq_len - 1].mean().item(), per[seq_len:2 * seq_len - 1].mean().item()
    lo, hi = _band(model.config.vocab_size, None, None)
    return {"per_position_loss": per.tolist(), "first_copy_loss": first, "second_copy_loss": second,
            "induction_bump_nats": first - second, "uniform_band_loss": math.log(hi - lo),
            "seq_len": seq_len, "batch_size": batch_size}


def score_heads(model: GPT, seq_len: int = 60, batch_size: int = 8, n_copy_tokens: int = 2000, seed: int = 0,
                device="cpu", with_ablation: bool = True) -> InductionScores:
    model = model.to(device).eval()
    pm, prev, chance, _ = prefix_matching_scores(model, seq_len, batch_size, seed, device)
    cp = copying_scores(model, n_copy_tokens, seed, device=device)
    cpf = copying_scores(model, n_copy_tokens, seed, device=device, fold_ln=True)
    abl, base = (ablation_scores(model, seq_len, batch_size, seed, device) if with_ablation
                 else (None, float("nan")))
    return InductionScores(pm, prev, cp, cpf, chance, abl, base,
                           {"seq_len": seq_len, "batch_size": batch_size, "n_copy_tokens": n_copy_tokens,
                            "seed": seed})
