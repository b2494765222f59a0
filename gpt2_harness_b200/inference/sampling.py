"""Sampling filters and KV-cached generation on the oracle model.

Reference semantics: src/transformer_internals/sampling.py:29-181.

* ``apply_temperature`` rejects T <= 0 (greedy is its own exact path);
* ``top_k_filter`` keeps the k largest logits (ties at the k-th value kept),
  no-op for k <= 0 or k >= vocab;
* ``top_p_filter`` keeps the smallest prefix of the descending order whose
  mass reaches p: a token is dropped only when the mass strictly before it
  already exceeds p, so the argmax always survives;
* ``generate`` encodes the prompt once, then feeds one token per step through
  the cache; stops on EOS (finished rows keep emitting EOS) or at the
  context limit, since learned positions do not extrapolate.

The B200 decode path with the same stopping rules is
:class:`gpt2_harness_b200.inference.decode.DecodeEngine`.
"""

from __future__ import annotations

import torch

from ..models.gpt import GPT, KVCache

__all__ = ["apply_temperature", "top_k_filter", "top_p_filter", "sample_next", "generate"]


def apply_temperature(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    if temperature <= 0:
        raise ValueError("temperature must be > 0; use do_sample=False for greedy decoding")
    return logits / temperature


def top_k_filter(logits: torch.Tensor, k: int) -> torch.Tensor:
    vocab = logits.size(-1)
    if k <= 0 or k >= vocab:
        return logits
    threshold = logits.topk(k, dim=-1).values[..., -1:]
    return torch.where(logits < threshold, torch.full_like(logits, float("-inf")), logits)


def top_p_filter(logits: torch.Tensor, p: float) -> torch.Tensor:
    if p >= 1.0:
        return logits
    if p <= 0.0:
        raise ValueError("top_p must be in (0, 1]")
    order = logits.argsort(dim=-1, descending=True)
    sorted_logits = logits.gather(-1, order)
    probs = sorted_logits.softmax(dim=-1)
    mass_before = probs.cumsum(dim=-1) - probs
    drop_sorted = mass_before > p
    drop_sorted[..., 0] = False
    drop = torch.empty_like(drop_sorted).scatter_(-1, order, drop_sorted)
    return logits.masked_fill(drop, float("-inf"))


def sample_next(logits: torch.Tensor, *, do_sample: bool, temperature: float = 1.0, top_k: int = 0,
                top_p: float = 1.0, generator: torch.Generator | None = None) -> torch.Tensor:
    """(B, V) logits -> (B, 1) next tokens (argmax, or filtered multinomial)."""
    if not do_sample:
        return logits.argmax(dim=-1, keepdim=True)
    logits = top_p_filter(top_k_filter(apply_temperature(logits, temperature), top_k), top_p)
    probs = logits.float().softmax(dim=-1)
    if generator is not None and generator.device != probs.device:
        return torch.multinomial(probs.cpu(), 1, generator=generator).to(probs.device)
    return torch.multinomial(probs, 1, generator=generator)


@torch.no_grad()
def generate(model: GPT, idx: torch.Tensor, max_new_tokens: int, *, do_sample: bool = False,
             temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0, eos_token_id: int | None = None,
             use_cache: bool = True, generator: torch.Generator | None = None) -> torch.Tensor:
    """(B, T) prompt -> (B, T + n) with n <= max_new_tokens."""
    was_training = model.training
    model.eval()
    try:
        limit = model.config.n_positions
        cache = KVCache.empty(model.config.n_layer) if use_cache else None
        done = torch.zeros(idx.size(0), dtype=torch.bool, device=idx.device)
        fed = 0  # tokens already inside the cache
        for _ in range(max_new_tokens):
            if idx.size(1) >= limit:
                break
            if cache is not None:
                step_in = idx[:, fed:]
                fed = idx.size(1)
            else:
                step_in = idx[:, -limit:]
            logits = model(step_in, cache=cache)["logits"][:, -1, :]
            nxt = sample_next(logits, do_sample=do_sample, temperature=temperature, top_k=top_k,
                              top_p=top_p, generator=generator)
            if eos_token_id is not None:
                nxt = nxt.masked_fill(done.unsqueeze(1), eos_token_id)
                done |= nxt.squeeze(1) == eos_token_id
            idx = torch.cat([idx, nxt], dim=1)
            if eos_token_id is not None and bool(done.all()):
                break
        return idx
    finally:
        model.train(was_training)
