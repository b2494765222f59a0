"""Rank-local device binding and determinism helpers for the strategy workers.

Reference: src/transformer_internals/parallel/common.py:52-167. Every rank
builds an identical model / batch on the CPU from a seed and only then moves
it to its device, so weights never depend on a device RNG; byte accounting
counts distinct storages once.
"""

from __future__ import annotations

import resource
import sys
from contextlib import contextmanager
from typing import Any, Iterator, Optional

import torch

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.gpt import GPT, Block

__all__ = [
    "current_device",
    "set_device",
    "device_scope",
    "parallel_config",
    "identical_model",
    "identical_block",
    "identical_batch",
    "state_bytes",
    "max_rss_bytes",
]

_DEVICE = torch.device("cpu")


def current_device() -> torch.device:
    return _DEVICE


def set_device(device) -> torch.device:
    global _DEVICE
    _DEVICE = torch.device(device) if device is not None else torch.device("cpu")
    if _DEVICE.type == "cuda":
        torch.cuda.set_device(_DEVICE)
    return _DEVICE


@contextmanager
def device_scope(device) -> Iterator[torch.device]:
    prev = _DEVICE
    try:
        yield set_device(device)
    finally:
        set_device(prev)


def parallel_config(**overrides: Any) -> GPTConfig:
    """The toy shape every equivalence worker uses by default: vocab 128,
    context 64, 4 layers, 4 heads, width 32, no dropout (the reference's
    parallel_config; its byte closed forms are quoted at this size)."""
    base = dict(vocab_size=128, n_positions=64, n_layer=4, n_head=4, n_embd=32, dropout=0.0)
    base.update(overrides)
    return GPTConfig(**base)


def identical_model(config: GPTConfig, seed: int = 0) -> GPT:
    """The same GPT on every rank: built on CPU under `seed`, then moved."""
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        model = GPT(config)
    return model.to(current_device())


def identical_block(config: GPTConfig, seed: int = 0, layer_idx: int = 0) -> Block:
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        blk = Block(config, layer_idx=layer_idx)
    return blk.to(current_device())


def identical_batch(config: GPTConfig, batch: int, seq: int, seed: int = 0):
    """(idx, targets) drawn uniformly from the vocabulary on the CPU."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, config.vocab_size, (batch, seq + 1), generator=g)
    dev = current_device()
    return x[:, :-1].contiguous().to(dev), x[:, 1:].contiguous().to(dev)


def state_bytes(tensors: Any) -> int:
    """Bytes of distinct storages among `tensors` (a tensor, module, or
    iterable of tensors/None); tied or aliased tensors count once."""
    if isinstance(tensors, torch.nn.Module):
        tensors = list(tensors.parameters()) + list(tensors.buffers())
    elif isinstance(tensors, torch.Tensor):
        tensors = [tensors]
    seen: set = set()
    total = 0
    for t in tensors:
        if t is None:
            continue
        st = t.untyped_storage()
        key = (st.data_ptr(), t.device.type, t.device.index)
        if key in seen:
            continue
        seen.add(key)
        total += st.nbytes()
    return total


def max_rss_bytes() -> int:
    """Peak resident set size of this process in bytes."""
    r = resource.getrusage(resource.RUSAGE_SELF).ru_maxrss
    return int(r if sys.platform == "darwin" else r * 1024)
