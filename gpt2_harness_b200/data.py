"""Text corpus -> token stream -> (input, target) windows.

Reference: src/transformer_internals/data.py:46-274 (TinyStories text, BPE
encode with an on-disk cache keyed by a content hash, random-crop
``TokenDataset`` with a contiguous tail validation split, deterministic
non-overlapping windows for perplexity, and a compact vocabulary of the most
frequent ids with id 0 as ``<unk>``).

This machine has no network, so :func:`load_text` reads a local file
(argument, ``$G2B_CORPUS``, or a cached TinyStories download) and
:func:`synthetic_stories` provides a deterministic, TinyStories-shaped corpus
for offline runs and tests. Batches can be staged in pinned host memory so the
host->device copy is an asynchronous DMA.
"""

from __future__ import annotations

import hashlib
import os
import random
from pathlib import Path
from typing import Optional

import numpy as np
import torch

__all__ = ["DEFAULT_DATA_DIR", "load_text", "synthetic_stories", "encode_corpus", "TokenDataset",
           "compact_vocabulary"]

DEFAULT_DATA_DIR = Path("data")


def load_text(path: Optional[str] = None, max_chars: Optional[int] = 8_000_000) -> str:
    """Corpus text from ``path``, ``$G2B_CORPUS`` or a local TinyStories copy."""
    cands = [p for p in (path, os.environ.get("G2B_CORPUS")) if p]
    hub = Path(os.environ.get("HF_HOME", Path.home() / ".cache/huggingface")) / "hub"
    ts = hub / "datasets--roneneldan--TinyStories" / "snapshots"
    if ts.is_dir():
        cands += [str(p / "TinyStories-valid.txt") for p in sorted(ts.iterdir())]
    for c in cands:
        if Path(c).exists():
            text = Path(c).read_text(encoding="utf-8", errors="replace")
            return text if max_chars is None else text[:max_chars]
    raise FileNotFoundError("no corpus text found (pass a path or set G2B_CORPUS); "
                            "synthetic_stories() gives an offline corpus")


_NAMES = ["Lily", "Tom", "Mia", "Ben", "Sara", "Max", "Anna", "Leo", "Zoe", "Sam"]
_ANIMALS = ["dog", "cat", "bird", "bunny", "frog", "duck", "bear", "fish"]
_PLACES = ["park", "garden", "forest", "beach", "house", "school", "pond", "farm"]
_THINGS = ["ball", "kite", "box", "flower", "toy car", "red hat", "book", "cake"]
_FEEL = ["happy", "sad", "excited", "scared", "tired", "proud", "curious", "angry"]


def synthetic_stories(n_stories: int = 2000, seed: int = 0) -> str:
    """Deterministic short stories with TinyStories' vocabulary and shape:
    named characters, a place, a problem, a resolution, repeated structure
    (so a small model has something learnable, including copying)."""
    rng = random.Random(seed)
    out = []
    for _ in range(n_stories):
        a, b = rng.sample(_NAMES, 2)
        an, pl, th = rng.choice(_ANIMALS), rng.choice(_PLACES), rng.choice(_THINGS)
        f1, f2 = rng.sample(_FEEL, 2)
        s = [f"Once upon a time, there was a little {rng.choice(['girl', 'boy'])} named {a}.",
             f"{a} liked to play with a {th} in the {pl}.",
             f"One day, {a} saw a {an} near the {pl}. The {an} was {f1}.",
             f"\"Why are you {f1}?\" asked {a}. The {an} said, \"I lost my {th}.\"",
             f"{a} and {b} looked everywhere for the {th}.",
             f"At last, {b} found the {th} under a big tree.",
             f"The {an} was {f2} and said, \"Thank you, {a} and {b}!\"",
             f"From that day on, {a}, {b} and the {an} played in the {pl} every day."]
        out.append(" ".join(s))
    return "\n\n".join(out) + "\n\n"


def encode_corpus(tokenizer, text: Optional[str] = None, data_dir=DEFAULT_DATA_DIR,
                  max_chars: Optional[int] = 8_000_000, cache: bool = True) -> np.ndarray:
    """Tokenize (paragraph by paragraph, so no BPE word is cut at a chunk
    boundary) and cache as .npy keyed by text length, head and vocab size."""
    if text is None:
        text = load_text(max_chars=max_chars)
    key = hashlib.sha256(f"{len(text)}|{text[:4096]}|{tokenizer.vocab_size}".encode()).hexdigest()[:16]
    path = Path(data_dir) / f"tokens_{key}.npy"
    if cache and path.exists():
        return np.load(path)
    ids: list[int] = []
    for para in text.split("\n\n"):
        if para:
            ids.extend(tokenizer.encode(para + "\n\n"))
    arr = np.asarray(ids, dtype=np.uint16 if tokenizer.vocab_size < 65536 else np.int32)
    if cache:
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(".tmp.npy")
        np.save(tmp, arr)
        os.replace(tmp, path)
    return arr


class TokenDataset:
    """Flat token stream sliced into (x, y) windows of ``block_size``; the
    last ``val_fraction`` of the stream is the validation split (contiguous,
    so no window straddles train and val)."""

    def __init__(self, tokens: np.ndarray, block_size: int, val_fraction: float = 0.1) -> None:
        tokens = np.asarray(tokens)
        if tokens.ndim != 1:
            raise ValueError(f"expected a 1-D token stream, got shape {tokens.shape}")
        n_val = int(len(tokens) * val_fraction)
        if len(tokens) - n_val <= block_size + 1:
            raise ValueError(f"corpus of {len(tokens)} tokens is too short for block_size={block_size}")
        self.block_size = block_size
        self.train = tokens[: len(tokens) - n_val]
        self.val = tokens[len(tokens) - n_val:]
        self._pinned: dict = {}

    def _split(self, split: str) -> np.ndarray:
        if split not in ("train", "val"):
            raise ValueError(f"unknown split {split!r}")
        return self.train if split == "train" else self.val

    def get_batch(self, split: str, batch_size: int, device="cpu", generator: Optional[torch.Generator] = None,
                  pin: bool = False):
        """Random crops (with replacement). ``generator`` makes two runs see
        identical batches; ``pin`` stages them in reusable pinned buffers and
        copies asynchronously to a CUDA ``device``."""
        data = self._split(split)
        T = self.block_size
        starts = torch.randint(len(data) - T - 1, (batch_size,), generator=generator).numpy()
        win = data[starts[:, None] + np.arange(T + 1)[None, :]].astype(np.int64)
        dev = torch.device(device)
        if pin and dev.type == "cuda":
            # two (x, y) pinned pairs used alternately; a pair is refilled only
            # after the device copy that last read it has completed
            key = (split, batch_size)
            ring = self._pinned.get(key)
            if ring is None:
                ring = self._pinned[key] = {"i": 0, "pairs": [
                    [torch.empty(batch_size, T, dtype=torch.int64).pin_memory() for _ in range(2)] + [None]
                    for _ in range(2)]}
            pair = ring["pairs"][ring["i"]]
            ring["i"] ^= 1
            if pair[2] is not None:
                pair[2].synchronize()
            w = torch.from_numpy(win)
            pair[0].copy_(w[:, :-1])
            pair[1].copy_(w[:, 1:])
            x, y = pair[0].to(dev, non_blocking=True), pair[1].to(dev, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            pair[2] = ev
            return x, y
        b = torch.from_numpy(win)
        return b[:, :-1].contiguous().to(dev), b[:, 1:].contiguous().to(dev)

    def sequential_batches(self, split: str, batch_size: int, limit: Optional[int] = None) -> list:
        """Non-overlapping windows in order (every token predicted once):
        the perplexity estimator."""
        data = self._split(split)
        T = self.block_size
        n_win = (len(data) - 1) // T
        out, rows = [], []
        for w in range(n_win):
            rows.append(data[w * T: w * T + T + 1].astype(np.int64))
            if len(rows) == batch_size:
                b = torch.from_numpy(np.stack(rows))
                out.append((b[:, :-1].contiguous(), b[:, 1:].contiguous()))
                rows = []
                if limit is not None and len(out) >= limit:
                    break
        return out


def compact_vocabulary(tokens: np.ndarray, vocab_size: int = 4096) -> tuple[np.ndarray, np.ndarray, float]:
    """Remap onto the ``vocab_size - 1`` most frequent ids (+ id 0 = <unk>).

    Returns (remapped int32 stream, id_map with id_map[0] = -1 and
    id_map[c] = original id of compact id c, coverage = kept occurrences /
    all occurrences)."""
    if vocab_size < 2:
        raise ValueError("vocab_size must be at least 2")
    t = np.asarray(tokens).astype(np.int64)
    counts = np.bincount(t)
    order = np.argsort(-counts, kind="stable")[: vocab_size - 1]
    order = order[counts[order] > 0]
    lut = np.zeros(len(counts), dtype=np.int32)
    lut[order] = np.arange(1, len(order) + 1, dtype=np.int32)
    coverage = float(counts[order].sum() / max(1, counts.sum()))
    return lut[t], np.concatenate([[-1], order]).astype(np.int64), coverage
