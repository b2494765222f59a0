"""Byte-level BPE tokenizer (GPT-2 scheme), plus a small BPE trainer.

Reference: src/transformer_internals/tokenizer.py:60-284. The pieces that must
be identical to produce GPT-2's ids are the published ones: the
pre-tokenisation regex, the reversible byte -> printable-character map, and
the merge rule (repeatedly merge the adjacent pair with the lowest rank).
Everything else is this module's own code.

* ``BPETokenizer(encoder, merges)``: ``encode`` / ``decode`` with a per-word
  cache, ``from_files(vocab.json, merges.txt)`` / ``from_pretrained(dir)``,
  ``<|endoftext|>`` as the end-of-text token when the vocabulary has it;
* ``train_bpe(texts, vocab_size)``: learns merges from a corpus (most frequent
  adjacent pair first, ties broken by the pair itself), so a usable tokenizer
  exists without the published files (this machine has no network), and
  ``save`` writes the GPT-2 file format that other tokenizers read.
"""

from __future__ import annotations

import json
from collections import Counter
from functools import lru_cache
from pathlib import Path
from typing import Iterable, Optional

import regex

__all__ = ["GPT2_SPLIT_PATTERN", "ENDOFTEXT", "bytes_to_unicode", "get_pairs", "BPETokenizer", "train_bpe"]

#: GPT-2's pre-tokenisation: contractions, optionally space-prefixed runs of
#: letters / digits / other symbols, then whitespace runs (a run of spaces
#: before a word leaves its last space to the word).
GPT2_SPLIT_PATTERN = r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"
ENDOFTEXT = "<|endoftext|>"


@lru_cache(maxsize=1)
def bytes_to_unicode() -> dict[int, str]:
    """Byte -> single printable, non-space character. The 188 bytes that are
    already printable Latin-1 characters map to themselves; the remaining 68
    map, in byte order, to the code points 256, 257, ..."""
    printable = set(range(ord("!"), ord("~") + 1)) | set(range(ord("¡"), ord("¬") + 1)) | \
        set(range(ord("®"), ord("ÿ") + 1))
    out, extra = {}, 0
    for b in range(256):
        if b in printable:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + extra)
            extra += 1
    return out


def get_pairs(word: tuple) -> set:
    """Set of adjacent symbol pairs of a word."""
    return {(word[i], word[i + 1]) for i in range(len(word) - 1)}


class BPETokenizer:
    def __init__(self, encoder: dict[str, int], bpe_merges: Iterable[tuple[str, str]]) -> None:
        self.encoder = dict(encoder)
        self.decoder = {i: s for s, i in self.encoder.items()}
        self.bpe_ranks = {tuple(m): r for r, m in enumerate(bpe_merges)}
        self.byte_encoder = bytes_to_unicode()
        self.byte_decoder = {c: b for b, c in self.byte_encoder.items()}
        self._pat = regex.compile(GPT2_SPLIT_PATTERN)
        self._cache: dict[str, tuple[str, ...]] = {}

    # ------------------------------------------------------------- loading --
    @classmethod
    def from_files(cls, vocab_path, merges_path) -> "BPETokenizer":
        encoder = json.loads(Path(vocab_path).read_text(encoding="utf-8"))
        merges = []
        for line in Path(merges_path).read_text(encoding="utf-8").splitlines():
            if not line or line.startswith("#version"):
                continue
            a, b = line.split(" ")
            merges.append((a, b))
        return cls(encoder, merges)

    @classmethod
    def from_pretrained(cls, model_dir) -> "BPETokenizer":
        d = Path(model_dir)
        return cls.from_files(d / "vocab.json", d / "merges.txt")

    def save(self, out_dir) -> Path:
        """Write vocab.json + merges.txt (GPT-2 layout)."""
        d = Path(out_dir)
        d.mkdir(parents=True, exist_ok=True)
        (d / "vocab.json").write_text(json.dumps(self.encoder, ensure_ascii=False), encoding="utf-8")
        merges = sorted(self.bpe_ranks.items(), key=lambda kv: kv[1])
        (d / "merges.txt").write_text("#version: 0.2\n" + "".join(f"{a} {b}\n" for (a, b), _ in merges),
                                      encoding="utf-8")
        return d

    # ---------------------------------------------------------------- core --
    def bpe(self, token: str) -> tuple[str, ...]:
        """Merge the symbols of one pre-token, lowest-ranked pair first."""
        hit = self._cache.get(token)
        if hit is not None:
            return hit
        word = tuple(token)
        ranks = self.bpe_ranks
        while len(word) > 1:
            best, best_rank = None, None
            for pair in zip(word, word[1:]):
                r = ranks.get(pair)
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = pair, r
            if best is None:
                break
            a, b = best
            merged, i, n = [], 0, len(word)
            while i < n:
                if i < n - 1 and word[i] == a and word[i + 1] == b:
                    merged.append(a + b)
                    i += 2
                else:
                    merged.append(word[i])
                    i += 1
            word = tuple(merged)
        if len(self._cache) < 100_000:
            self._cache[token] = word
        return word

    def _encode_chunk(self, text: str, out: list[int]) -> None:
        be, enc = self.byte_encoder, self.encoder
        for piece in self._pat.findall(text):
            mapped = "".join(be[b] for b in piece.encode("utf-8"))
            for sym in self.bpe(mapped):
                out.append(enc[sym])

    def encode(self, text: str, allow_special: bool = True) -> list[int]:
        """Text -> ids. ``<|endoftext|>`` in the text becomes the special id
        when the vocabulary has one and ``allow_special`` is set."""
        out: list[int] = []
        if allow_special and ENDOFTEXT in self.encoder and ENDOFTEXT in text:
            parts = text.split(ENDOFTEXT)
            for i, part in enumerate(parts):
                if i:
                    out.append(self.encoder[ENDOFTEXT])
                self._encode_chunk(part, out)
            return out
        self._encode_chunk(text, out)
        return out

    def decode(self, ids: Iterable[int], errors: str = "replace") -> str:
        text = "".join(self.decoder[int(i)] for i in ids)
        bd = self.byte_decoder
        data = bytearray()
        for ch in text:
            b = bd.get(ch)
            if b is None:  # a special token spelled outside the byte alphabet
                data.extend(ch.encode("utf-8"))
            else:
                data.append(b)
        return data.decode("utf-8", errors=errors)

    @property
    def eot_token_id(self) -> Optional[int]:
        return self.encoder.get(ENDOFTEXT)

    @property
    def vocab_size(self) -> int:
        return len(self.encoder)

    def __len__(self) -> int:
        return self.vocab_size


def train_bpe(texts: Iterable[str], vocab_size: int, add_endoftext: bool = True) -> BPETokenizer:
    """Learn a byte-level BPE vocabulary of ``vocab_size`` entries.

    Starts from the 256 byte symbols and repeatedly merges the most frequent
    adjacent pair inside pre-tokens (ties: the lexicographically largest
    pair), never across pre-token boundaries, exactly the structure GPT-2's
    merges have. Incremental pair counts keep it linear in merges x affected
    words rather than in merges x corpus.
    """
    be = bytes_to_unicode()
    pat = regex.compile(GPT2_SPLIT_PATTERN)
    freq: Counter = Counter()
    for t in texts:
        for piece in pat.findall(t):
            freq["".join(be[b] for b in piece.encode("utf-8"))] += 1
    words = [list(w) for w in freq]
    counts = list(freq.values())
    encoder = {be[b]: i for i, b in enumerate(range(256))}
    n_target = vocab_size - (1 if add_endoftext else 0)
    pair_count: Counter = Counter()
    where: dict[tuple, set] = {}
    for wi, w in enumerate(words):
        for p in zip(w, w[1:]):
            pair_count[p] += counts[wi]
            where.setdefault(p, set()).add(wi)
    merges: list[tuple[str, str]] = []
    while len(encoder) < n_target and pair_count:
        (a, b), c = max(pair_count.items(), key=lambda kv: (kv[1], kv[0]))
        if c <= 0:
            break
        merges.append((a, b))
        encoder[a + b] = len(encoder)
        for wi in list(where.get((a, b), ())):
            w = words[wi]
            for p in zip(w, w[1:]):
                pair_count[p] -= counts[wi]
                if pair_count[p] <= 0:
                    del pair_count[p]
            i, nw = 0, []
            while i < len(w):
                if i < len(w) - 1 and w[i] == a and w[i + 1] == b:
                    nw.append(a + b)
                    i += 2
                else:
                    nw.append(w[i])
                    i += 1
            words[wi] = nw
            for p in zip(nw, nw[1:]):
                pair_count[p] += counts[wi]
                where.setdefault(p, set()).add(wi)
        where.pop((a, b), None)
    if add_endoftext:
        encoder[ENDOFTEXT] = len(encoder)
    return BPETokenizer(encoder, merges)
