"""Byte-level BPE: byte map, merge order, lossless round trips, and id-for-id
agreement with HuggingFace's GPT-2 tokenizer on a vocabulary trained here
(the published GPT-2 files need a network this machine does not have)."""

import json

import pytest

from gpt2_harness_b200.tokenizer import ENDOFTEXT, BPETokenizer, bytes_to_unicode, get_pairs, train_bpe

SAMPLES = [
    "Hello, world!", "  leading and trailing spaces  ", "multiple   internal    spaces",
    "newlines\nand\ttabs\r\n", "emoji 🌍🚀 and CJK 你好世界 and Cyrillic Привет",
    "punctuation!?...,;:'\"()[]{}<>/\\|@#$%^&*", "numbers 0123456789 and 3.14159 and 1,000,000",
    "def f(x):\n    return x ** 2  # comment", "", "a", " ", "\x00\x01\x02 control bytes \x7f",
    "MixedCASE camelCase snake_case SCREAMING_SNAKE", "ünïcödé àccênts and ß ligatures œ æ",
    "it's they're we've I'm you'll he'd",
]

CORPUS = [
    "Once upon a time there was a little girl named Lily. She liked to play outside in the sun.",
    "One day, Lily's mom said they're going to the park. Lily was very happy and said \"Yay!\"",
    "The dog ran to the tree, and the cat ran to the house. It's 3.14 o'clock, 1,000,000 times.",
] * 20


def test_byte_map_bijection():
    m = bytes_to_unicode()
    assert len(m) == 256 and len(set(m.values())) == 256
    assert all(len(v) == 1 and not v.isspace() for v in m.values())
    assert m[ord("A")] == "A" and m[ord(" ")] == chr(256 + 32)


def test_get_pairs():
    assert get_pairs(("a", "b", "c")) == {("a", "b"), ("b", "c")}
    assert get_pairs(("a",)) == set()
    assert get_pairs(("a", "b", "a", "b")) == {("a", "b"), ("b", "a")}


def test_byte_only_tokenizer_roundtrips():
    enc = {ch: i for i, ch in enumerate(bytes_to_unicode().values())}
    tok = BPETokenizer(enc, [])
    for s in SAMPLES:
        assert tok.decode(tok.encode(s)) == s


def test_merges_in_rank_order():
    enc = {ch: i for i, ch in enumerate(bytes_to_unicode().values())}
    enc["ab"], enc["abc"] = 300, 301
    tok = BPETokenizer(enc, [("a", "b"), ("ab", "c")])
    assert tok.encode("abc") == [301] and tok.decode([301]) == "abc"
    assert len(tok.encode("acb")) == 3


def test_trained_tokenizer_roundtrips_and_compresses(tmp_path):
    tok = train_bpe(CORPUS, 400)
    assert tok.vocab_size <= 400 and tok.eot_token_id == tok.vocab_size - 1
    for s in SAMPLES + CORPUS[:3]:
        assert tok.decode(tok.encode(s)) == s
    text = CORPUS[0]
    assert len(tok.encode(text)) < 0.6 * len(text.encode("utf-8"))
    ids = tok.encode("a" + ENDOFTEXT + "b")
    assert ids[1] == tok.eot_token_id
    tok.save(tmp_path)
    again = BPETokenizer.from_pretrained(tmp_path)
    assert again.encode(text) == tok.encode(text)
    assert json.loads((tmp_path / "vocab.json").read_text(encoding="utf-8")) == tok.encoder


def test_ids_match_huggingface_byte_level_bpe(tmp_path):
    """HuggingFace's GPT-2 tokenizer is a BPE model behind a byte-level
    pre-tokenizer (no prefix space); built from the same files, it must give
    the same ids, which checks the split regex, byte map and merge order."""
    tokenizers = pytest.importorskip("tokenizers")
    tok = train_bpe(CORPUS, 420)
    tok.save(tmp_path)
    ref = tokenizers.Tokenizer(tokenizers.models.BPE.from_file(str(tmp_path / "vocab.json"),
                                                               str(tmp_path / "merges.txt")))
    ref.pre_tokenizer = tokenizers.pre_tokenizers.ByteLevel(add_prefix_space=False)
    for s in SAMPLES + CORPUS[:3]:
        assert tok.encode(s, allow_special=False) == ref.encode(s).ids, s
