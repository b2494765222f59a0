"""Corpus, token windows, compact vocabulary, and the single-process training
loop (oracle on CPU; the native backend on a GPU)."""

import math

import numpy as np
import pytest
import torch

from gpt2_harness_b200.config import GPTConfig, TrainConfig
from gpt2_harness_b200.data import TokenDataset, compact_vocabulary, encode_corpus, synthetic_stories
from gpt2_harness_b200.tokenizer import train_bpe
from gpt2_harness_b200.train import lr_at_step, train


@pytest.fixture(scope="module")
def corpus():
    text = synthetic_stories(300, seed=1)
    tok = train_bpe(text.split("\n\n")[:200], 512)
    return text, tok


def test_synthetic_stories_deterministic():
    assert synthetic_stories(5, 3) == synthetic_stories(5, 3)
    assert synthetic_stories(5, 3) != synthetic_stories(5, 4)


def test_encode_corpus_caches_and_roundtrips(tmp_path, corpus):
    text, tok = corpus
    a = encode_corpus(tok, text, data_dir=tmp_path)
    assert len(list(tmp_path.glob("tokens_*.npy"))) == 1
    b = encode_corpus(tok, text, data_dir=tmp_path)
    assert np.array_equal(a, b) and a.dtype == np.uint16
    assert tok.decode(a.tolist()) == text


def test_token_dataset_windows(corpus):
    text, tok = corpus
    ds = TokenDataset(encode_corpus(tok, text, cache=False), block_size=32)
    x, y = ds.get_batch("train", 4, generator=torch.Generator().manual_seed(0))
    assert x.shape == y.shape == (4, 32) and torch.equal(x[:, 1:], y[:, :-1])
    x2, _ = ds.get_batch("train", 4, generator=torch.Generator().manual_seed(0))
    assert torch.equal(x, x2)
    seq = ds.sequential_batches("val", 2, limit=3)
    flat = torch.cat([b[0].reshape(-1) for b in seq])
    assert len(seq) <= 3 and torch.equal(flat[:32], torch.from_numpy(ds.val[:32].astype(np.int64)))
    with pytest.raises(ValueError):
        TokenDataset(np.arange(10), block_size=32)


def test_compact_vocabulary():
    t = np.array([5, 5, 5, 7, 7, 9, 1])
    remapped, id_map, cov = compact_vocabulary(t, vocab_size=3)
    assert id_map.tolist() == [-1, 5, 7]
    assert remapped.tolist() == [1, 1, 1, 2, 2, 0, 0]
    assert math.isclose(cov, 5 / 7)


def test_lr_schedule():
    c = TrainConfig(steps=100, warmup_steps=10, lr=1.0, min_lr_ratio=0.1)
    assert lr_at_step(0, c) == pytest.approx(0.1) and lr_at_step(9, c) == pytest.approx(1.0)
    assert lr_at_step(99, c) == pytest.approx(0.1, abs=1e-3)


def _cfgs(tok, **kw):
    m = GPTConfig(vocab_size=tok.vocab_size, n_positions=32, n_layer=2, n_head=2, n_embd=32)
    t = dict(steps=40, batch_size=8, block_size=32, lr=3e-3, warmup_steps=5, eval_interval=20, eval_batches=2)
    t.update(kw)
    return m, TrainConfig(**t)


def test_oracle_training_learns_and_is_reproducible(corpus):
    text, tok = corpus
    ds = TokenDataset(encode_corpus(tok, text, cache=False), 32)
    m, t = _cfgs(tok)
    _, r1 = train(m, t, ds, device="cpu")
    _, r2 = train(m, t, ds, device="cpu")
    assert r1.history == r2.history and r1.grad_norms == r2.grad_norms
    assert r1.history[-1]["val_loss"] < math.log(tok.vocab_size) - 1.0
    assert len(r1.grad_norms) == 40 and not r1.diverged and r1.tokens_seen == 40 * 8 * 32


def test_divergence_is_recorded_not_raised(corpus):
    text, tok = corpus
    ds = TokenDataset(encode_corpus(tok, text, cache=False), 32)
    m, t = _cfgs(tok, lr=1e6, grad_clip=0.0, steps=30, warmup_steps=1)
    _, r = train(m, t, ds, device="cpu")
    assert r.diverged or not math.isfinite(r.history[-1]["val_loss"]) or r.history[-1]["val_loss"] > 5


@pytest.mark.gpu
def test_native_training_learns(corpus):
    text, tok = corpus
    ds = TokenDataset(encode_corpus(tok, text, cache=False), 64)
    m = GPTConfig(vocab_size=tok.vocab_size, n_positions=64, n_layer=2, n_head=2, n_embd=128)
    t = TrainConfig(steps=60, batch_size=8, block_size=64, lr=2e-3, warmup_steps=5, eval_interval=30,
                    eval_batches=2, grad_accum=2)
    eng, r = train(m, t, ds, device="cuda", backend="native")
    assert not r.diverged and r.history[-1]["val_loss"] < math.log(tok.vocab_size) - 1.0
    assert len(r.grad_norms) == 60 and all(math.isfinite(g) for g in r.grad_norms)


def test_native_training_loop_on_cpu(corpus, monkeypatch):
    """The native backend's loop (grad accumulation, LR schedule, clipping,
    evaluation) on the torch versions of the kernel contracts."""
    import native_fake

    text, tok = corpus
    ds = TokenDataset(encode_corpus(tok, text, cache=False), 64)
    m = GPTConfig(vocab_size=tok.vocab_size, n_positions=64, n_layer=2, n_head=2, n_embd=128)
    t = TrainConfig(steps=30, batch_size=4, block_size=64, lr=2e-3, warmup_steps=3, eval_interval=15,
                    eval_batches=2, grad_accum=2)
    with native_fake.installed(monkeypatch):
        eng, r = train(m, t, ds, device="cpu", backend="native")
    assert not r.diverged and len(r.grad_norms) == 30 and all(math.isfinite(g) for g in r.grad_norms)
    assert r.history[-1]["val_loss"] < r.history[0]["val_loss"]
