"""Tensor parallelism (parity mode and sequence parallel) and the
vocab-parallel head on CPU/gloo ranks vs unsharded modules."""

import pytest

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.tensor_parallel import (padded_vocab, tp_equivalence_worker,
                                                        tp_payload_bytes, vocab_parallel_worker)

TOL = 1e-5
_CACHE = {}


def run(fn, world, **kw):
    key = (fn.__name__, world, tuple(sorted(kw.items())))
    if key not in _CACHE:
        _CACHE[key] = comms.spawn_workers(fn, world, kw, backend="gloo", timeout=300)
    return _CACHE[key]


@pytest.mark.parametrize("world", [2, 4])
def test_tp_block_forward_and_backward(world):
    for r in run(tp_equivalence_worker, world, batch=4, seq=12):
        assert r.value["forward_error"] < TOL
        assert r.value["max_grad_error"] < TOL


def test_tp_exactly_four_allreduces_per_block():
    res = run(tp_equivalence_worker, 2, batch=4, seq=12)
    pay = res[0].payload
    assert pay["per_collective"]["all_reduce"]["calls"] == 4
    assert pay["payload_bytes_per_step"] == 24_576 == 4 * 4 * 4 * 12 * 32


def test_sequence_parallel_block_matches():
    for r in run(tp_equivalence_worker, 2, batch=4, seq=12, sequence_parallel=True):
        assert r.value["forward_error"] < TOL
        assert r.value["max_grad_error"] < TOL


def test_sequence_parallel_payload_is_twice_raw_same_ar_equivalent():
    res = run(tp_equivalence_worker, 2, batch=4, seq=12, sequence_parallel=True)
    pay = res[0].payload["per_collective"]
    assert pay["all_gather"]["calls"] == 4 and pay["reduce_scatter"]["calls"] == 4
    raw = pay["all_gather"]["payload_bytes"] + pay["reduce_scatter"]["payload_bytes"]
    cf = tp_payload_bytes(4, 12, 32, 1, sequence_parallel=True)
    assert raw == cf["raw"] == 2 * 24_576
    assert cf["allreduce_equivalent"] == 24_576
    # ring wire bytes equal parity mode: 2(p-1)/p * S per AR vs (p-1)/p * S per AG/RS
    par = run(tp_equivalence_worker, 2, batch=4, seq=12)[0].payload
    assert res[0].payload["total_wire_bytes_ring_model"] == pytest.approx(par["total_wire_bytes_ring_model"])


def test_padded_vocab():
    # the padded GPT-2 vocabulary at every power-of-two group size up to 8:
    # a multiple of 64, split in equal per-rank blocks of a multiple of 16 rows
    assert all(padded_vocab(50257, p) == 50304 for p in (1, 2, 4, 8))
    assert all(padded_vocab(50257, p) % 64 == 0 and (padded_vocab(50257, p) // p) % 16 == 0
               for p in (1, 2, 3, 4, 5, 6, 7, 8))


@pytest.mark.parametrize("world", [2, 4])
def test_vocab_parallel_embedding_and_cross_entropy(world):
    res = run(vocab_parallel_worker, world, batch=4, seq=16)
    for r in res:
        assert r.value["loss_error"] < TOL
        assert r.value["grad_error"] < TOL
    pay = res[0].payload["per_collective"]
    # one embedding all-reduce (B*T*C) + three (B*T,) loss all-reduces + f's backward
    assert pay["all_reduce"]["calls"] == 5


def test_tensor_parallel_holds_a_fraction_of_the_block():
    import torch

    from gpt2_harness_b200.parallel.common import identical_block, parallel_config
    from gpt2_harness_b200.parallel.tensor_parallel import TensorParallelBlock

    cfg = parallel_config()
    C = cfg.n_embd
    full = sum(p.numel() for p in identical_block(cfg).parameters())
    replicated = 4 * C + C + C  # two LayerNorms, c_proj and mlp c_proj biases (added once)
    for p in (2, 4):
        tp = TensorParallelBlock(identical_block(cfg), 0, p)
        held = sum(t.numel() for t in tp.parameters())
        assert held == (full - replicated) // p + replicated
