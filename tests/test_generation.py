"""Sampling filters and KV-cached generation on the oracle model (CPU).

Same properties as the reference suite (tests/test_generation.py there):
cached and uncached greedy decoding agree token for token, the cached logits
equal a full forward at every step, the filters keep the right sets, and
generation stops at EOS and at the context limit.
"""

import pytest
import torch

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.inference.sampling import apply_temperature, generate, top_k_filter, top_p_filter
from gpt2_harness_b200.models.gpt import GPT, KVCache


def _model(**kw):
    base = dict(vocab_size=64, n_positions=96, n_layer=3, n_head=4, n_embd=32)
    base.update(kw)
    torch.manual_seed(0)
    return GPT(GPTConfig(**base)).eval()


@pytest.mark.parametrize("n_kv_head", [None, 1, 2])
def test_cached_generation_is_token_exact(n_kv_head):
    model = _model(n_kv_head=n_kv_head)
    prompt = torch.randint(0, 64, (2, 5))
    a = generate(model, prompt, 60, use_cache=True)
    b = generate(model, prompt, 60, use_cache=False)
    assert torch.equal(a, b)


def test_cached_logits_equal_full_forward():
    model = _model(n_positions=32, n_layer=2)
    idx = torch.randint(0, 64, (1, 4))
    cache = KVCache.empty(2)
    with torch.no_grad():
        out = model(idx, cache=cache)
        for _ in range(10):
            nxt = out["logits"][:, -1:].argmax(-1)
            idx = torch.cat([idx, nxt], 1)
            out = model(nxt, cache=cache)
            assert torch.allclose(out["logits"][:, -1], model(idx)["logits"][:, -1], atol=1e-5)


def test_greedy_deterministic_and_sampling_reproducible():
    model = _model(n_positions=32, n_layer=2)
    p = torch.randint(0, 64, (1, 4))
    assert torch.equal(generate(model, p, 12), generate(model, p, 12))
    a = generate(model, p, 12, do_sample=True, temperature=0.8, generator=torch.Generator().manual_seed(7))
    b = generate(model, p, 12, do_sample=True, temperature=0.8, generator=torch.Generator().manual_seed(7))
    assert torch.equal(a, b)


def test_top_k():
    logits = torch.tensor([[3.0, 1.0, 2.0, 0.5, -1.0]])
    out = top_k_filter(logits, 2)
    assert torch.isfinite(out).tolist() == [[True, False, True, False, False]]
    r = torch.randn(2, 9)
    assert torch.equal(top_k_filter(r, 0), r) and torch.equal(top_k_filter(r, 9), r)


def test_top_p_membership():
    logits = torch.log(torch.tensor([[0.1, 0.2, 0.7]]))
    assert torch.isfinite(top_p_filter(logits, 0.65)).tolist() == [[False, False, True]]
    assert torch.isfinite(top_p_filter(logits, 0.70)).tolist() == [[False, True, True]]
    assert torch.isfinite(top_p_filter(logits, 0.95)).all()
    peaked = torch.log(torch.tensor([[0.99, 0.005, 0.005]]))
    assert torch.isfinite(top_p_filter(peaked, 0.5)[0, 0])
    with pytest.raises(ValueError):
        top_p_filter(logits, 0.0)


def test_temperature_rejects_zero():
    with pytest.raises(ValueError):
        apply_temperature(torch.randn(1, 4), 0.0)


def test_context_limit_and_eos():
    m = _model(vocab_size=32, n_positions=12, n_layer=1, n_head=2, n_embd=16)
    assert generate(m, torch.randint(0, 32, (1, 10)), 50).shape[1] == 12
    m = _model(vocab_size=8, n_positions=32, n_layer=1, n_head=2, n_embd=16)
    with torch.no_grad():
        m.lm_head.weight.zero_()
        m.wte.weight.zero_()
        m.wte.weight[3] = 1.0
    out = generate(m, torch.zeros(1, 2, dtype=torch.long), 20, eos_token_id=3)
    assert out.shape[1] < 22 and out[0, -1].item() == 3


def test_kv_memory_formula_matches_allocated_tensors():
    from gpt2_harness_b200.inference.benchmark import (attention_variant_memory, kv_cache_memory,
                                                       measure_cache_tensor_bytes, model_size_bytes)
    m = _model(n_positions=64, n_layer=2)
    r = measure_cache_tensor_bytes(m, 8, 5, batch_size=2)
    assert r["measured_bytes"] == r["predicted_bytes"]
    cfg = GPTConfig(vocab_size=64, n_positions=64, n_layer=2, n_head=4, n_embd=32)
    rows = attention_variant_memory(cfg, [None, 2, 1], seq_len=64, batch_size=2)
    assert [x["reduction_vs_mha"] for x in rows] == [1.0, 2.0, 4.0]
    assert [x["variant"] for x in rows] == ["MHA", "GQA-2", "MQA"]
    k = kv_cache_memory(cfg, [64], [2], dtype_bytes=4, model_bytes=model_size_bytes(m))
    assert k[0]["cache_bytes"] == 2 * 2 * 4 * 8 * 4 * 64 * 2


def test_benchmark_generation_runs_on_cpu():
    from gpt2_harness_b200.inference.benchmark import benchmark_generation
    m = _model(n_positions=64, n_layer=1)
    rows = benchmark_generation(m, [8], new_tokens=4, repeats=1, warmup=0)
    assert {r.arm for r in rows} == {"cached", "uncached"}
    assert all(r.tokens_per_s > 0 for r in rows)
