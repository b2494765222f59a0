"""MFU arithmetic and the roofline peak model (CPU).

Reference coverage: tests/test_perf.py of gpt2-harness (analytic parameter
count equals the built model and GPT-2's published size, exact count exceeds
6ND by the attention term, causal-aware counting halves it, training is three
forward passes, published peaks carry citations, modelled MFU is division by
the published peak, measured MFU is self-consistent, ridge and attainable
rate).
"""

import math

import pytest
import torch

from gpt2_harness_b200.config import GPTConfig, gpt2_config
from gpt2_harness_b200.models.gpt import GPT
from gpt2_harness_b200.perf.mfu import (PUBLISHED_ACCELERATORS, flops_6nd, flops_per_token_exact,
                                        measure_step_mfu, measured_peak_tflops, mfu_on_published_gpu,
                                        param_count)
from gpt2_harness_b200.perf.roofline import MachinePeak, peak_from_file


@pytest.mark.parametrize("kw", [{}, {"n_kv_head": 2}, {"tie_weights": False}, {"pos_embedding": "sinusoidal"}])
def test_analytic_count_matches_the_built_model(kw):
    cfg = GPTConfig(vocab_size=101, n_positions=40, n_layer=3, n_head=4, n_embd=48, **kw)
    assert param_count(cfg) == GPT(cfg).num_parameters()


def test_published_gpt2_sizes():
    assert param_count(gpt2_config("gpt2")) == 124_439_808
    assert param_count(gpt2_config("gpt2-medium")) == 354_823_168
    assert param_count(gpt2_config("gpt2-xl", vocab_size=50304)) == 1_557_686_400


def test_exact_count_exceeds_6nd_by_the_attention_term():
    cfg = gpt2_config("gpt2")
    d = flops_per_token_exact(cfg, 1024)
    assert d["training_flops_per_token"] == 3 * d["forward_total_flops_per_token"]
    assert d["training_flops_per_token"] > d["flops_6n_non_embedding_per_token"]
    quad = 3 * 2 * 2 * 1024 * 768 * 12
    assert d["training_attention_quadratic_flops_per_token"] == pytest.approx(quad)
    causal = flops_per_token_exact(cfg, 1024, causal_aware=True)
    assert causal["forward_attention_quadratic_flops_per_token"] == pytest.approx(
        d["forward_attention_quadratic_flops_per_token"] / 2)
    assert causal["forward_projection_flops_per_token"] == d["forward_projection_flops_per_token"]
    assert flops_6nd(10, 7) == 420
    # 16k context: the quadratic term dominates GPT-2 large
    big = flops_per_token_exact(gpt2_config("gpt2-large", n_positions=16384), 16384)
    assert big["attention_quadratic_fraction"] > 0.5


def test_published_peaks_and_modelled_mfu():
    assert PUBLISHED_ACCELERATORS["B200"]["bf16"] == 2250.0
    assert PUBLISHED_ACCELERATORS["H100-SXM"]["bf16"] == 989.0
    m = mfu_on_published_gpu(1e9, 1e6, "B200")
    assert m == pytest.approx(1e15 / 2.25e15)


def test_measured_peak_file_and_fallback(tmp_path):
    peak, label = measured_peak_tflops()
    assert peak > 100 and label.startswith(("measured", "fallback"))
    p, l2 = measured_peak_tflops(str(tmp_path / "missing.json"))
    assert l2 == "fallback" and p == 1400.0
    mp = peak_from_file()
    assert mp.ridge_flops_per_byte == pytest.approx(mp.peak_flops_per_s / mp.peak_bytes_per_s)


def test_ridge_and_attainable_rate():
    mp = MachinePeak("x", "bf16", 100.0, 10.0, 10.0)
    assert mp.attainable_flops_per_s(1.0) == 10.0
    assert mp.attainable_flops_per_s(10.0) == 100.0
    assert mp.attainable_flops_per_s(1e6) == 100.0


def test_measured_mfu_is_self_consistent():
    cfg = GPTConfig(vocab_size=64, n_positions=16, n_layer=1, n_head=2, n_embd=16)
    calls = []
    rep = measure_step_mfu(lambda: calls.append(1), cfg, batch=2, seq_len=16, steps=4, warmup=2,
                           peak_tflops=1.0, n_gpus=2)
    assert len(calls) == 6
    assert rep.tokens_per_step == 2 * 16 * 2
    assert rep.achieved_tflops == pytest.approx(rep.flops_per_token * rep.tokens_per_step / rep.step_time_s / 1e12)
    assert rep.mfu == pytest.approx(rep.achieved_tflops / 2.0)
    assert rep.as_dict()["tokens_per_s"] == pytest.approx(rep.tokens_per_step / rep.step_time_s)
