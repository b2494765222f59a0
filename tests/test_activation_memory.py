"""Activation memory (CPU): the saved-tensor meter against the analytic
enumeration of the oracle model's saved set (exact at fp32, dropout 0), the
refusals of the analytic count, and the native engine's planned stash.

Reference coverage: tests/test_activation_memory.py of gpt2-harness (exact
activation count, GELU's four saved tensors, the T^2 attention terms).
"""

import pytest
import torch

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.gpt import GPT
from gpt2_harness_b200.perf.activation_memory import (GELU_TANH_SAVED_TENSORS, ActivationMeter,
                                                      analytic_activation_bytes, measure_activation_bytes,
                                                      native_activation_bytes)

TINY = dict(vocab_size=97, n_positions=32, n_layer=2, n_head=4, n_embd=32)


@pytest.mark.parametrize("kw", [{}, {"activation": "relu"}, {"activation": "gelu_exact"},
                                {"pos_embedding": "sinusoidal"}, {"n_layer": 3, "n_head": 2}])
@pytest.mark.parametrize("with_loss", [True, False])
def test_measured_equals_analytic_exactly(kw, with_loss):
    torch.manual_seed(0)
    cfg = GPTConfig(**{**TINY, **kw})
    m = GPT(cfg)
    idx = torch.randint(0, 97, (2, 16))
    tgt = torch.randint(0, 97, (2, 16)) if with_loss else None
    r = measure_activation_bytes(m, idx, tgt)
    assert r.measured_bytes == r.analytic_bytes
    assert r.ratio == 1.0


def test_gelu_saves_four_wide_tensors_and_attention_is_quadratic():
    cfg = GPTConfig(**TINY)
    a = analytic_activation_bytes(cfg, 2, 16)
    relu = analytic_activation_bytes(GPTConfig(**TINY, activation="relu"), 2, 16)
    act = 2 * 16 * 32 * 4
    assert a["per_layer.mlp_activation_intermediates"] == GELU_TANH_SAVED_TENSORS * 4 * act
    assert relu["per_layer.mlp_activation_intermediates"] == 0
    t1 = analytic_activation_bytes(cfg, 1, 16)["per_layer.attention_probabilities"]
    t2 = analytic_activation_bytes(cfg, 1, 32)["per_layer.attention_probabilities"]
    assert t2 == 4 * t1
    assert a["total"] == a["all_layers"] + a["root_subtotal"]


def test_analytic_refusals():
    for kw in ({"dropout": 0.1}, {"use_sdpa": True}, {"n_kv_head": 2}):
        with pytest.raises(ValueError):
            analytic_activation_bytes(GPTConfig(**{**TINY, **kw}), 2, 16)
    with pytest.raises(ValueError, match="fp32 only"):
        analytic_activation_bytes(GPTConfig(**TINY), 2, 16, dtype_bytes=2)


def test_meter_excludes_parameters_and_releases_storages():
    lin = torch.nn.Linear(8, 8)
    x = torch.randn(4, 8, requires_grad=True)
    meter = ActivationMeter(exclude=list(lin.parameters()))
    with meter:
        y = lin(x).relu().sum()
    snap = meter.snapshot()
    assert snap["activation_bytes"] > 0
    assert meter.to_dict()["excluded_parameter_bytes"] > 0
    y.backward()
    del y
    # the relu output is freed with the graph; the input x, saved for the
    # weight gradient, is still referenced here and stays counted
    assert meter.stash_bytes() == x.numel() * 4


def test_native_stash_is_far_below_the_oracle():
    cfg = GPTConfig(vocab_size=50257, n_positions=1024, n_layer=12, n_head=12, n_embd=768)
    nat = native_activation_bytes(cfg, 16, 1024)
    M, C = 16 * 1024, 768
    assert nat["per_layer.qkv_bf16"] == M * 3 * C * 2
    assert nat["root.logits_bf16_padded"] == M * 50304 * 2
    oracle = analytic_activation_bytes(cfg, 16, 1024)
    # no T x T probabilities, bf16 operands: several times smaller
    assert nat["total"] * 4 < oracle["total"]
