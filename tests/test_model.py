"""The oracle GPT-2 model (CPU): parameter counts, attention against a naive
loop, causality, SDPA parity, grouped-query attention, activations, ablation
switches, masks, optimiser groups and determinism.

Reference coverage: tests/test_model.py, test_attention.py and
test_determinism.py of gpt2-harness (parameter count 124,439,808; attention vs
a triple loop; future-token invariance; SDPA parity 1e-6; GQA; tanh GELU).
"""

import math

import pytest
import torch
import torch.nn.functional as F

from gpt2_harness_b200.config import GPT2_SIZES, GPTConfig, gpt2_config
from gpt2_harness_b200.models.gpt import GPT, CausalSelfAttention, gelu_tanh, sinusoidal_position_embeddings
from gpt2_harness_b200.perf.mfu import param_count

TINY = dict(vocab_size=97, n_positions=32, n_layer=2, n_head=4, n_embd=32)


def _model(seed=0, **kw):
    torch.manual_seed(seed)
    return GPT(GPTConfig(**{**TINY, **kw}))


def test_gpt2_small_parameter_count():
    cfg = gpt2_config("gpt2")
    assert param_count(cfg) == 124_439_808
    with torch.device("meta"):
        m = GPT(cfg)
    assert m.num_parameters() == 124_439_808
    assert m.num_parameters(non_embedding=True) == 124_439_808 - 1024 * 768
    assert set(GPT2_SIZES) >= {"gpt2", "gpt2-medium", "gpt2-large", "gpt2-xl"}


def test_untied_head_counts_twice():
    cfg = GPTConfig(**TINY, tie_weights=False)
    assert param_count(cfg) == param_count(GPTConfig(**TINY)) + 97 * 32
    assert _model(tie_weights=False).num_parameters() == param_count(cfg)


def _naive_attention(attn: CausalSelfAttention, x):
    B, T, C = x.shape
    H, D = attn.n_head, attn.head_dim
    q, k, v = attn.c_attn(x).split([C, attn.kv_dim, attn.kv_dim], dim=2)
    rep = H // attn.n_kv_head
    out = torch.zeros(B, T, C, dtype=x.dtype)
    for b in range(B):
        for h in range(H):
            hk = h // rep
            for t in range(T):
                qv = q[b, t, h * D:(h + 1) * D]
                s = torch.stack([qv @ k[b, u, hk * D:(hk + 1) * D] / math.sqrt(D) for u in range(t + 1)])
                p = torch.softmax(s, 0)
                out[b, t, h * D:(h + 1) * D] = sum(p[u] * v[b, u, hk * D:(hk + 1) * D] for u in range(t + 1))
    return attn.c_proj(out)


@pytest.mark.parametrize("n_kv_head", [None, 2, 1])
def test_attention_matches_naive_loop(n_kv_head):
    torch.manual_seed(1)
    cfg = GPTConfig(**{**TINY, "n_kv_head": n_kv_head})
    attn = CausalSelfAttention(cfg).double()
    x = torch.randn(2, 7, 32, dtype=torch.float64)
    y, _ = attn(x)
    assert torch.allclose(y, _naive_attention(attn, x), atol=1e-10)


def test_future_tokens_do_not_change_the_past():
    m = _model().eval()
    idx = torch.randint(0, 97, (2, 16))
    other = idx.clone()
    other[:, 10:] = torch.randint(0, 97, (2, 6))
    a, b = m(idx)["logits"], m(other)["logits"]
    assert torch.equal(a[:, :10], b[:, :10])
    assert not torch.allclose(a[:, 10:], b[:, 10:])


def test_attention_weights_are_causal_rows():
    m = _model().eval()
    out = m(torch.randint(0, 97, (1, 9)), need_weights=True)
    for w in out["attentions"]:
        assert torch.allclose(w.sum(-1), torch.ones_like(w.sum(-1)))
        assert torch.all(w.triu(1) == 0)


def test_sdpa_arm_matches_explicit_path():
    torch.manual_seed(2)
    explicit = _model(seed=3).double().eval()
    sdpa = _model(seed=3, use_sdpa=True).double().eval()
    idx = torch.randint(0, 97, (2, 20))
    assert (explicit(idx)["logits"] - sdpa(idx)["logits"]).abs().max() < 1e-6


def test_gelu_tanh_formula_and_closeness_to_exact():
    x = torch.linspace(-6, 6, 1001, dtype=torch.float64)
    ref = 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
    assert torch.allclose(gelu_tanh(x), ref)
    assert (gelu_tanh(x) - F.gelu(x)).abs().max() < 1e-3


@pytest.mark.parametrize("kw", [dict(norm_position="post"), dict(pos_embedding="sinusoidal"),
                                dict(activation="relu"), dict(activation="gelu_exact"),
                                dict(attn_bias=False, mlp_bias=False), dict(residual_scaled_init=False)])
def test_ablation_switches_train(kw):
    m = _model(**kw)
    idx = torch.randint(0, 97, (2, 12))
    out = m(idx, idx)
    out["loss"].backward()
    assert torch.isfinite(out["loss"])
    assert all(p.grad is not None for p in m.parameters() if p.requires_grad)


def test_sinusoidal_table():
    pe = sinusoidal_position_embeddings(16, 8)
    assert pe.shape == (16, 8)
    assert torch.allclose(pe[0, 0::2], torch.zeros(4)) and torch.allclose(pe[0, 1::2], torch.ones(4))


def test_init_statistics():
    torch.manual_seed(0)
    m = GPT(GPTConfig(vocab_size=500, n_positions=64, n_layer=4, n_head=4, n_embd=256))
    assert abs(m.h[0].attn.c_attn.weight.std().item() - 0.02) < 2e-3
    assert abs(m.h[0].mlp.c_proj.weight.std().item() - 0.02 / math.sqrt(8)) < 1e-3
    assert torch.all(m.h[0].attn.c_attn.bias == 0) and torch.all(m.ln_f.weight == 1)
    assert m.lm_head.weight is m.wte.weight


def test_context_limit_and_ignore_index():
    m = _model()
    with pytest.raises(ValueError, match="n_positions"):
        m(torch.zeros(1, 33, dtype=torch.long))
    idx = torch.randint(0, 97, (1, 8))
    tgt = idx.clone()
    tgt[0, 4:] = -100
    full = F.cross_entropy(m(idx)["logits"][0, :4], tgt[0, :4])
    assert torch.allclose(m(idx, tgt)["loss"], full)


def test_head_and_neuron_masks():
    m = _model().eval()
    idx = torch.randint(0, 97, (1, 8))
    base = m(idx)["logits"]
    m.h[0].attn.head_mask = torch.ones(4)
    m.h[0].mlp.neuron_mask = torch.ones(128)
    assert torch.allclose(m(idx)["logits"], base)
    m.h[0].attn.head_mask = torch.tensor([1.0, 0.0, 1.0, 1.0])
    assert not torch.allclose(m(idx)["logits"], base)


def test_optimizer_groups_decay_only_matrices():
    m = _model()
    opt = m.configure_optimizers(0.1, 3e-4, (0.9, 0.95))
    decay, rest = opt.param_groups
    assert decay["weight_decay"] == 0.1 and rest["weight_decay"] == 0.0
    assert all(p.dim() >= 2 for p in decay["params"]) and all(p.dim() < 2 for p in rest["params"])
    assert sum(p.numel() for g in opt.param_groups for p in g["params"]) == m.num_parameters()


def test_training_is_deterministic():
    def run():
        m = _model(seed=7)
        opt = m.configure_optimizers(0.1, 1e-3, (0.9, 0.95))
        g = torch.Generator().manual_seed(0)
        losses = []
        for _ in range(3):
            idx = torch.randint(0, 97, (2, 16), generator=g)
            loss = m(idx, idx)["loss"]
            opt.zero_grad()
            loss.backward()
            opt.step()
            losses.append(loss.item())
        return losses, [p.detach().clone() for p in m.parameters()]

    (l1, p1), (l2, p2) = run(), run()
    assert l1 == l2 and all(torch.equal(a, b) for a, b in zip(p1, p2))
    assert l1[-1] < l1[0]
