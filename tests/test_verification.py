"""Verification against HuggingFace GPT-2, offline: a randomly initialised HF
model holding our weights (the published checkpoint needs a network)."""

import copy

import pytest
import torch

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.gpt import GPT

transformers = pytest.importorskip("transformers")

from gpt2_harness_b200.verify import (LOGIT_TOLERANCE, compare_activations, compare_greedy_generation,  # noqa: E402
                                      compare_perplexity, hf_reference_from, run_verification)
from gpt2_harness_b200.weights import (convert_hf_state_dict, load_gpt2_state_dict,  # noqa: E402
                                       save_hf_checkpoint, to_hf_state_dict)


@pytest.fixture(scope="module")
def pair():
    torch.manual_seed(0)
    cfg = GPTConfig(vocab_size=100, n_positions=64, n_layer=2, n_head=4, n_embd=32)
    model = GPT(cfg).eval()
    # larger weights than the 0.02 init so greedy decoding has clear winners
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() == 2:
                p.mul_(8.0)
    return model, hf_reference_from(model)


def test_parameter_count_matches_hf(pair):
    model, ref = pair
    theirs = sum(p.numel() for p in {id(p): p for p in ref.parameters()}.values())
    assert model.num_parameters() == theirs


def test_every_activation_and_the_logits_match(pair):
    model, ref = pair
    x = torch.randint(0, 100, (2, 40))
    rows, lo, lr = compare_activations(model, ref, x)
    assert len(rows) == 1 + 6 * model.config.n_layer + 2
    for r in rows:
        assert r.max_abs < 1e-4, (r.name, r.max_abs)
    assert (lo - lr).abs().max().item() < LOGIT_TOLERANCE


def test_greedy_generation_token_exact_and_perplexity(pair):
    model, ref = pair
    prompts = [torch.randint(0, 100, (6,)).tolist() for _ in range(2)]
    for r in compare_greedy_generation(model, ref, prompts, max_new_tokens=40):
        assert r["match"], r["first_divergence"]
    batches = [(torch.randint(0, 100, (2, 32)), torch.randint(0, 100, (2, 32))) for _ in range(2)]
    out = compare_perplexity(model, ref, batches)
    assert out["abs_ppl_diff"] < 1e-3 * out["reference_ppl"]


def test_a_transposed_projection_is_detected(pair):
    model, ref = pair
    broken = copy.deepcopy(model)
    with torch.no_grad():
        w = broken.h[1].attn.c_proj.weight
        w.copy_(w.t().contiguous())
    x = torch.randint(0, 100, (1, 20))
    with torch.no_grad():
        assert (broken(x)["logits"] - ref(x).logits).abs().max().item() > LOGIT_TOLERANCE


def test_run_verification_report(pair):
    model, ref = pair
    rep = run_verification(model, ref, max_new_tokens=20)
    assert rep.logits_ok and rep.all_generations_match
    assert rep.worst_layer is not None and rep.to_dict()["logits_ok"]


def test_hf_checkpoint_roundtrip(tmp_path, pair):
    model, _ = pair
    save_hf_checkpoint(model.state_dict(), tmp_path)
    loaded = convert_hf_state_dict(load_gpt2_state_dict(tmp_path), model.config)
    sd = model.state_dict()
    for k, v in loaded.items():
        assert torch.equal(v, sd[k]), k
    hf = to_hf_state_dict(sd)
    assert hf["transformer.h.0.attn.c_attn.weight"].shape == (32, 96)  # Conv1D layout [in, out]


def test_shape_mismatch_is_rejected(pair):
    model, _ = pair
    hf = to_hf_state_dict(model.state_dict())
    bad = GPTConfig(vocab_size=101, n_positions=64, n_layer=2, n_head=4, n_embd=32)
    with pytest.raises(ValueError):
        convert_hf_state_dict(hf, bad)


@pytest.mark.gpu
def test_native_engine_logits_match_oracle():
    from gpt2_harness_b200.verify import compare_native_logits
    torch.manual_seed(0)
    model = GPT(GPTConfig(vocab_size=512, n_positions=128, n_layer=2, n_head=2, n_embd=128)).eval()
    out = compare_native_logits(model, torch.randint(0, 512, (2, 128)))
    assert out["max_abs"] < 2e-2 * max(1.0, out["ref_scale"]), out
    assert out["argmax_agreement"] > 0.97, out
