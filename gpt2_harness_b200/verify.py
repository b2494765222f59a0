"""Numerical verification against HuggingFace GPT-2 (and of the B200 engine
against the oracle).

Reference: src/transformer_internals/verify.py:67-498. Levels, strictest
localisation first:

1. every named activation (embedding, per block ln_1 / attn / resid_mid /
   ln_2 / mlp / resid_out, ln_f, logits) against HF forward hooks, so a
   discrepancy is pinned to one sub-module of one block; ``resid_mid`` is
   ``ln_2``'s input and the last block's output is ``ln_f``'s input (HF's
   last hidden state is already normalised);
2. final logits within ``LOGIT_TOLERANCE`` (1e-3, fp32);
3. greedy generation token-exact (KV-cached ours vs ``ref.generate``), with
   the index of the first divergence on a mismatch;
4. perplexity on identical windows (token-weighted mean NLL).

Added: :func:`compare_native_logits`, the B200 engine's bf16 forward against
the fp32 oracle on the same weights (a bf16 tolerance), so the hot path is
tied to the HF-verified model through the oracle.
"""

from __future__ import annotations

import argparse
import json
import math
from dataclasses import asdict, dataclass, field
from typing import Any, Callable, Iterable, Optional

import torch
import torch.nn.functional as F

from .inference.sampling import generate
from .models.gpt import GPT

__all__ = ["LOGIT_TOLERANCE", "LayerDiff", "VerificationReport", "reference_taps", "compare_activations",
           "compare_logits", "compare_greedy_generation", "compare_perplexity", "compare_native_logits",
           "run_verification", "hf_reference_from"]

LOGIT_TOLERANCE = 1e-3


@dataclass
class LayerDiff:
    name: str
    max_abs: float
    max_rel: float
    ref_scale: float

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass
class VerificationReport:
    layers: list = field(default_factory=list)
    logits_max_abs: Optional[float] = None
    logit_tolerance: float = LOGIT_TOLERANCE
    generations: list = field(default_factory=list)
    perplexity: Optional[dict] = None
    native: Optional[dict] = None

    @property
    def logits_ok(self) -> bool:
        return self.logits_max_abs is not None and self.logits_max_abs < self.logit_tolerance

    @property
    def all_generations_match(self) -> bool:
        return all(g["match"] for g in self.generations)

    @property
    def worst_layer(self) -> Optional[LayerDiff]:
        return max(self.layers, key=lambda r: r.max_abs) if self.layers else None

    def to_dict(self) -> dict:
        return {"layers": [r.to_dict() for r in self.layers], "logits_max_abs": self.logits_max_abs,
                "logit_tolerance": self.logit_tolerance, "logits_ok": self.logits_ok,
                "generations": self.generations, "all_generations_match": self.all_generations_match,
                "perplexity": self.perplexity, "native": self.native}


def _diff(name: str, ours: torch.Tensor, ref: torch.Tensor, rel_floor: float = 1e-2) -> LayerDiff:
    a, b = ours.detach().float().cpu(), ref.detach().float().cpu()
    if a.shape != b.shape:
        raise ValueError(f"{name}: shape {tuple(a.shape)} vs {tuple(b.shape)}")
    d = (a - b).abs()
    scale = b.abs().max().item()
    return LayerDiff(name, d.max().item(), (d / b.abs().clamp_min(rel_floor)).max().item(), scale)


def hf_reference_from(model: GPT):
    """A HuggingFace ``GPT2LMHeadModel`` holding ``model``'s weights (eager
    attention), for offline verification with any weights."""
    import transformers

    from .weights import to_hf_state_dict
    c = model.config
    hcfg = transformers.GPT2Config(vocab_size=c.vocab_size, n_positions=c.n_positions, n_embd=c.n_embd,
                                   n_layer=c.n_layer, n_head=c.n_head, layer_norm_epsilon=c.layer_norm_epsilon,
                                   resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0,
                                   activation_function="gelu_new", tie_word_embeddings=c.tie_weights)
    ref = transformers.GPT2LMHeadModel(hcfg)
    ref.config._attn_implementation = "eager"
    missing, unexpected = ref.load_state_dict(to_hf_state_dict(model.state_dict()), strict=False)
    bad = [k for k in missing if not k.endswith((".attn.bias", ".attn.masked_bias"))]
    if bad or unexpected:
        raise RuntimeError(f"HF load mismatch: missing={bad} unexpected={unexpected}")
    return ref.eval()


def reference_taps(ref, x: torch.Tensor) -> dict[str, torch.Tensor]:
    """Activations of a HF GPT-2 keyed like ours (forward hooks)."""
    taps: dict[str, torch.Tensor] = {}
    handles = []

    def out_hook(key, first=False) -> Callable:
        def h(_m, _i, out):
            taps[key] = (out[0] if first and isinstance(out, (tuple, list)) else out).detach()
        return h

    def in_hook(key) -> Callable:
        def h(_m, inp, _o):
            taps[key] = inp[0].detach()
        return h

    tr = ref.transformer
    for i, blk in enumerate(tr.h):
        handles += [blk.ln_1.register_forward_hook(out_hook(f"h.{i}.ln_1")),
                    blk.attn.register_forward_hook(out_hook(f"h.{i}.attn", first=True)),
                    blk.ln_2.register_forward_hook(in_hook(f"h.{i}.resid_mid")),
                    blk.ln_2.register_forward_hook(out_hook(f"h.{i}.ln_2")),
                    blk.mlp.register_forward_hook(out_hook(f"h.{i}.mlp")),
                    blk.register_forward_hook(out_hook(f"h.{i}.resid_out", first=True))]
    handles += [tr.ln_f.register_forward_hook(out_hook("ln_f")),
                tr.ln_f.register_forward_hook(in_hook("final_resid"))]
    try:
        with torch.no_grad():
            out = ref(x, output_hidden_states=True)
    finally:
        for h in handles:
            h.remove()
    taps["embed"] = out.hidden_states[0].detach()
    taps[f"h.{len(tr.h) - 1}.resid_out"] = taps.pop("final_resid")
    taps["logits"] = out.logits.detach()
    return taps


def compare_activations(model: GPT, ref, x: torch.Tensor):
    """Rows ordered by depth, our logits, reference logits."""
    with torch.no_grad():
        ours = model(x, collect_taps=True)
    mine, theirs = ours["taps"], reference_taps(ref, x)
    order = ["embed"]
    for i in range(model.config.n_layer):
        order += [f"h.{i}.{s}" for s in ("ln_1", "attn", "resid_mid", "ln_2", "mlp", "resid_out")]
    order += ["ln_f", "logits"]
    rows = [_diff(k, mine[k], theirs[k]) for k in order if k in mine and k in theirs]
    return rows, ours["logits"], theirs["logits"]


def compare_logits(ours: torch.Tensor, ref: torch.Tensor) -> tuple[float, float, float]:
    d = _diff("logits", ours, ref)
    return d.max_abs, d.max_rel, d.ref_scale


def compare_greedy_generation(model: GPT, ref, prompts: Iterable, max_new_tokens: int = 300, tokenizer=None,
                              device="cpu") -> list[dict]:
    """Greedy continuation of each prompt (str with a tokenizer, or id list)."""
    recs = []
    for p in prompts:
        ids = tokenizer.encode(p) if isinstance(p, str) else list(p)
        x = torch.tensor([ids], dtype=torch.long)
        ours = generate(model, x.to(device), max_new_tokens, use_cache=True)[0].tolist()
        pad = tokenizer.eot_token_id if tokenizer is not None and tokenizer.eot_token_id is not None else 0
        with torch.no_grad():
            theirs = ref.generate(x, attention_mask=torch.ones_like(x), max_new_tokens=max_new_tokens,
                                  do_sample=False, pad_token_id=pad)[0].tolist()
        first = None
        if ours != theirs:
            first = next((i for i, (a, b) in enumerate(zip(ours, theirs)) if a != b), min(len(ours), len(theirs)))
        recs.append({"prompt": p if isinstance(p, str) else None, "n_prompt_tokens": len(ids),
                     "n_new_tokens": len(ours) - len(ids), "match": ours == theirs, "first_divergence": first,
                     "text": tokenizer.decode(ours) if tokenizer is not None else None})
    return recs


def compare_perplexity(model: GPT, ref, batches: Iterable, device="cpu") -> dict:
    """Perplexity of both models over (x, y) batches, token-weighted."""
    s_ours = s_ref = 0.0
    n_tok = n_b = 0
    for x, y in batches:
        with torch.no_grad():
            lo = model(x.to(device))["logits"].float().cpu()
            lr = ref(x).logits.float()
        s_ours += F.cross_entropy(lo.reshape(-1, lo.size(-1)), y.reshape(-1), reduction="sum").item()
        s_ref += F.cross_entropy(lr.reshape(-1, lr.size(-1)), y.reshape(-1), reduction="sum").item()
        n_tok += y.numel()
        n_b += 1
    lo_, lr_ = s_ours / n_tok, s_ref / n_tok
    return {"n_tokens": n_tok, "n_batches": n_b, "ours_loss": lo_, "reference_loss": lr_,
            "ours_ppl": math.exp(lo_), "reference_ppl": math.exp(lr_),
            "abs_ppl_diff": abs(math.exp(lo_) - math.exp(lr_))}


def compare_native_logits(model: GPT, x: torch.Tensor, device="cuda") -> dict:
    """B200 engine (bf16 hot path) vs the fp32 oracle on the same weights."""
    from .models.engine import Engine
    B, T = x.shape
    eng = Engine.from_module(model, device=device)
    V = model.config.vocab_size
    native = eng.logits(x.to(device)).float().cpu().reshape(B, T, V)
    with torch.no_grad():
        ref = model.to("cpu")(x)["logits"].float()
    d = (native - ref).abs()
    agree = (native.argmax(-1) == ref.argmax(-1)).float().mean().item()
    return {"max_abs": d.max().item(), "mean_abs": d.mean().item(), "ref_scale": ref.abs().max().item(),
            "argmax_agreement": agree}


def run_verification(model: GPT, ref=None, x: Optional[torch.Tensor] = None, prompts: Optional[list] = None,
                     max_new_tokens: int = 100, batches: Optional[Iterable] = None, tokenizer=None,
                     native: bool = False) -> VerificationReport:
    ref = hf_reference_from(model) if ref is None else ref
    g = torch.Generator().manual_seed(0)
    V, T = model.config.vocab_size, min(64, model.config.n_positions)
    x = torch.randint(0, V, (2, T), generator=g) if x is None else x
    rep = VerificationReport()
    rep.layers, lo, lr = compare_activations(model, ref, x)
    rep.logits_max_abs = compare_logits(lo, lr)[0]
    if prompts is None:
        prompts = [torch.randint(0, V, (8,), generator=g).tolist() for _ in range(2)]
    rep.generations = compare_greedy_generation(model, ref, prompts, max_new_tokens, tokenizer)
    if batches is not None:
        rep.perplexity = compare_perplexity(model, ref, batches)
    if native:
        rep.native = compare_native_logits(model, x)
    return rep


def _main() -> None:
    ap = argparse.ArgumentParser(description="verify the oracle GPT (and the B200 engine) against HF GPT-2")
    ap.add_argument("--size", default="gpt2")
    ap.add_argument("--checkpoint-dir", default=None, help="local HF checkpoint; random weights when absent")
    ap.add_argument("--max-new-tokens", type=int, default=100)
    ap.add_argument("--native", action="store_true")
    a = ap.parse_args()
    from .config import gpt2_config
    if a.checkpoint_dir:
        from .weights import load_pretrained_gpt2
        model, _ = load_pretrained_gpt2(a.size, a.checkpoint_dir)
    else:
        torch.manual_seed(0)
        model = GPT(gpt2_config(a.size)).eval()
    rep = run_verification(model, max_new_tokens=a.max_new_tokens, native=a.native)
    d = rep.to_dict()
    d["worst_layer"] = rep.worst_layer.to_dict() if rep.worst_layer else None
    d.pop("layers")
    print(json.dumps(d))


if __name__ == "__main__":
    _main()
