"""Experiment runners: one subcommand per study, each writing the results JSON
that :mod:`gpt2_harness_b200.viz` draws.

Reference: scripts/run_verification.py, run_kv_cache.py, run_quantization.py,
run_pruning.py, run_distillation.py, run_induction.py, run_ablations.py,
make_pareto.py, make_figures.py. Data is the local corpus when one is
configured (``--corpus`` / ``$G2B_CORPUS``) and the offline synthetic
stories otherwise; weights are a local HF checkpoint when given, a model
trained here otherwise (this machine has no network).

    python -m gpt2_harness_b200.experiments kv_cache --out results
    python -m gpt2_harness_b200.experiments all --quick --out results
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Any, Optional

import torch

from .config import GPTConfig, TrainConfig

__all__ = ["STUDIES", "run_study", "main"]


def _save(out: Path, name: str, payload: dict) -> Path:
    out.mkdir(parents=True, exist_ok=True)
    p = out / f"{name}.json"
    p.write_text(json.dumps(payload, indent=1, default=lambda o: o.to_dict() if hasattr(o, "to_dict") else str(o)))
    return p


def _dataset(quick: bool, corpus: Optional[str], block: int = 64):
    from .data import TokenDataset, encode_corpus, load_text, synthetic_stories
    from .tokenizer import train_bpe
    text = load_text(corpus) if corpus else synthetic_stories(600 if quick else 4000)
    tok = train_bpe(text.split("\n\n")[:300 if quick else 2000], 512 if quick else 2048)
    return TokenDataset(encode_corpus(tok, text, cache=False), block), tok


def _trained_model(ds, tok, quick: bool, device):
    from .train import train
    cfg = GPTConfig(vocab_size=tok.vocab_size, n_positions=ds.block_size, n_layer=2 if quick else 4, n_head=4,
                    n_embd=64 if quick else 256)
    tc = TrainConfig(steps=60 if quick else 600, batch_size=16, block_size=ds.block_size, lr=2e-3,
                     warmup_steps=10, eval_interval=60 if quick else 200, eval_batches=2)
    model, _ = train(cfg, tc, ds, device=device)
    return model.eval()


def study_verification(a) -> dict:
    from .models.gpt import GPT
    from .verify import run_verification
    torch.manual_seed(0)
    model = GPT(GPTConfig(vocab_size=512, n_positions=64, n_layer=2, n_head=4, n_embd=64)).eval()
    rep = run_verification(model, max_new_tokens=20 if a.quick else 100, native=torch.cuda.is_available())
    return rep.to_dict()


def study_kv_cache(a) -> dict:
    from .config import gpt2_config
    from .inference.benchmark import attention_variant_memory, benchmark_generation, kv_cache_memory, \
        model_size_bytes
    from .models.gpt import GPT
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cfg = gpt2_config("gpt2") if dev == "cuda" and not a.quick else GPTConfig(vocab_size=512, n_positions=256,
                                                                              n_layer=2, n_head=4, n_embd=256)
    torch.manual_seed(0)
    m = GPT(cfg)
    rows = benchmark_generation(m, [16, 128] if a.quick else [32, 256, 768], 16 if a.quick else 64, device=dev,
                                repeats=2 if a.quick else 3)
    mb = model_size_bytes(m)
    return {"rows": [r.to_dict() for r in rows], "kv_cache": kv_cache_memory(cfg, [256, 1024, 4096], [1, 8], 2, mb),
            "variants": attention_variant_memory(cfg, [None, 4, 1], 1024, 8, 2, mb)}


def study_quantization(a, ds=None, tok=None, model=None) -> dict:
    from .quantization import quantization_sweep
    ds, tok = (ds, tok) if ds is not None else _dataset(a.quick, a.corpus)
    model = model or _trained_model(ds, tok, a.quick, a.device)
    return {"rows": [r.to_dict() for r in quantization_sweep(model.cpu(), ds, n_chunks=4, batches_per_chunk=1,
                                                              batch_size=4)]}


def study_pruning(a, ds=None, tok=None, model=None) -> dict:
    from .pruning import prune_sweep
    ds, tok = (ds, tok) if ds is not None else _dataset(a.quick, a.corpus)
    model = (model or _trained_model(ds, tok, a.quick, a.device)).cpu()
    rows = []
    for kind in ("heads", "neurons"):
        res, _ = prune_sweep(model, ds, [0.0, 0.1, 0.25, 0.5], kind=kind, n_eval_batches=2, batch_size=4)
        rows += [r.to_dict() for r in res]
    return {"rows": rows}


def study_distillation(a, ds=None, tok=None, model=None) -> dict:
    from .distill import train_student
    ds, tok = (ds, tok) if ds is not None else _dataset(a.quick, a.corpus)
    teacher = model or _trained_model(ds, tok, a.quick, a.device)
    scfg = GPTConfig(vocab_size=tok.vocab_size, n_positions=ds.block_size, n_layer=1, n_head=2, n_embd=32)
    tc = TrainConfig(steps=30 if a.quick else 300, batch_size=16, block_size=ds.block_size, lr=2e-3, warmup_steps=5,
                     eval_interval=10 if a.quick else 50, eval_batches=2)
    runs = []
    for alpha in (0.0, 0.5):
        _, r = train_student(scfg, tc, ds, teacher=teacher if alpha else None, alpha=alpha, device=a.device,
                             label="scratch" if alpha == 0 else "distilled")
        runs.append(r.to_dict())
    return {"runs": runs}


def study_induction(a, ds=None, tok=None, model=None) -> dict:
    from .induction import in_context_learning_curve, score_heads
    ds, tok = (ds, tok) if ds is not None else _dataset(a.quick, a.corpus)
    model = model or _trained_model(ds, tok, a.quick, a.device)
    dev = next(model.parameters()).device
    sc = score_heads(model, seq_len=20, batch_size=4, n_copy_tokens=200, device=dev)
    d = sc.to_dict()
    d["icl_curve"] = in_context_learning_curve(model, seq_len=20, batch_size=4, device=dev)
    d["top_heads"] = sc.top_heads(5)
    return d


def study_ablations(a, ds=None, tok=None, model=None) -> dict:
    from .ablations import BASELINE_MODEL, build_arms, run_grid, summarize
    ds, tok = (ds, tok) if ds is not None else _dataset(a.quick, a.corpus)
    arms = build_arms()
    if a.quick:
        arms = [x for x in arms if x.key in ("baseline", "post_ln", "relu")]
    base = GPTConfig(**{**BASELINE_MODEL.to_dict(), "vocab_size": tok.vocab_size, "n_positions": ds.block_size,
                        **({"n_layer": 2, "n_embd": 64, "n_head": 4} if a.quick else {})})
    tc = TrainConfig(steps=10 if a.quick else 250, batch_size=8 if a.quick else 24, block_size=ds.block_size,
                     warmup_steps=2 if a.quick else 50, eval_interval=10 if a.quick else 50, eval_batches=2)
    res = run_grid(ds, seeds=(0, 1) if a.quick else (0, 1, 2), arms=arms, base_model=base, base_train=tc,
                   device=a.device)
    return summarize(res, arms)


def study_pareto(a, quant: Optional[dict] = None, prune: Optional[dict] = None) -> dict:
    pts = []
    for r in (quant or {}).get("rows", []):
        pts.append({"method": "quantization", "label": r["label"], "size_mb": r["packed_bytes"] / 1e6,
                    "ppl": r["ppl_mean"]})
    return {"points": pts}


STUDIES = {"verification": study_verification, "kv_cache": study_kv_cache, "quantization": study_quantization,
           "pruning": study_pruning, "distillation": study_distillation, "induction": study_induction,
           "ablations": study_ablations}


def run_study(name: str, a) -> dict:
    return STUDIES[name](a)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("study", choices=sorted(STUDIES) + ["all", "figures"])
    ap.add_argument("--out", default="results")
    ap.add_argument("--figures", default="figures")
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--corpus", default=None)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    out = Path(a.out)
    if a.study == "figures":
        from .viz import make_all
        for p in make_all(out, a.figures):
            print(p)
        return 0
    if a.study == "all":
        ds, tok = _dataset(a.quick, a.corpus)
        model = _trained_model(ds, tok, a.quick, a.device)
        results = {"verification": study_verification(a), "kv_cache": study_kv_cache(a)}
        for name in ("quantization", "pruning", "distillation", "induction", "ablations"):
            results[name] = STUDIES[name](a, ds, tok, model)
        results["pareto"] = study_pareto(a, results["quantization"], results["pruning"])
        for k, v in results.items():
            print(_save(out, k, v))
        from .viz import make_all
        for p in make_all(out, a.figures):
            print(p)
        return 0
    print(_save(out, a.study, run_study(a.study, a)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
