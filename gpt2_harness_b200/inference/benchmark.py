"""Inference efficiency: cached vs uncached latency, KV-cache memory.

Reference: src/transformer_internals/benchmark.py:61-369 (``time_call`` with
warm-up and median of repeats, ``benchmark_generation`` over prompt lengths
with both cache arms, exact cache-size formula
``2 * n_layer * kv_heads * head_dim * dtype_bytes`` per token per sequence,
GQA/MQA savings ``n_head / n_kv_head``, and a check of the formula against the
tensors a real cache allocates).

Added here: a third arm, the B200 decode engine (preallocated cache, fused
decode attention, CUDA-graph step), and CUDA-event timing on GPUs.

    python -m gpt2_harness_b200.inference.benchmark --prompt-lens 32 256 --new-tokens 64
"""

from __future__ import annotations

import argparse
import json
import statistics
import time
from dataclasses import asdict, dataclass, field
from typing import Any, Callable, Optional

import torch

from ..config import GPTConfig
from ..models.gpt import GPT, KVCache
from .sampling import generate

__all__ = ["synchronize", "time_call", "BenchRow", "benchmark_generation", "model_size_bytes",
           "kv_cache_memory", "attention_variant_memory", "measure_cache_tensor_bytes"]


def synchronize(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    elif device.type == "mps":
        torch.mps.synchronize()


def time_call(fn: Callable[[], Any], device: torch.device, repeats: int = 5, warmup: int = 2) -> dict:
    """Median / min / mean / std seconds of ``fn`` after ``warmup`` untimed
    calls. On CUDA each repeat is bracketed by events on the current stream."""
    device = torch.device(device)
    for _ in range(warmup):
        fn()
    synchronize(device)
    samples = []
    for _ in range(repeats):
        if device.type == "cuda":
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            samples.append(e0.elapsed_time(e1) / 1e3)
        else:
            t0 = time.perf_counter()
            fn()
            synchronize(device)
            samples.append(time.perf_counter() - t0)
    return {"median_s": statistics.median(samples), "min_s": min(samples), "mean_s": statistics.fmean(samples),
            "std_s": statistics.stdev(samples) if len(samples) > 1 else 0.0}


@dataclass
class BenchRow:
    arm: str                 # "cached", "uncached" or "native"
    prompt_len: int
    new_tokens: int
    batch_size: int
    median_s: float
    min_s: float
    std_s: float
    ms_per_token: float
    tokens_per_s: float
    device: str
    extra: dict = field(default_factory=dict)

    @property
    def use_cache(self) -> bool:
        return self.arm != "uncached"

    def to_dict(self) -> dict:
        d = asdict(self)
        d.update(d.pop("extra"))
        d["use_cache"] = self.use_cache
        return d


@torch.no_grad()
def benchmark_generation(model: GPT, prompt_lens: list[int], new_tokens: int = 64, batch_size: int = 1,
                         device="cpu", repeats: int = 3, warmup: int = 1, both_arms: bool = True,
                         native: Optional[bool] = None) -> list[BenchRow]:
    """Greedy generation latency per prompt length: cached and (optionally)
    uncached oracle arms, plus the native engine on CUDA."""
    device = torch.device(device)
    model = model.to(device).eval()
    if native is None:
        native = device.type == "cuda"
    rows: list[BenchRow] = []
    for T0 in prompt_lens:
        if T0 + new_tokens > model.config.n_positions:
            continue
        torch.manual_seed(0)
        prompt = torch.randint(0, model.config.vocab_size, (batch_size, T0), device=device)
        arms: list[tuple[str, Callable]] = [("cached", lambda: generate(model, prompt, new_tokens, use_cache=True))]
        if both_arms:
            arms.append(("uncached", lambda: generate(model, prompt, new_tokens, use_cache=False)))
        if native:
            from .decode import DecodeEngine
            eng = DecodeEngine.from_model(model, batch=batch_size, max_len=T0 + new_tokens, device=device)
            arms.append(("native", lambda: eng.generate(prompt, new_tokens)))
        for arm, fn in arms:
            st = time_call(fn, device, repeats=repeats, warmup=warmup)
            rows.append(BenchRow(arm, T0, new_tokens, batch_size, st["median_s"], st["min_s"], st["std_s"],
                                 1e3 * st["median_s"] / new_tokens, new_tokens * batch_size / st["median_s"],
                                 str(device)))
    return rows


def model_size_bytes(model: torch.nn.Module, count_tied_once: bool = True) -> int:
    """Parameter bytes; a tied embedding/head counts once unless asked."""
    return sum(p.numel() * p.element_size() for _, p in model.named_parameters(remove_duplicate=count_tied_once))


def kv_cache_memory(config: GPTConfig, seq_lens: list[int], batch_sizes: list[int], dtype_bytes: int = 4,
                    model_bytes: Optional[int] = None) -> list[dict]:
    per_tok = config.kv_cache_bytes_per_token(dtype_bytes)
    out = []
    for bs in batch_sizes:
        for t in seq_lens:
            total = per_tok * t * bs
            out.append({"seq_len": t, "batch_size": bs, "dtype_bytes": dtype_bytes, "bytes_per_token_per_seq": per_tok,
                        "cache_bytes": total, "cache_mb": total / 1e6, "model_bytes": model_bytes,
                        "cache_fraction_of_model": total / model_bytes if model_bytes else None})
    return out


def attention_variant_memory(base: GPTConfig, kv_head_options: list, seq_len: int = 1024, batch_size: int = 8,
                             dtype_bytes: int = 4, model_bytes: Optional[int] = None) -> list[dict]:
    """Cache size of MHA / GQA-k / MQA; the saving is exactly n_head / n_kv_head."""
    mha = GPTConfig(**{**base.to_dict(), "n_kv_head": None}).kv_cache_bytes_per_token(dtype_bytes)
    rows = []
    for opt in kv_head_options:
        cfg = GPTConfig(**{**base.to_dict(), "n_kv_head": opt})
        per_tok = cfg.kv_cache_bytes_per_token(dtype_bytes)
        kv = cfg.kv_heads
        total = per_tok * seq_len * batch_size
        rows.append({"n_kv_head": kv, "variant": "MHA" if kv == cfg.n_head else ("MQA" if kv == 1 else f"GQA-{kv}"),
                     "bytes_per_token_per_seq": per_tok, "cache_mb": total / 1e6, "reduction_vs_mha": mha / per_tok,
                     "seq_len": seq_len, "batch_size": batch_size,
                     "cache_fraction_of_model": total / model_bytes if model_bytes else None})
    return rows


@torch.no_grad()
def measure_cache_tensor_bytes(model: GPT, prompt_len: int, new_tokens: int, batch_size: int = 1,
                               device="cpu") -> dict:
    """Bytes the grown cache really holds after decoding, against the formula."""
    dev = torch.device(device)
    model = model.to(dev).eval()
    idx = torch.randint(0, model.config.vocab_size, (batch_size, prompt_len), device=dev)
    cache = KVCache.empty(model.config.n_layer)
    out = model(idx, cache=cache)
    for _ in range(new_tokens):
        nxt = out["logits"][:, -1:].argmax(-1)
        out = model(nxt, cache=cache)
    measured = sum(t.numel() * t.element_size() for lst in (cache.keys, cache.values) for t in lst if t is not None)
    total = prompt_len + new_tokens
    predicted = model.config.kv_cache_bytes_per_token(next(model.parameters()).element_size()) * total * batch_size
    return {"prompt_len": prompt_len, "new_tokens": new_tokens, "batch_size": batch_size, "total_len": total,
            "measured_bytes": measured, "predicted_bytes": predicted, "ratio": measured / predicted}


def _main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--model", default="gpt2")
    ap.add_argument("--prompt-lens", type=int, nargs="+", default=[32, 256, 768])
    ap.add_argument("--new-tokens", type=int, default=64)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--no-uncached", action="store_true")
    a = ap.parse_args()
    from ..config import gpt2_config
    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    torch.manual_seed(0)
    model = GPT(gpt2_config(a.model))
    if dev.type == "cuda":
        model = model.to(dev)
    rows = benchmark_generation(model, a.prompt_lens, a.new_tokens, a.batch, dev, a.repeats,
                                both_arms=not a.no_uncached)
    for r in rows:
        print(json.dumps(r.to_dict()))
    mb = model_size_bytes(model)
    print(json.dumps({"kv_cache": kv_cache_memory(model.config, [1024], [1, 8], 2, mb)}))


if __name__ == "__main__":
    _main()
