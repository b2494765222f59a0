"""Post-training weight quantization (simulated), with measured sizes and
perplexity error bars.

Reference: src/transformer_internals/quantization.py:75-343.

* symmetric signed integer codes, 2..8 bits, one scale per tensor or per
  output channel (row), ``q = clamp(round(w / s), -2^(b-1), 2^(b-1) - 1)``
  with ``s = amax / (2^(b-1) - 1)``;
* quantize-dequantize ("simulated"): the model computes with exactly the
  matrix an integer kernel would, so quality numbers are real;
* int4 codes packed two per byte (even index -> low nibble, values biased by
  +8), and the packed checkpoint's size measured on disk;
* the tied embedding / head is left alone unless asked (it is the most
  sensitive tensor);
* perplexity reported as mean +- std over disjoint held-out chunks, so a
  quantization delta can be compared with the estimator's own spread.

Added for B200: ``bits="fp8"`` (OCP e4m3 with a per-channel scale to 448),
the format Blackwell's tensor cores consume natively.
"""

from __future__ import annotations

import copy
import math
import statistics
import tempfile
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Literal, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["TARGET_SUFFIXES", "quantize_tensor", "quantize_dequantize", "pack_int4", "unpack_int4",
           "quantize_model", "packed_size_bytes", "perplexity_with_error_bars", "QuantResult", "quantization_sweep"]

Granularity = Literal["per_tensor", "per_channel"]
Bits = Union[int, str]
TARGET_SUFFIXES = ("attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj")
FP8_MAX = 448.0


def _amax(w: torch.Tensor, granularity: str) -> torch.Tensor:
    if granularity == "per_channel":
        return w.abs().amax(dim=1, keepdim=True)
    if granularity == "per_tensor":
        return w.abs().amax()
    raise ValueError(f"unknown granularity {granularity!r}")


def quantize_tensor(w: torch.Tensor, bits: Bits, granularity: Granularity = "per_channel"):
    """Integer codes (int8 storage) or fp8 codes, and the broadcastable scale."""
    amax = _amax(w.float(), granularity)
    if bits == "fp8":
        scale = (amax / FP8_MAX).clamp_min(torch.finfo(torch.float32).tiny)
        return (w.float() / scale).to(torch.float8_e4m3fn), scale
    if not isinstance(bits, int) or bits < 2 or bits > 8:
        raise ValueError(f"bits must be an int in [2, 8] or 'fp8', got {bits!r}")
    qmax, qmin = 2 ** (bits - 1) - 1, -(2 ** (bits - 1))
    scale = (amax / qmax).clamp_min(torch.finfo(torch.float32).tiny)
    return torch.round(w.float() / scale).clamp(qmin, qmax).to(torch.int8), scale


def quantize_dequantize(w: torch.Tensor, bits: Bits, granularity: Granularity = "per_channel") -> torch.Tensor:
    q, s = quantize_tensor(w, bits, granularity)
    return (q.to(torch.float32) * s).to(w.dtype)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """Codes in [-8, 7] -> uint8, two per byte (even index in the low nibble)."""
    v = (q.reshape(-1).to(torch.int16) + 8)
    if v.numel() % 2:
        v = torch.cat([v, v.new_zeros(1)])
    return (v[0::2] | (v[1::2] << 4)).to(torch.uint8)


def unpack_int4(packed: torch.Tensor, numel: int) -> torch.Tensor:
    p = packed.to(torch.int16)
    both = torch.stack([(p & 0xF) - 8, (p >> 4) - 8], dim=1).reshape(-1)
    return both[:numel].to(torch.int8)


def packed_size_bytes(model: nn.Module, codes: dict, bits: Bits) -> int:
    """Bytes of a checkpoint that really stores the packed codes (+ fp32
    scales and shapes) and every other tensor in fp32, measured on disk."""
    payload = {}
    for name, (q, s) in codes.items():
        if bits == "fp8":
            payload[f"{name}.q"] = q.view(torch.uint8)
        else:
            payload[f"{name}.q"] = pack_int4(q) if bits == 4 else q
        payload[f"{name}.scale"] = s.float()
        payload[f"{name}.shape"] = torch.tensor(list(q.shape), dtype=torch.int32)
    done = {f"{n}.weight" for n in codes}
    seen = set()
    for n, p in model.named_parameters():
        if n in done or id(p) in seen:
            continue
        seen.add(id(p))
        payload[n] = p.detach().float().cpu()
    with tempfile.TemporaryDirectory() as d:
        f = Path(d) / "q.pt"
        torch.save(payload, f)
        return f.stat().st_size


def quantize_model(model: nn.Module, bits: Bits, granularity: Granularity = "per_channel",
                   include_embedding: bool = False):
    """A deep copy with the target projections (and optionally ``wte``)
    quantize-dequantized, plus a stats record."""
    qm = copy.deepcopy(model)
    codes, n_q = {}, 0
    for name, mod in qm.named_modules():
        target = name.endswith(TARGET_SUFFIXES) or (include_embedding and name == "wte")
        if not target or not isinstance(mod, (nn.Linear, nn.Embedding)):
            continue
        with torch.no_grad():
            w = mod.weight.data
            q, s = quantize_tensor(w, bits, granularity)
            codes[name] = (q.cpu(), s.cpu())
            mod.weight.data = (q.to(torch.float32) * s).to(w.dtype)
        n_q += w.numel()
    total = sum(p.numel() for p in {id(p): p for p in model.parameters()}.values())
    stats = {"bits": bits, "granularity": granularity, "include_embedding": include_embedding,
             "n_quantized_tensors": len(codes), "n_quantized_params": n_q, "n_total_params": total,
             "fraction_quantized": n_q / total, "packed_bytes": packed_size_bytes(qm, codes, bits),
             "fp32_bytes": total * 4}
    stats["compression_ratio"] = stats["fp32_bytes"] / stats["packed_bytes"]
    return qm, stats


@torch.no_grad()
def perplexity_with_error_bars(model: nn.Module, dataset, n_chunks: int = 8, batches_per_chunk: int = 2,
                               batch_size: int = 4, device="cpu") -> dict:
    model = model.to(device).eval()
    batches = dataset.sequential_batches("val", batch_size=batch_size, limit=n_chunks * batches_per_chunk)
    losses = []
    for c in range(0, len(batches), batches_per_chunk):
        tot, n = 0.0, 0
        for x, y in batches[c:c + batches_per_chunk]:
            lo = model(x.to(device))["logits"].float().cpu()
            tot += F.cross_entropy(lo.reshape(-1, lo.size(-1)), y.reshape(-1), reduction="sum").item()
            n += y.numel()
        if n:
            losses.append(tot / n)
    ppl = [math.exp(v) for v in losses]
    sd = lambda xs: statistics.stdev(xs) if len(xs) > 1 else 0.0  # noqa: E731
    return {"loss_mean": statistics.fmean(losses), "loss_std": sd(losses), "ppl_mean": statistics.fmean(ppl),
            "ppl_std": sd(ppl), "chunk_losses": losses, "n_chunks": len(losses)}


@dataclass
class QuantResult:
    label: str
    bits: object
    granularity: str
    include_embedding: bool
    ppl_mean: float
    ppl_std: float
    loss_mean: float
    delta_ppl_vs_fp32: float
    packed_bytes: int
    compression_ratio: float
    extra: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        return asdict(self)


def quantization_sweep(model: nn.Module, dataset, settings=((8, "per_channel"), (4, "per_channel"),
                                                             (4, "per_tensor"), ("fp8", "per_channel")),
                       device="cpu", **ppl_kw) -> list[QuantResult]:
    """fp32 baseline then one row per (bits, granularity)."""
    base = perplexity_with_error_bars(model, dataset, device=device, **ppl_kw)
    fp32_bytes = packed_size_bytes(model, {}, 8)
    rows = [QuantResult("fp32", 32, "-", False, base["ppl_mean"], base["ppl_std"], base["loss_mean"], 0.0,
                        fp32_bytes, 1.0)]
    for bits, gran in settings:
        qm, st = quantize_model(model, bits, gran)
        r = perplexity_with_error_bars(qm, dataset, device=device, **ppl_kw)
        rows.append(QuantResult(f"{'fp8' if bits == 'fp8' else 'int' + str(bits)}-{gran}", bits, gran, False,
                                r["ppl_mean"], r["ppl_std"], r["loss_mean"], r["ppl_mean"] - base["ppl_mean"],
                                st["packed_bytes"], st["compression_ratio"]))
    return rows
