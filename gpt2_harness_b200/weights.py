"""Load HuggingFace GPT-2 checkpoints into this framework's parameter names.

Reference: src/transformer_internals/weights.py:61-206.

* HF stores the four projections as ``Conv1D`` ([in, out]); ``nn.Linear``
  wants [out, in], so ``c_attn``, ``c_proj`` (both) and ``c_fc`` weights are
  transposed;
* both layouts are accepted: bare ``GPT2Model`` keys (``h.0...``) and
  ``GPT2LMHeadModel`` keys (``transformer.h.0...``);
* the causal-mask buffers (``.attn.bias``, ``.attn.masked_bias``, matched with
  the leading dot so ``c_attn.bias`` survives) and the tied ``lm_head.weight``
  are dropped;
* embedding / final-norm shapes are checked against the target config.

This machine has no network, so :func:`resolve_checkpoint_dir` only looks at
an explicit directory, ``$GPT2_CHECKPOINT_DIR``, and the local HuggingFace
cache; ``save_hf_checkpoint`` writes a checkpoint in the HF layout (used by
the tests with a randomly initialised HF model).
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import Any, Optional

import torch

from .config import GPTConfig, gpt2_config
from .models.gpt import GPT

__all__ = ["CONV1D_TRANSPOSED", "resolve_checkpoint_dir", "load_gpt2_state_dict", "convert_hf_state_dict",
           "to_hf_state_dict", "save_hf_checkpoint", "load_pretrained_gpt2"]

CONV1D_TRANSPOSED = ("attn.c_attn.weight", "attn.c_proj.weight", "mlp.c_fc.weight", "mlp.c_proj.weight")
_DROPPED_SUFFIXES = (".attn.bias", ".attn.masked_bias")


def resolve_checkpoint_dir(model_id: str = "openai-community/gpt2", checkpoint_dir: Optional[str] = None) -> Path:
    """A local directory with ``model.safetensors`` (and usually vocab.json +
    merges.txt). Looks at ``checkpoint_dir``, ``$GPT2_CHECKPOINT_DIR``, then the
    HuggingFace cache snapshots of ``model_id``; never downloads."""
    cands = []
    if checkpoint_dir:
        cands.append(Path(checkpoint_dir))
    if os.environ.get("GPT2_CHECKPOINT_DIR"):
        cands.append(Path(os.environ["GPT2_CHECKPOINT_DIR"]))
    hub = Path(os.environ.get("HF_HUB_CACHE", Path(os.environ.get("HF_HOME", Path.home() / ".cache/huggingface"))
                              / "hub"))
    snap = hub / ("models--" + model_id.replace("/", "--")) / "snapshots"
    if snap.is_dir():
        cands.extend(sorted(snap.iterdir()))
    for c in cands:
        if (c / "model.safetensors").exists():
            return c
    raise FileNotFoundError(f"no local checkpoint for {model_id!r} (looked at {[str(c) for c in cands]}); "
                            "pass checkpoint_dir or set GPT2_CHECKPOINT_DIR")


def load_gpt2_state_dict(checkpoint_dir) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file
    path = Path(checkpoint_dir) / "model.safetensors"
    if not path.exists():
        raise FileNotFoundError(f"no model.safetensors under {checkpoint_dir}")
    return load_file(str(path))


def convert_hf_state_dict(hf_state: dict, config: GPTConfig) -> dict[str, torch.Tensor]:
    """HF names/layouts -> ours (loadable with strict=False: lm_head is tied)."""
    out = {}
    for raw, t in hf_state.items():
        key = raw[len("transformer."):] if raw.startswith("transformer.") else raw
        if key.endswith(_DROPPED_SUFFIXES) or key == "lm_head.weight":
            continue
        if key.endswith(CONV1D_TRANSPOSED):
            t = t.t().contiguous()
        out[key] = t
    want = {"wte.weight": (config.vocab_size, config.n_embd), "wpe.weight": (config.n_positions, config.n_embd),
            "ln_f.weight": (config.n_embd,)}
    for k, shape in want.items():
        if k in out and tuple(out[k].shape) != shape:
            raise ValueError(f"{k}: checkpoint has {tuple(out[k].shape)}, model wants {shape}")
    return out


def to_hf_state_dict(state: dict) -> dict[str, torch.Tensor]:
    """Ours -> HF ``GPT2LMHeadModel`` layout (inverse of the conversion)."""
    out = {}
    for k, t in state.items():
        if k.endswith("causal_mask"):
            continue
        if k.endswith(CONV1D_TRANSPOSED):
            t = t.t().contiguous()
        out[k if k == "lm_head.weight" else "transformer." + k] = t.detach().cpu().contiguous()
    if "lm_head.weight" not in out:
        out["lm_head.weight"] = out["transformer.wte.weight"]
    return out


def save_hf_checkpoint(state: dict, out_dir) -> Path:
    """Write ``model.safetensors`` in the HF GPT-2 layout (tied head omitted)."""
    from safetensors.torch import save_file
    d = Path(out_dir)
    d.mkdir(parents=True, exist_ok=True)
    hf = to_hf_state_dict(state)
    hf.pop("lm_head.weight", None)
    save_file({k: v.clone() for k, v in hf.items()}, str(d / "model.safetensors"))
    return d


def load_pretrained_gpt2(size: str = "gpt2", checkpoint_dir=None, device="cpu", dtype=torch.float32,
                         **overrides: Any) -> tuple[GPT, Path]:
    """Build ``GPT`` for a released size and load a local checkpoint into it."""
    model_id = "openai-community/gpt2" if size == "gpt2" else f"openai-community/{size}"
    path = resolve_checkpoint_dir(model_id, checkpoint_dir)
    config = gpt2_config(size, dropout=0.0, **overrides)
    model = GPT(config)
    missing, unexpected = model.load_state_dict(convert_hf_state_dict(load_gpt2_state_dict(path), config),
                                                strict=False)
    missing = [k for k in missing if k != "lm_head.weight" and not k.endswith("causal_mask")]
    if missing or unexpected:
        raise RuntimeError(f"checkpoint mismatch: missing={missing} unexpected={unexpected}")
    return model.to(device=device, dtype=dtype).eval(), path
