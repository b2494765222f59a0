"""Single-process training loop (research harness), on the oracle model or
on the B200 engine.

Reference: src/transformer_internals/train.py:40-308. Semantics kept:

* AdamW from ``configure_optimizers`` (decay on >=2-D tensors), linear warmup
  then cosine decay to ``min_lr_ratio * lr``;
* gradient accumulation (loss / accum), global-norm clipping with the
  pre-clip norm recorded every step, optional autocast (bf16, or fp16 with a
  GradScaler that skips non-finite steps);
* a divergence flag instead of an exception (a diverging arm is a result);
* training batches from one seeded generator, evaluation batches from a
  fresh generator with a fixed seed at every eval, so every arm of an
  ablation sees byte-identical batches.

``backend="native"`` runs the same loop on :class:`~gpt2_harness_b200.models.
engine.Engine` (bf16 tensor-core kernels, fp32 master weights, fused AdamW);
accumulation averages micro-batch gradients through the optimiser's gradient
scale, so the update equals one step on the concatenated batch.

    python -m gpt2_harness_b200.train --steps 200 --backend native
"""

from __future__ import annotations

import argparse
import json
import math
import platform
import random
import time
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

import numpy as np
import torch

from .config import GPTConfig, TrainConfig
from .data import TokenDataset
from .models.gpt import GPT
from .precision import autocast_context, make_grad_scaler, master_weight_report, resolve_amp
from .trainer import lr_at_step

__all__ = ["pick_device", "set_seed", "lr_at_step", "TrainResult", "estimate_loss", "train"]


def pick_device(prefer: Optional[str] = None) -> torch.device:
    if prefer is not None:
        return torch.device(prefer)
    if torch.cuda.is_available():
        return torch.device("cuda")
    if getattr(torch.backends, "mps", None) is not None and torch.backends.mps.is_available():
        return torch.device("mps")
    return torch.device("cpu")


def set_seed(seed: int) -> None:
    random.seed(seed)
    np.random.seed(seed)  # noqa: NPY002
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


@dataclass
class TrainResult:
    history: list = field(default_factory=list)   # {step, train_loss, val_loss, lr}
    final_val_loss: float = float("nan")
    best_val_loss: float = float("nan")
    steps: int = 0
    wall_clock_s: float = 0.0
    tokens_seen: int = 0
    n_params: int = 0
    diverged: bool = False
    grad_norms: list = field(default_factory=list)  # pre-clip global norm per step
    meta: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        return asdict(self)


@torch.no_grad()
def estimate_loss(model, dataset: TokenDataset, cfg: TrainConfig, device, generator: torch.Generator) -> dict:
    """Mean loss over ``eval_batches`` batches of each split. ``model`` is an
    oracle ``GPT`` or a native ``Engine``."""
    out = {}
    is_module = isinstance(model, torch.nn.Module)
    if is_module:
        was = model.training
        model.eval()
    for split in ("train", "val"):
        tot = 0.0
        for _ in range(cfg.eval_batches):
            x, y = dataset.get_batch(split, cfg.batch_size, device=device, generator=generator)
            loss = model(x, targets=y)["loss"] if is_module else model.forward(x, y)
            tot += float(loss.item())
        out[split] = tot / cfg.eval_batches
    if is_module:
        model.train(was)
    return out


def _eval_record(model, dataset, cfg, device, seed, step, lr, result, progress):
    gen = torch.Generator().manual_seed(seed)
    losses = estimate_loss(model, dataset, cfg, device, gen)
    result.history.append({"step": step, "train_loss": losses["train"], "val_loss": losses["val"], "lr": lr})
    if progress:
        print(f"  step {step:5d}/{cfg.steps}  train {losses['train']:.4f}  val {losses['val']:.4f}  lr {lr:.2e}",
              flush=True)


def train(model_config: GPTConfig, train_config: TrainConfig, dataset: TokenDataset, device=None,
          progress: bool = False, backend: str = "oracle"):
    """Train and return ``(model, TrainResult)``; ``model`` is a ``GPT``
    (oracle) or an ``Engine`` (native)."""
    if backend not in ("oracle", "native"):
        raise ValueError(f"backend must be 'oracle' or 'native', got {backend!r}")
    cfg, mcfg = train_config, model_config
    device = pick_device(device) if not isinstance(device, torch.device) else device
    set_seed(cfg.seed)
    train_gen = torch.Generator().manual_seed(cfg.seed)
    eval_seed = cfg.seed + 10_000
    if backend == "native":
        return _train_native(mcfg, cfg, dataset, device, train_gen, eval_seed, progress)
    model = GPT(mcfg).to(device)
    model.train()
    opt = model.configure_optimizers(cfg.weight_decay, cfg.lr, cfg.betas, cfg.eps)
    amp = resolve_amp(cfg.amp, cfg.amp_dtype, device)
    scaler = make_grad_scaler(amp)
    res = TrainResult(n_params=model.num_parameters())
    res.meta = {"backend": "oracle", "device": str(device), "platform": platform.platform(),
                "torch": torch.__version__, "model_config": mcfg.to_dict(), "train_config": cfg.to_dict(),
                "precision": amp.to_dict(), "master_weights": master_weight_report(model)}
    t0 = time.perf_counter()
    for step in range(cfg.steps):
        lr = lr_at_step(step, cfg)
        for g in opt.param_groups:
            g["lr"] = lr
        opt.zero_grad(set_to_none=True)
        for _ in range(cfg.grad_accum):
            x, y = dataset.get_batch("train", cfg.batch_size, device=device, generator=train_gen)
            with autocast_context(amp):
                loss = model(x, targets=y)["loss"]
            scaled = loss / cfg.grad_accum
            (scaler.scale(scaled) if scaler is not None else scaled).backward()
        if scaler is not None:
            scaler.unscale_(opt)
        res.grad_norms.append(float(torch.nn.utils.clip_grad_norm_(model.parameters(), cfg.grad_clip)))
        if scaler is None:
            opt.step()
        else:
            scaler.step(opt)
            scaler.update()
        res.tokens_seen += cfg.batch_size * cfg.grad_accum * cfg.block_size
        res.steps = step + 1
        if not math.isfinite(float(loss.item())):
            res.diverged = True
            break
        if (step + 1) % cfg.eval_interval == 0 or step == cfg.steps - 1:
            _eval_record(model, dataset, cfg, device, eval_seed, step + 1, lr, res,
                         progress and ((step + 1) % cfg.log_every == 0 or step == cfg.steps - 1))
    res.wall_clock_s = time.perf_counter() - t0
    if res.history:
        res.final_val_loss = res.history[-1]["val_loss"]
        res.best_val_loss = min(h["val_loss"] for h in res.history)
    return model, res


def _train_native(mcfg, cfg, dataset, device, train_gen, eval_seed, progress):
    from .models import engine as engine_mod
    from .models.engine import Engine, OptimConfig
    if device.type not in engine_mod.DEVICE_TYPES:
        raise RuntimeError("the native backend needs a CUDA device")
    eng = Engine(mcfg, device, optim=OptimConfig(lr=cfg.lr, betas=tuple(cfg.betas), eps=cfg.eps,
                                                 weight_decay=cfg.weight_decay, grad_clip=cfg.grad_clip),
                 seed=cfg.seed)
    eng.grad_scale = 1.0 / cfg.grad_accum
    res = TrainResult(n_params=eng.layout.num_parameters)
    res.meta = {"backend": "native", "device": str(device), "platform": platform.platform(),
                "torch": torch.__version__, "model_config": mcfg.to_dict(), "train_config": cfg.to_dict(),
                "precision": {"compute": "bf16", "master": "fp32", "optimizer": "fused AdamW"}}
    t0 = time.perf_counter()
    for step in range(cfg.steps):
        lr = lr_at_step(step, cfg)
        eng.set_lr(lr)
        for j in range(cfg.grad_accum):
            x, y = dataset.get_batch("train", cfg.batch_size, device=device, generator=train_gen, pin=True)
            loss = eng.forward(x, y)
            eng.backward(x, accumulate=j > 0)
        eng.optimizer_step()
        res.grad_norms.append(float(eng.grad_norm.item()))
        res.tokens_seen += cfg.batch_size * cfg.grad_accum * cfg.block_size
        res.steps = step + 1
        if not math.isfinite(float(loss.item())):
            res.diverged = True
            break
        if (step + 1) % cfg.eval_interval == 0 or step == cfg.steps - 1:
            _eval_record(eng, dataset, cfg, device, eval_seed, step + 1, lr, res,
                         progress and ((step + 1) % cfg.log_every == 0 or step == cfg.steps - 1))
    res.wall_clock_s = time.perf_counter() - t0
    if res.history:
        res.final_val_loss = res.history[-1]["val_loss"]
        res.best_val_loss = min(h["val_loss"] for h in res.history)
    return eng, res


def _main() -> None:
    ap = argparse.ArgumentParser(description="train a GPT-2 on a local or synthetic corpus")
    ap.add_argument("--backend", choices=["oracle", "native"], default="native")
    ap.add_argument("--corpus", default=None, help="text file; synthetic stories when absent")
    ap.add_argument("--vocab", type=int, default=2048, help="BPE vocabulary trained on the corpus")
    ap.add_argument("--n-layer", type=int, default=4)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=256)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--block", type=int, default=128)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    from .data import encode_corpus, load_text, synthetic_stories
    from .tokenizer import train_bpe
    text = load_text(a.corpus) if a.corpus else synthetic_stories(4000)
    tok = train_bpe(text.split("\n\n")[:2000], a.vocab)
    ds = TokenDataset(encode_corpus(tok, text, cache=False), a.block)
    mcfg = GPTConfig(vocab_size=tok.vocab_size, n_positions=a.block, n_layer=a.n_layer, n_head=a.n_head,
                     n_embd=a.n_embd)
    tcfg = TrainConfig(steps=a.steps, batch_size=a.batch, block_size=a.block, lr=a.lr,
                       warmup_steps=max(1, a.steps // 10), eval_interval=max(1, a.steps // 4), eval_batches=5)
    _, res = train(mcfg, tcfg, ds, backend=a.backend, progress=True)
    out = {k: v for k, v in res.to_dict().items() if k != "grad_norms"}
    print(json.dumps(out)[:2000])
    if a.out:
        with open(a.out, "w") as f:
            json.dump(res.to_dict(), f)


if __name__ == "__main__":
    _main()
