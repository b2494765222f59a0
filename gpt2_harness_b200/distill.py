"""Knowledge distillation into a small student.

Reference: src/transformer_internals/distill.py:52-255. Loss =
(1 - alpha) * CE(student, labels) + alpha * T^2 * KL(softmax(t/T) || softmax(s/T))
with ``batchmean`` KL (Hinton et al., 2015); ``alpha = 0`` is the from-scratch
control through the same code path. Validation loss (hard-label CE) is scored
on a fixed set of batches re-seeded at every evaluation, so arms compare on
identical windows.
"""

from __future__ import annotations

import math
import time
from dataclasses import asdict, dataclass, field
from typing import Optional

import torch
import torch.nn.functional as F

from .config import GPTConfig, TrainConfig
from .models.gpt import GPT
from .train import lr_at_step, pick_device, set_seed

__all__ = ["STUDENT_CONFIG", "distillation_loss", "DistillResult", "train_student"]

#: The 4-layer student of the reference study (vocabulary set by the data).
STUDENT_CONFIG = GPTConfig(vocab_size=50257, n_positions=128, n_layer=4, n_head=8, n_embd=256, dropout=0.0)


def distillation_loss(student_logits: torch.Tensor, teacher_logits: torch.Tensor, targets: torch.Tensor,
                      temperature: float = 2.0, alpha: float = 0.5):
    """(total, ce, kl); ``kl`` already carries the T^2 factor."""
    V = student_logits.size(-1)
    s = student_logits.reshape(-1, V)
    ce = F.cross_entropy(s, targets.reshape(-1))
    if alpha == 0.0:
        return ce, ce, ce.new_zeros(())
    log_p = F.log_softmax(s / temperature, dim=-1)
    q = F.softmax(teacher_logits.reshape(-1, V) / temperature, dim=-1)
    kl = F.kl_div(log_p, q, reduction="batchmean") * temperature ** 2
    return (1.0 - alpha) * ce + alpha * kl, ce, kl


@dataclass
class DistillResult:
    label: str
    alpha: float
    temperature: float
    seed: int
    final_val_loss: float = float("nan")
    final_val_ppl: float = float("nan")
    history: list = field(default_factory=list)
    wall_clock_s: float = 0.0
    n_params: int = 0
    teacher_params: int = 0
    meta: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        return asdict(self)


@torch.no_grad()
def _val_loss(model: GPT, dataset, cfg: TrainConfig, device) -> float:
    was = model.training
    model.eval()
    g = torch.Generator().manual_seed(1234)
    tot = 0.0
    for _ in range(cfg.eval_batches):
        x, y = dataset.get_batch("val", cfg.batch_size, device=device, generator=g)
        tot += float(model(x, targets=y)["loss"])
    model.train(was)
    return tot / cfg.eval_batches


def train_student(student_config: GPTConfig, train_config: TrainConfig, dataset, teacher: Optional[GPT] = None,
                  alpha: float = 0.0, temperature: float = 2.0, device=None, label: str = "student",
                  progress: bool = False):
    if alpha > 0 and teacher is None:
        raise ValueError("distillation requires a teacher")
    cfg = train_config
    device = pick_device(device) if not isinstance(device, torch.device) else device
    set_seed(cfg.seed)
    student = GPT(student_config).to(device).train()
    opt = student.configure_optimizers(cfg.weight_decay, cfg.lr, cfg.betas, cfg.eps)
    if teacher is not None:
        teacher = teacher.to(device).eval()
        teacher.requires_grad_(False)
    gen = torch.Generator().manual_seed(cfg.seed)
    res = DistillResult(label, alpha, temperature, cfg.seed, n_params=student.num_parameters(),
                        teacher_params=teacher.num_parameters() if teacher is not None else 0)
    t0 = time.perf_counter()
    for step in range(cfg.steps):
        lr = lr_at_step(step, cfg)
        for g in opt.param_groups:
            g["lr"] = lr
        opt.zero_grad(set_to_none=True)
        x, y = dataset.get_batch("train", cfg.batch_size, device=device, generator=gen)
        s_logits = student(x)["logits"]
        if alpha > 0:
            with torch.no_grad():
                t_logits = teacher(x)["logits"]
        else:
            t_logits = s_logits.detach()
        loss, ce, kl = distillation_loss(s_logits, t_logits, y, temperature, alpha)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(student.parameters(), cfg.grad_clip)
        opt.step()
        if (step + 1) % cfg.eval_interval == 0 or step == cfg.steps - 1:
            v = _val_loss(student, dataset, cfg, device)
            res.history.append({"step": step + 1, "val_loss": v, "train_ce": float(ce.detach()), "kl": float(kl.detach()),
                                "lr": lr})
            if progress:
                print(f"  [{label}] step {step + 1}/{cfg.steps} val {v:.4f}", flush=True)
    res.wall_clock_s = time.perf_counter() - t0
    if res.history:
        res.final_val_loss = res.history[-1]["val_loss"]
        res.final_val_ppl = math.exp(min(res.final_val_loss, 20.0))
    return student, res
