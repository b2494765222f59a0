"""The native engine against the PyTorch oracle model (same weights).

Forward loss and every parameter gradient are compared with the fp32 oracle
(tolerance set by bf16 matmul inputs), and a 10-step training trajectory is
compared with torch bf16 autocast + torch.optim.AdamW.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from gpt2_harness_b200.config import GPTConfig  # noqa: E402
from gpt2_harness_b200.models.engine import Engine, OptimConfig  # noqa: E402
from gpt2_harness_b200.models.gpt import GPT  # noqa: E402
from gpt2_harness_b200.ops import native as N  # noqa: E402


def small_config(**kw):
    base = dict(vocab_size=1000, n_positions=256, n_layer=2, n_head=4, n_embd=256)
    base.update(kw)
    return GPTConfig(**base)


def make_batch(cfg, B, T, seed=0):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, cfg.vocab_size, (B, T), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (B, T), generator=g)
    return idx, tgt


@pytest.mark.parametrize("B,T,fused_ce,kv", [(2, 128, False, None), (3, 200, False, None),
                                              (3, 200, True, None), (2, 256, False, 2), (2, 128, False, 1)])
def test_engine_loss_and_grads_match_oracle(B, T, fused_ce, kv):
    """kv: key/value heads (grouped-query / multi-query attention) or None."""
    torch.manual_seed(0)
    cfg = small_config(n_kv_head=kv)
    model = GPT(cfg)
    idx, tgt = make_batch(cfg, B, T)
    tgt[0, :5] = -100
    out = model(idx, tgt)
    out["loss"].backward()
    ref_grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}

    dev = torch.device("cuda", 0)
    eng = Engine.from_module(model, dev)
    eng.fused_ce = fused_ce
    loss = eng.forward(idx.to(dev), tgt.to(dev))
    eng.backward(idx.to(dev))
    torch.cuda.synchronize()
    N.check_errors()
    assert abs(loss.item() - out["loss"].item()) < 2e-2 * abs(out["loss"].item())
    for name, ref in ref_grads.items():
        got = eng.g32(name).cpu()
        err = (got - ref).abs().max().item() / (ref.abs().max().item() + 1e-12)
        assert err < 6e-2, f"{name}: rel err {err:.3e}"


def test_engine_training_tracks_autocast_adamw():
    torch.manual_seed(1)
    cfg = small_config(n_layer=2)
    dev = torch.device("cuda", 0)
    model = GPT(cfg).to(dev)
    eng = Engine.from_module(model, dev, optim=OptimConfig(lr=1e-3, grad_clip=1.0))
    opt = model.configure_optimizers(0.1, 1e-3, (0.9, 0.95))
    losses_ref, losses_eng = [], []
    for step in range(10):
        idx, tgt = make_batch(cfg, 4, 128, seed=100 + step % 3)
        idx, tgt = idx.to(dev), tgt.to(dev)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(idx, tgt)["loss"]
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        losses_ref.append(loss.item())
        losses_eng.append(eng.train_step(idx, tgt).item())
    N.check_errors()
    for a, b in zip(losses_ref, losses_eng):
        assert abs(a - b) < 0.05 * abs(a), (losses_ref, losses_eng)
    assert losses_eng[-1] < losses_eng[0]


def test_engine_gpt2_small_shapes_run():
    """Full GPT-2 124M shapes at a short sequence: finite loss near ln(V)."""
    cfg = GPTConfig()
    dev = torch.device("cuda", 0)
    eng = Engine(cfg, dev, seed=0)
    assert eng.layout.num_parameters == 124_439_808
    idx = torch.randint(0, cfg.vocab_size, (2, 256), device=dev)
    tgt = torch.randint(0, cfg.vocab_size, (2, 256), device=dev)
    l0 = eng.train_step(idx, tgt).item()
    l1 = eng.train_step(idx, tgt).item()
    N.check_errors()
    assert math.isfinite(l0) and abs(l0 - math.log(cfg.vocab_size)) < 0.5
    assert l1 < l0


def test_graph_replay_matches_eager_steps():
    """The trainer's CUDA-graph step (captured on its second step, replayed
    after) runs the eager step's kernels in the same order: losses and the
    final weights are bit-identical."""
    from gpt2_harness_b200.config import TrainConfig
    from gpt2_harness_b200.trainer import Trainer

    cfg = small_config(n_layer=2)
    tc = TrainConfig(lr=1e-3, warmup_steps=0)
    runs = []
    for graph in (False, True):
        tr = Trainer(cfg, 2, 128, train=tc, schedule=False, seed=3, graph=graph)
        losses = []
        for step in range(5):
            idx, tgt = make_batch(cfg, 2, 128, seed=step)
            losses.append(tr.step(idx.pin_memory(), tgt.pin_memory()))
        tr.check()
        runs.append((losses, tr.engine.master.clone()))
    assert runs[0][0] == runs[1][0], runs
    assert torch.equal(runs[0][1], runs[1][1])
    assert tr.graph_launches > 0
