"""Tensor-parallel layout planning (CPU): uneven head partition, the
replicated region and wte shard at identical offsets on every rank, and
shard slicing that reassembles the full tensors exactly."""

import math

import pytest
import torch

from gpt2_harness_b200.config import gpt2_config
from gpt2_harness_b200.models.engine import ParamLayout
from gpt2_harness_b200.parallel.tensor_parallel import padded_vocab
from gpt2_harness_b200.parallel.tp_native import D, TPLayout, head_partition


def test_head_partition_uneven():
    assert head_partition(25, 8) == [(0, 4), (4, 7), (7, 10), (10, 13), (13, 16), (16, 19),
                                     (19, 22), (22, 25)]
    assert head_partition(12, 4) == [(0, 3), (3, 6), (6, 9), (9, 12)]
    assert head_partition(3, 2) == [(0, 2), (2, 3)]


@pytest.mark.parametrize("p", [1, 2, 4, 8])
def test_padded_vocab_is_50304(p):
    vp = padded_vocab(50257, p)
    assert vp == 50304 and vp % p == 0 and (vp // p) % 16 == 0


@pytest.mark.parametrize("world", [2, 8])
def test_shared_offsets_on_every_rank(world):
    cfg = gpt2_config("gpt2-xl", n_layer=2)
    lays = [TPLayout(cfg, r, world) for r in range(world)]
    assert len({l.repl_hi for l in lays}) == 1
    assert len({l.specs["wte.weight"][0] for l in lays}) == 1
    assert sum(l.Hl for l in lays) == cfg.n_head
    for l in lays:
        for off, shape, _ in l.specs.values():
            assert off % 64 == 0


def _reassemble(lays, pieces, name, cfg):
    if name == "wte.weight":
        return torch.cat(pieces, 0)[:cfg.vocab_size]
    if name.endswith("c_attn.weight") or name.endswith("c_attn.bias"):
        secs = [[pc[s * l.Hl * D:(s + 1) * l.Hl * D] for l, pc in zip(lays, pieces)] for s in range(3)]
        return torch.cat([torch.cat(x, 0) for x in secs], 0)
    if name.endswith("attn.c_proj.weight") or name.endswith("mlp.c_proj.weight"):
        return torch.cat(pieces, 1)
    if name.endswith("mlp.c_fc.weight") or name.endswith("mlp.c_fc.bias"):
        return torch.cat(pieces, 0)
    return pieces[0]


@pytest.mark.parametrize("world,heads", [(2, 3), (4, 6), (3, 12)])
def test_shards_reassemble_exactly(world, heads):
    cfg = gpt2_config("gpt2", n_layer=1, n_embd=heads * 64, n_head=heads, n_positions=64,
                      vocab_size=1000)
    full_layout = ParamLayout(cfg)
    g = torch.Generator().manual_seed(0)
    full = {s.name: torch.randn(s.shape, generator=g) for s in full_layout.specs}
    lays = [TPLayout(cfg, r, world) for r in range(world)]
    for name in lays[0].specs:
        pieces = [l.shard_of(name, full[name]) for l in lays]
        for l, pc in zip(lays, pieces):
            assert tuple(pc.shape) == l.specs[name][1]
        assert torch.equal(_reassemble(lays, pieces, name, cfg), full[name]), name
    # every parameter element is counted once across the sharded tensors
    sharded = sum(math.prod(l.specs[n][1]) for l in lays for n in l.specs if l.specs[n][0] >= l.repl_hi)
    repl = sum(math.prod(lays[0].specs[n][1]) for n in lays[0].specs if lays[0].specs[n][0] < lays[0].repl_hi)
    padded_rows = padded_vocab(cfg.vocab_size, world) - cfg.vocab_size
    assert sharded + repl == full_layout.num_parameters + padded_rows * cfg.n_embd
