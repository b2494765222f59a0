"""Sharded checkpoint format, resharding across world sizes, and the async
checkpointer (reference tests/test_cluster.py checkpoint section)."""

import json

import pytest
import torch

from gpt2_harness_b200.cluster.checkpoint import (FORMAT, REPLICATE, AsyncCheckpointer, CheckpointIndex,
                                                  ShardSpec, gpt2_tp_plan, load_extra, load_full,
                                                  load_reshard, merge_pieces, pad_vocab_rows, save_sharded,
                                                  shard_path, shard_state_dict, split_tensor)
from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.models.gpt import GPT


def tiny_gpt(vocab=128):
    torch.manual_seed(0)
    return GPT(GPTConfig(vocab_size=vocab, n_positions=32, n_layer=2, n_head=4, n_embd=32))


def save_layout(tmp_path, model, world, vocab_pad=None, step=7):
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    if vocab_pad:
        for k in ("wte.weight", "lm_head.weight"):
            sd[k] = pad_vocab_rows(sd[k], vocab_pad)
    plan = gpt2_tp_plan(sd)
    shapes = {k: list(v.shape) for k, v in sd.items()}
    for r in range(world):
        save_sharded(tmp_path, shard_state_dict(sd, plan, r, world), plan, rank=r, world_size=world, step=step,
                     global_shapes=shapes, extra={"rank": r, "pos": 10 * r})
    return sd, plan


def test_split_merge_identity():
    t = torch.arange(24.0).view(6, 4)
    for spec in (ShardSpec("shard", 0), ShardSpec("shard", 1), ShardSpec("shard", 0, sections=3), REPLICATE):
        world = 2
        assert torch.equal(merge_pieces(split_tensor(t, spec, world), spec), t)


def test_qkv_sections_give_whole_heads():
    t = torch.arange(12.0).view(12, 1)  # q rows 0-3, k 4-7, v 8-11
    pieces = split_tensor(t, ShardSpec("shard", 0, sections=3), 2)
    assert pieces[0].flatten().tolist() == [0, 1, 4, 5, 8, 9]
    assert pieces[1].flatten().tolist() == [2, 3, 6, 7, 10, 11]


def test_uneven_split_refused_and_padding_fixes_it():
    with pytest.raises(ValueError):
        split_tensor(torch.zeros(50257, 4), ShardSpec("shard", 0), 4)
    padded = pad_vocab_rows(torch.zeros(50257, 4), 50304)
    assert [p.shape[0] for p in split_tensor(padded, ShardSpec("shard", 0), 8)] == [6288] * 8


@pytest.mark.parametrize("src,dst", [(4, 2), (4, 1), (2, 8), (4, 8), (8, 4), (1, 4)])
def test_reshard_exact(tmp_path, src, dst):
    model = tiny_gpt()
    sd, plan = save_layout(tmp_path, model, src)
    for r in range(dst):
        local, idx, files = load_reshard(tmp_path, rank=r, world_size=dst)
        want = shard_state_dict(sd, plan, r, dst)
        for k in want:
            assert torch.equal(local[k], want[k]), k
        assert idx.step == 7 and idx.world_size == src
        if dst >= src:
            assert files == 1  # each destination rank touches one source file
        else:
            assert files == src // dst


def test_full_reload_gives_same_logits(tmp_path):
    model = tiny_gpt()
    save_layout(tmp_path, model, 4)
    full, _ = load_full(tmp_path)
    fresh = GPT(model.config)
    fresh.load_state_dict(full)
    x = torch.randint(0, 128, (2, 16))
    assert torch.equal(fresh(x)["logits"], model(x)["logits"])


def test_index_self_describing(tmp_path):
    save_layout(tmp_path, tiny_gpt(), 2)
    d = json.loads((tmp_path / "index.json").read_text())
    assert d["format"] == FORMAT == "transformer-internals-sharded-v1"
    assert set(d) == {"format", "world_size", "step", "plan", "global_shapes", "meta"}
    assert shard_path(tmp_path, 1, 2).name == "shard_0001_of_0002.pt"
    assert CheckpointIndex.read(tmp_path).plan["h.0.attn.c_attn.weight"].sections == 3
    assert load_extra(tmp_path, 1)["pos"] == 10


def test_padded_vocab_layout_reshards(tmp_path):
    torch.manual_seed(1)
    model = GPT(GPTConfig(vocab_size=50257, n_positions=16, n_layer=1, n_head=2, n_embd=16))
    sd, plan = save_layout(tmp_path, model, 8, vocab_pad=50304)
    local, _, _ = load_reshard(tmp_path, rank=3, world_size=4)
    assert local["wte.weight"].shape == (50304 // 4, 16)


def test_async_checkpointer_matches_sync_and_surfaces_errors(tmp_path):
    model = tiny_gpt()
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    plan = {k: REPLICATE for k in sd}
    shapes = {k: list(v.shape) for k, v in sd.items()}
    ck = AsyncCheckpointer()
    ck.save(tmp_path / "a", sd, plan=plan, rank=0, world_size=1, step=3, global_shapes=shapes)
    ck.wait()
    full, idx = load_full(tmp_path / "a")
    assert idx.step == 3 and all(torch.equal(full[k], sd[k]) for k in sd)
    ck.save(tmp_path / "b", sd, plan=plan, rank=0, world_size=1, step=3, global_shapes=None)
    with pytest.raises(ValueError):
        ck.wait()


# ------------------------------------------------------ plan and shard math --
def test_plan_covers_every_parameter_and_shards_the_right_ones():
    sd = tiny_gpt().state_dict()
    plan = gpt2_tp_plan(sd)
    assert set(plan) == set(sd)
    for n, spec in plan.items():
        if n.endswith(("c_attn.weight", "c_attn.bias")):
            assert (spec.kind, spec.dim, spec.sections) == ("shard", 0, 3)
        elif n.endswith(("attn.c_proj.weight", "mlp.c_proj.weight")):
            assert (spec.kind, spec.dim) == ("shard", 1)
        elif n.endswith(("mlp.c_fc.weight", "mlp.c_fc.bias")) or n in ("wte.weight", "lm_head.weight"):
            assert (spec.kind, spec.dim) == ("shard", 0)
        else:
            assert spec.kind == "replicate", n
    assert gpt2_tp_plan(sd, vocab_parallel=False)["wte.weight"].kind == "replicate"


def test_column_and_row_parallel_shards_reproduce_the_full_matmul():
    torch.manual_seed(3)
    x = torch.randn(5, 32, dtype=torch.float64)
    w_fc = torch.randn(128, 32, dtype=torch.float64)
    w_pr = torch.randn(32, 128, dtype=torch.float64)
    full = (x @ w_fc.t()).relu() @ w_pr.t()
    for p in (1, 2, 4):
        cols = split_tensor(w_fc, ShardSpec("shard", dim=0), p)
        rows = split_tensor(w_pr, ShardSpec("shard", dim=1), p)
        # column shards give slices of the hidden layer; row shards' partial
        # products sum to the output
        out = sum((x @ c.t()).relu() @ r.t() for c, r in zip(cols, rows))
        assert torch.allclose(out, full)


def test_reshard_reads_only_the_shards_it_needs(tmp_path):
    m = tiny_gpt()
    _, plan = save_layout(tmp_path, m, 4)
    # 4 -> 4 same layout: each rank's shards sit in one file (replicated
    # tensors are read from that same file)
    _, _, files = load_reshard(tmp_path, rank=2, world_size=4)
    assert files == 1
    # 4 -> 2: rank 0 of 2 needs source ranks 0 and 1
    _, _, files = load_reshard(tmp_path, rank=0, world_size=2)
    assert files == 2
    # 4 -> 1: everything
    _, _, files = load_reshard(tmp_path, rank=0, world_size=1)
    assert files == 4


def test_reserved_port_stays_reserved_and_launch_replaces_a_taken_port():
    import socket
    from dataclasses import replace

    from gpt2_harness_b200.cluster.failure import JobSpec, _usable_port, port_is_free, reserved_port

    with reserved_port() as p:
        assert not port_is_free(p)
        spec = JobSpec(data_path="d", ckpt_dir="c", log_path="l", master_port=p)
        fixed = _usable_port(spec)
        assert fixed.master_port != p and fixed.master_port > 0
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        s.listen(1)
        taken = s.getsockname()[1]
        assert _usable_port(JobSpec(data_path="d", ckpt_dir="c", log_path="l", master_port=taken)).master_port != taken
    free = _usable_port(replace(spec, master_port=0))
    assert free.master_port > 0
