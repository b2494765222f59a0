"""Stage layout of the native pipeline engine (CPU): the stages partition the
blocks, stage 0 owns the embeddings, the last stage ln_f and an untied
lm_head, and the decay table covers exactly the matrices and embeddings."""

import math

import pytest

from gpt2_harness_b200.config import gpt2_config
from gpt2_harness_b200.models.engine import ParamLayout
from gpt2_harness_b200.parallel.pp_native import StageLayout


@pytest.mark.parametrize("p", [1, 2, 4])
def test_stage_layouts_partition_the_model(p):
    cfg = gpt2_config("gpt2")
    full = ParamLayout(cfg)
    seen = {}
    for s in range(p):
        lay = StageLayout(cfg, s, p)
        assert lay.first == (s == 0) and lay.last == (s == p - 1)
        assert (lay.l0, lay.l1) == (s * cfg.n_layer // p, (s + 1) * cfg.n_layer // p)
        for name, (off, shape, decay) in lay.specs.items():
            assert name not in seen
            seen[name] = (shape, decay)
            assert off % 64 == 0
        # decay ranges: sorted, disjoint, and the union is the decayed tensors
        r = lay.decay_ranges()
        assert r == sorted(r)
        covered = sum(hi - lo for lo, hi in zip(r[::2], r[1::2]))
        want = sum(-(-math.prod(sh) // 64) * 64 for (_, sh, d) in lay.specs.values() if d)
        assert covered == want
    names = {sp.name for sp in full.specs} | {"lm_head.weight"}
    assert set(seen) == names
    assert seen["lm_head.weight"] == ((cfg.vocab_size, cfg.n_embd), True)


def test_uneven_split_rejected():
    with pytest.raises(ValueError):
        StageLayout(gpt2_config("gpt2"), 0, 5)


def _mesh_worker(rank, world, pp, cp):
    import torch
    import torch.distributed as dist

    from gpt2_harness_b200.parallel.pp_native import make_mesh

    mesh = make_mesh(pp, cp)
    out = {"stage": mesh.stage, "c": mesh.cp_rank,
           "pp_ranks": dist.get_process_group_ranks(mesh.pp_group),
           "fwd_ranks": dist.get_process_group_ranks(mesh.fwd_group),
           "cp_ranks": dist.get_process_group_ranks(mesh.cp_group) if mesh.cp_group is not None else None}
    # the pp group carries a real collective among the same-slice ranks
    t = torch.tensor([float(rank)])
    dist.all_reduce(t, group=mesh.pp_group)
    out["pp_sum"] = float(t)
    return out


def test_mesh_groups_gloo():
    from gpt2_harness_b200.parallel.comms import spawn_workers

    res = spawn_workers(_mesh_worker, 4, {"pp": 2, "cp": 2}, backend="gloo", timeout=120)
    by = {r.rank: r.value for r in res}
    for rank, v in by.items():
        s, c = divmod(rank, 2)
        assert (v["stage"], v["c"]) == (s, c)
        assert v["pp_ranks"] == v["fwd_ranks"] == [c, 2 + c]
        assert v["cp_ranks"] == [2 * s, 2 * s + 1]
        assert v["pp_sum"] == float(c + 2 + c)
