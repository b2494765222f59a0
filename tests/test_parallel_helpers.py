"""Shared parallel helpers on CPU/gloo: determinism helpers, storage-deduped
byte accounting, the N-D mesh, the DTensor formulation of the tensor-parallel
MLP, and the torch.profiler wrapper."""

import pytest
import torch

from gpt2_harness_b200.parallel.comms import spawn_workers
from gpt2_harness_b200.parallel.common import (identical_batch, identical_block, identical_model,
                                               max_rss_bytes, parallel_config, state_bytes)
from gpt2_harness_b200.parallel.mesh import mesh_coords


def test_parallel_config_is_the_reference_toy():
    cfg = parallel_config()
    assert (cfg.vocab_size, cfg.n_positions, cfg.n_layer, cfg.n_head, cfg.n_embd, cfg.dropout) == \
        (128, 64, 4, 4, 32, 0.0)
    assert parallel_config(n_layer=8).n_layer == 8


def test_identical_builders_do_not_touch_the_global_rng():
    cfg = parallel_config()
    torch.manual_seed(123)
    before = torch.rand(1)
    torch.manual_seed(123)
    a = identical_model(cfg, seed=4)
    after = torch.rand(1)
    assert torch.equal(before, after)
    b = identical_model(cfg, seed=4)
    assert all(torch.equal(p, q) for p, q in zip(a.parameters(), b.parameters()))
    c = identical_model(cfg, seed=5)
    assert not torch.equal(a.wte.weight, c.wte.weight)
    blk1, blk2 = identical_block(cfg, 1), identical_block(cfg, 1)
    assert all(torch.equal(p, q) for p, q in zip(blk1.parameters(), blk2.parameters()))
    x1, y1 = identical_batch(cfg, 2, 8, seed=9)
    x2, y2 = identical_batch(cfg, 2, 8, seed=9)
    assert torch.equal(x1, x2) and torch.equal(y1, y2) and torch.equal(x1[:, 1:], y1[:, :-1])


def test_state_bytes_counts_storages_once():
    cfg = parallel_config()
    m = identical_model(cfg)
    tied = m.wte.weight.numel() * 4
    params = sum(p.numel() * 4 for p in m.parameters())  # tied once in parameters()
    buffers = sum(b.numel() * b.element_size() for b in m.buffers())
    assert state_bytes(m) == params + buffers
    t = torch.zeros(10)
    assert state_bytes([t, t[:5], t.view(2, 5), None]) == 40
    assert state_bytes(m.wte.weight) == tied
    assert max_rss_bytes() > 0


def test_mesh_coords_row_major():
    shape = {"pp": 4, "cp": 2}
    coords = [mesh_coords(r, shape) for r in range(8)]
    assert coords[0] == {"pp": 0, "cp": 0} and coords[1] == {"pp": 0, "cp": 1}
    assert coords[7] == {"pp": 3, "cp": 1}
    assert mesh_coords(5, {"dp": 2, "tp": 2, "x": 2}) == {"dp": 1, "tp": 0, "x": 1}


def _mesh_worker(rank, world):
    import torch.distributed as dist

    from gpt2_harness_b200.parallel.mesh import Mesh

    m = Mesh({"dp": 2, "tp": 2})
    t = torch.tensor([float(rank)])
    dist.all_reduce(t, group=m.group("tp"))
    return {"coords": m.coords, "tp": m.group_ranks["tp"], "dp": m.group_ranks["dp"], "tp_sum": float(t),
            "next_tp": m.neighbor("tp", 1), "prev_dp": m.neighbor("dp", -1)}


def test_mesh_groups_over_gloo():
    res = {r.rank: r.value for r in spawn_workers(_mesh_worker, 4, backend="gloo", timeout=120)}
    for rank, v in res.items():
        d, t = divmod(rank, 2)
        assert v["coords"] == {"dp": d, "tp": t}
        assert v["tp"] == [2 * d, 2 * d + 1] and v["dp"] == [t, 2 + t]
        assert v["tp_sum"] == float(4 * d + 1)
        assert v["next_tp"] == (rank + 1 if t == 0 else None)
        assert v["prev_dp"] == (rank - 2 if d == 1 else None)


def _dtensor_entry(rank, world):
    from gpt2_harness_b200.parallel.dtensor_demo import dtensor_worker

    return dtensor_worker(rank, world)


def test_dtensor_tp_mlp_matches_manual_and_single_process():
    res = [r.value for r in spawn_workers(_dtensor_entry, 2, backend="gloo", timeout=180)]
    for r in res:
        scale = r["output_scale"]
        assert r["dtensor_error"] < 1e-5 * max(scale, 1.0)
        assert r["parallelize_module_error"] < 1e-5 * max(scale, 1.0)
        assert r["manual_error"] < 1e-5 * max(scale, 1.0)
        assert r["manual_vs_dtensor"] < 1e-5 * max(scale, 1.0)
        assert r["local_fc_weight_shape"] == [64, 32] and r["local_proj_weight_shape"] == [32, 64]


def test_profiler_wrapper_on_cpu():
    from gpt2_harness_b200.perf.profiling import categorize_op, profile_training_step

    m = identical_model(parallel_config())
    x, y = identical_batch(parallel_config(), 2, 16)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)

    def step():
        loss = m(x, y)["loss"]
        opt.zero_grad()
        loss.backward()
        opt.step()

    rep = profile_training_step(step, wait=0, warmup=1, active=2)
    assert rep.steps == 2 and rep.total_device_us > 0 and rep.top
    assert sum(rep.categories.values()) == pytest.approx(1.0)
    assert "ms" in rep.format(5)
    assert 0.0 <= rep.memory_bound_fraction() <= 1.0
    assert categorize_op("aten::mm") != categorize_op("aten::native_layer_norm")
