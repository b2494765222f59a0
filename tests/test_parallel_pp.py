"""Pipeline parallel (GPipe, 1F1B) on CPU/gloo ranks vs the full-batch model;
schedule simulator vs the bubble formula; 1F1B stash bound; payload."""

import pytest

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.pipeline_parallel import (analytic_bubble, bubble_scan_worker,
                                                          pipeline_payload_bytes, pipeline_worker,
                                                          schedule_order, simulate)

TOL = 1e-5
_CACHE = {}


def run(fn, world, **kw):
    key = (fn.__name__, world, tuple(sorted(kw.items())))
    if key not in _CACHE:
        _CACHE[key] = comms.spawn_workers(fn, world, kw, backend="gloo", timeout=300)
    return _CACHE[key]


@pytest.mark.parametrize("kind", ["gpipe", "1f1b"])
def test_pipeline_gradients_match_full_batch(kind):
    for r in run(pipeline_worker, 4, micro_batches=4, batch=8, seq=16, kind=kind):
        assert r.value["max_grad_error"] < TOL
        assert r.value["compared_tensors"] > 0


def test_pipeline_send_bytes_closed_form():
    res = run(pipeline_worker, 4, micro_batches=4, batch=8, seq=16, kind="1f1b")
    first = res[0]
    assert first.payload["per_collective"]["send"]["payload_bytes"] == first.value["closed_form_send_bytes"]
    assert first.value["closed_form_send_bytes"] == pipeline_payload_bytes(4, 2, 16, 32) == 16_384
    mid = res[1]  # sends activations forward and gradients backward
    assert mid.payload["per_collective"]["send"]["payload_bytes"] == 2 * 16_384


@pytest.mark.parametrize("p,m", [(2, 1), (4, 1), (4, 4), (4, 8), (8, 16)])
@pytest.mark.parametrize("kind", ["gpipe", "1f1b"])
def test_simulator_equals_formula(p, m, kind):
    sim = simulate(p, m, 1.0, 2.0, kind)
    assert sim.bubble == pytest.approx(analytic_bubble(p, m), abs=1e-12)


def test_1f1b_stash_bounded_by_stages():
    assert simulate(4, 8, 1.0, 2.0, "1f1b").peak_stash == 4
    assert simulate(4, 8, 1.0, 2.0, "gpipe").peak_stash == 8


def test_schedule_orders():
    assert schedule_order(0, 4, 4, "gpipe")[:4] == [("F", i) for i in range(4)]
    o = schedule_order(3, 4, 4, "1f1b")
    assert o[:2] == [("F", 0), ("B", 0)]
    with pytest.raises(ValueError):
        schedule_order(0, 2, 2, "zigzag")


@pytest.mark.slow
def test_bubble_scan_orders_with_micro_batches():
    res = run(bubble_scan_worker, 2, micro_batch_counts=(1, 4), batch=8, seq=16, repeats=1)
    rows = res[0].value["rows"]
    assert {r["kind"] for r in rows} == {"gpipe", "1f1b"}
    assert all(r["analytic_bubble"] == pytest.approx(analytic_bubble(2, r["micro_batches"])) for r in rows)


def test_pipeline_stages_partition_the_model():
    import torch

    from gpt2_harness_b200.parallel.common import identical_model, parallel_config
    from gpt2_harness_b200.parallel.pipeline_parallel import PipelineStage

    cfg = parallel_config()
    full = identical_model(cfg)
    total = sum(p.numel() for p in full.parameters())
    counts = []
    for s in range(4):
        stage = PipelineStage(identical_model(cfg), s, 4)
        counts.append(sum(p.numel() for p in stage.parameters()))
        assert len(stage.blocks) == 1 and stage.is_first == (s == 0) and stage.is_last == (s == 3)
    # the tied table is held twice once the head is split off onto the last stage
    assert sum(counts) == total + cfg.vocab_size * cfg.n_embd
    with pytest.raises(ValueError):
        PipelineStage(identical_model(cfg), 0, 3)
    x = torch.randint(0, cfg.vocab_size, (2, 8))
    s0 = PipelineStage(identical_model(cfg), 0, 1)
    assert torch.allclose(s0(x), identical_model(cfg)(x)["logits"])
