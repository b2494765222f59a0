"""Data parallel on CPU/gloo ranks vs the single-process oracle, plus the
launcher and the byte counter. Mirrors the reference's tests/test_parallel.py
DDP section (tolerance 1e-5, exact payload bytes)."""

import pytest
import torch

from gpt2_harness_b200.hardware import Capabilities, HardwareError
from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.data_parallel import build_buckets, ddp_equivalence_worker, local_shard

TOL = 1e-5
_CACHE = {}


def run(fn, world, **kw):
    key = (fn.__module__, fn.__name__, world, tuple(sorted(kw.items())))
    if key not in _CACHE:
        _CACHE[key] = comms.spawn_workers(fn, world, kw, backend="gloo", timeout=300)
    return _CACHE[key]


def test_workers_report_backend_and_device():
    for r in run(ddp_equivalence_worker, 2, batch=8, seq=16, steps=3):
        assert r.backend == "gloo" and r.device == "cpu"


def test_impossible_placement_fails_in_parent():
    with pytest.raises(HardwareError, match="exceeds the 2 visible"):
        comms.spawn_workers(ddp_equivalence_worker, 8, {}, backend="nccl",
                            caps=Capabilities.stub(device_count=2))


def test_nccl_request_without_cuda_is_refused():
    caps = Capabilities.stub(device_count=0)
    with pytest.raises(HardwareError):
        comms.spawn_workers(ddp_equivalence_worker, 2, {}, backend="nccl", caps=caps)


def test_counter_exact_payload_and_ring_model():
    c = comms.CommCounter(world_size=4)
    c.record("all_reduce", torch.zeros(1000))
    c.record("all_gather", [torch.zeros(250) for _ in range(4)])
    assert c.records["all_reduce"].payload_bytes == 4000
    assert c.records["all_gather"].payload_bytes == 4000
    assert c.records["all_reduce"].wire_bytes == pytest.approx(2 * 0.75 * 4000)
    assert c.records["all_gather"].wire_bytes == pytest.approx(0.75 * 4000)
    s = c.summary()
    assert s["total_calls"] == 2 and s["total_payload_bytes"] == 8000


def test_local_shard_refuses_uneven():
    with pytest.raises(ValueError):
        local_shard(torch.zeros(7, 3), 0, 2)


def test_buckets_are_reverse_order_and_capped():
    ps = [torch.nn.Parameter(torch.zeros(n)) for n in (10, 20, 30, 40)]
    b = build_buckets(ps, bucket_bytes=200)
    assert [len(x) for x in b] == [1, 2, 1]  # 160 | 120+80 | 40 bytes
    assert b[0][0] is ps[-1]


def test_ddp_gradient_equals_full_batch():
    for r in run(ddp_equivalence_worker, 2, batch=8, seq=16, steps=3):
        assert r.value["max_grad_error"] < TOL
        assert r.value["max_param_error"] < TOL


def test_ddp_moves_one_gradient_per_step():
    res = run(ddp_equivalence_worker, 2, batch=8, seq=16, steps=3)
    pay, n = res[0].payload, res[0].value["n_params"]
    assert pay["payload_bytes_per_step"] == n * 4
    # toy model closed form quoted by the reference: 4N = 228,096 B
    assert n * 4 == 228_096


def test_ddp_unbucketed_same_answer():
    res = run(ddp_equivalence_worker, 2, batch=8, seq=16, steps=2, bucket_bytes=0)
    assert res[0].value["max_grad_error"] < TOL
    assert res[0].payload["per_collective"]["all_reduce"]["calls"] > 2


def test_bf16_wire_halves_bytes_with_bounded_error():
    fp32 = run(ddp_equivalence_worker, 2, batch=8, seq=16, steps=3)[0]
    bf16 = run(ddp_equivalence_worker, 2, batch=8, seq=16, steps=3, reduce_dtype="bf16")[0]
    assert bf16.payload["payload_bytes_per_step"] * 2 == fp32.payload["payload_bytes_per_step"]
    assert (bf16.payload["per_collective"]["all_reduce"]["calls"]
            == fp32.payload["per_collective"]["all_reduce"]["calls"])
    assert TOL < bf16.value["max_grad_error"] < 1e-2


def test_ddp_adamw_tiny_baseline_config():
    """L8, C128, H4, ctx64, V50257, per-rank 4x64, AdamW 3e-4."""
    kw = dict(batch=8, seq=64, steps=2, optimizer="adamw", lr=3e-4,
              config_kwargs=(("n_layer", 8), ("n_head", 4), ("n_embd", 128), ("n_positions", 64),
                             ("vocab_size", 50257)))
    res = run(_tiny_worker, 2, **kw)
    for r in res:
        assert r.value["max_grad_error"] < TOL
        assert r.value["max_param_error"] < TOL
    assert res[0].payload["payload_bytes_per_step"] == 4 * 8_027_520  # 32,110,080 B


def _tiny_worker(rank, world, config_kwargs=(), **kw):
    return ddp_equivalence_worker(rank, world, config_kwargs=dict(config_kwargs), **kw)
