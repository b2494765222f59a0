"""Context parallelism (all-gather KV and differentiable ring attention) on
CPU/gloo ranks vs full-sequence attention; exact payloads."""

import pytest

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.sequence_parallel import sequence_parallel_worker

TOL = 1e-5
_CACHE = {}


def run(fn, world, **kw):
    key = (fn.__name__, world, tuple(sorted(kw.items())))
    if key not in _CACHE:
        _CACHE[key] = comms.spawn_workers(fn, world, kw, backend="gloo", timeout=300)
    return _CACHE[key]


@pytest.mark.parametrize("path", ["all_gather", "ring"])
@pytest.mark.parametrize("world", [2, 4])
def test_cp_forward_and_backward(path, world):
    for r in run(sequence_parallel_worker, world, batch=2, seq=32, path=path):
        v = r.value
        assert v["forward_error"] < TOL
        assert v["input_grad_error"] < TOL
        assert v["weight_grad_error"] < TOL * max(1.0, v["weight_grad_scale"])


def test_all_gather_kv_payload():
    res = run(sequence_parallel_worker, 2, batch=2, seq=32, path="all_gather")
    pc = res[0].payload["per_collective"]
    cf = res[0].value["closed_form"]
    assert pc["all_gather"]["payload_bytes"] == cf["all_gather_kv_forward"] == 2 * 4 * 2 * 32 * 32
    assert pc["reduce_scatter"]["payload_bytes"] == cf["all_gather_kv_backward_reduce_scatter"]


def test_ring_forward_sends_two_per_hop():
    res = run(sequence_parallel_worker, 4, batch=2, seq=32, path="ring")
    pc = res[0].payload["per_collective"]
    # forward: 2(p-1) sends; backward: 4(p-1) + 2 (dK/dV return hop)
    assert pc["send"]["calls"] == 2 * 3 + 4 * 3 + 2
    fwd_bytes = res[0].value["closed_form"]["ring_forward_send"]
    assert fwd_bytes == pytest.approx(2 * 3 / 4 * 4 * 2 * 32 * 32)
