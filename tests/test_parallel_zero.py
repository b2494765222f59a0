"""ZeRO-1/2/3 on CPU/gloo ranks vs single-process torch AdamW.

Reference tolerance 1e-5 and its exact per-rank payloads at the toy size
(vocab 128, ctx 64, L4, C32; p=2): ZeRO-1 and ZeRO-2 456,192 B/step,
ZeRO-3 634,624 B/step, clipping adds 0 B (ZeRO-1) / 4 B (ZeRO-2)."""

import pytest
import torch

from gpt2_harness_b200.parallel import comms
from gpt2_harness_b200.parallel.zero import (adamw_update_, clip_coefficient, padded_numel,
                                             zero3_equivalence_worker, zero3_payload_bytes,
                                             zero_equivalence_worker)

TOL = 1e-5
_CACHE = {}


def run(fn, world, **kw):
    key = (fn.__name__, world, tuple(sorted(kw.items())))
    if key not in _CACHE:
        _CACHE[key] = comms.spawn_workers(fn, world, kw, backend="gloo", timeout=300)
    return _CACHE[key]


def test_adamw_update_matches_torch_bitwise_at_p1():
    torch.manual_seed(0)
    p = torch.randn(1000)
    ref = torch.nn.Parameter(p.clone())
    opt = torch.optim.AdamW([ref], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                            foreach=False)
    mine, m, v = p.clone(), torch.zeros(1000), torch.zeros(1000)
    for step in range(1, 4):
        g = torch.randn(1000)
        ref.grad = g.clone()
        opt.step()
        adamw_update_(mine, g, m, v, step, 1e-3, 0.9, 0.95, 1e-8, 0.1)
    assert torch.equal(mine, ref.detach())


def test_clip_coefficient_matches_torch():
    t = torch.tensor(3.0)
    assert float(clip_coefficient(t, 1.0)) == pytest.approx(1.0 / (3.0 + 1e-6))
    assert float(clip_coefficient(torch.tensor(0.5), 1.0)) == 1.0


@pytest.mark.parametrize("stage", [1, 2])
def test_zero12_trajectory_matches_adamw(stage):
    for r in run(zero_equivalence_worker, 2, stage=stage):
        assert r.value["max_param_error"] < TOL


@pytest.mark.parametrize("stage", [1, 2])
def test_zero12_payload_closed_form(stage):
    res = run(zero_equivalence_worker, 2, stage=stage)
    v, pay = res[0].value, res[0].payload
    n, npad = v["n_params"], v["padded_numel"]
    if stage == 1:
        assert pay["per_collective"]["all_reduce"]["payload_bytes"] / 4 == 4 * npad  # 4 steps
    else:
        assert pay["per_collective"]["reduce_scatter"]["payload_bytes"] / 4 == 4 * npad
    assert pay["per_collective"]["all_gather"]["payload_bytes"] / 4 == 4 * npad
    assert pay["payload_bytes_per_step"] == 456_192
    assert npad == padded_numel(n, 2)


def test_zero_sharded_clip_overhead():
    z1 = run(zero_equivalence_worker, 2, stage=1, grad_clip=0.05)[0]
    z2 = run(zero_equivalence_worker, 2, stage=2, grad_clip=0.05)[0]
    assert z1.value["max_param_error"] < TOL and z2.value["max_param_error"] < TOL
    assert z1.value["max_grad_norm_error"] < 1e-5 and z2.value["max_grad_norm_error"] < 1e-5
    assert z1.payload["payload_bytes_per_step"] == 456_192          # no extra collective
    assert z2.payload["payload_bytes_per_step"] == 456_192 + 4      # one fp32 scalar


def test_zero_state_is_sharded():
    v = run(zero_equivalence_worker, 2, stage=2)[0].value
    assert v["sharded_bytes"]["optimizer"] * 2 == pytest.approx(v["replicated_bytes"]["optimizer"], rel=0.01)


def test_zero3_trajectory_and_payload():
    res = run(zero3_equivalence_worker, 2)
    for r in res:
        assert r.value["max_param_error"] < TOL
    v, pay = res[0].value, res[0].payload
    assert pay["payload_bytes_per_step"] == v["closed_form_payload_bytes"] == 634_624
    steps = pay["steps"]
    assert pay["per_collective"]["all_gather"]["calls"] == 2 * 4 * steps   # 2 per unit per step
    assert pay["per_collective"]["reduce_scatter"]["calls"] == 4 * steps   # 1 per unit per step


def test_zero3_closed_form_at_gpt2_medium_p8():
    """The BASELINE ZeRO-3 config: 24 units of 12,596,224 params + 52,513,792 root."""
    assert zero3_payload_bytes([12_596_224] * 24, 52_513_792, 8) == 3_837_767_680
    assert zero3_payload_bytes([12_596_224] * 24, 52_513_792, 8, 2, 2, 2) == 1_918_883_840


# -------------------------------------------- reduced-precision wires and clipping --
def test_bf16_gradient_reduction_error_is_fresh_each_step_and_bounded():
    fp = run(zero_equivalence_worker, 2, stage=2)[0].value
    bf = run(zero_equivalence_worker, 2, stage=2, reduce_dtype="bf16")[0].value
    # a bf16 reduce-scatter costs accuracy, but the fp32 master keeps it from
    # compounding: every step's error stays within a small multiple of the first
    assert bf["max_param_error"] > fp["max_param_error"]
    errs = bf["param_errors"]
    assert max(errs) < 1e-2 and max(errs) < 8 * max(errs[0], 1e-12)


def test_bf16_parameter_gather_keeps_an_fp32_master_shard():
    v = run(zero_equivalence_worker, 2, stage=2, param_dtype="bf16")[0].value
    assert v["param_dtype"] == "bf16"
    # the error of the gathered bf16 parameters saturates at bf16's resolution
    # of the parameter scale, it does not grow step by step
    assert v["max_param_error"] <= v["reference_param_scale"] * 2 ** -7
    assert v["sharded_bytes"]["params"] > 0


@pytest.mark.parametrize("stage", [1, 2])
def test_sharded_clip_reproduces_single_process_clip_and_bites(stage):
    v = run(zero_equivalence_worker, 2, stage=stage, grad_clip=0.05)[0].value
    assert v["max_grad_norm_error"] < 1e-5
    assert any(n["reference"] > 0.05 for n in v["grad_norms"])  # the clip was active


def test_zero3_clips_shards_and_roots_consistently():
    res = run(zero3_equivalence_worker, 2, grad_clip=0.05)
    for r in res:
        assert r.value["max_param_error"] < TOL
