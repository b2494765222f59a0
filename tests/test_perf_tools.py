"""Roofline tables and the diagnosis on CPU (tiny shapes)."""

import pytest
import torch

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.perf.roofline import (MachinePeak, measure_machine_peak, op_costs, op_roofline_table,
                                             peak_from_file, roofline_payload)


def _peak():
    return MachinePeak("test", "bf16", 1e15, 5e12, 200.0)


def test_op_costs_closed_forms():
    cfg = GPTConfig()
    rows = {n: (f, b) for n, _, f, b in op_costs(cfg, 2, 64, 4, "eager")}
    B, T, C = 2, 64, 768
    assert rows["qkv projection (GEMM)"][0] == 2 * B * T * C * 3 * C
    assert rows["MLP down (GEMM)"][0] == 8 * B * T * C * C
    assert rows["softmax (+ causal mask)"][1] == 2 * B * 12 * T * T * 4
    eager_b = sum(b for *_, b in op_costs(cfg, 8, 1024, 2, "eager"))
    native_b = sum(b for *_, b in op_costs(cfg, 8, 1024, 2, "native"))
    assert native_b < 0.5 * eager_b  # fused attention never writes the score matrix
    with pytest.raises(ValueError):
        op_costs(cfg, 1, 1, 4, "mystery")


def test_roofline_classification_and_payload():
    peak = _peak()
    rows = op_roofline_table(peak, GPTConfig(), batch=8, seq=512)
    kinds = {r.name: r.bound for r in rows}
    assert kinds["MLP up 4x (GEMM)"] == "compute" and kinds["GELU (tanh)"] == "memory"
    assert all(r.roofline_seconds > 0 for r in rows)
    p = roofline_payload(peak, batch=8, seq=512)
    assert p["native_bytes_per_block"] < p["eager_bytes_per_block"]


def test_peaks_from_file_and_cpu_sweep():
    pk = peak_from_file()
    assert pk.peak_flops_per_s > 1e15 and pk.peak_bytes_per_s > 1e12 and pk.ridge_flops_per_byte > 100
    cpu = measure_machine_peak("cpu", gemm_sizes=(64, 128), stream_sizes_mib=(1, 2))
    assert cpu.peak_flops_per_s > 0 and cpu.attainable_flops_per_s(1e-3) < cpu.peak_flops_per_s


def test_diagnose_ranks_an_injected_loader_stall():
    from gpt2_harness_b200.perf.diagnose import diagnose, severity
    assert severity(0.5) == "critical" and severity(0.01) == "healthy"
    cfg = GPTConfig(vocab_size=128, n_positions=32, n_layer=1, n_head=2, n_embd=32)
    rep = diagnose(_peak(), cfg, batch=2, seq=32, loader_stall_s=0.05, steps=3, warmup=1, batch_sweep=(1, 2))
    top = rep.findings[0]
    assert top.name == "dataloader stall" and top.severity in ("critical", "significant")
    assert "ranked findings" in rep.text() and rep.to_dict()["throughput"]["tokens_per_s"] > 0
    healthy = diagnose(_peak(), cfg, batch=2, seq=32, steps=3, warmup=1, batch_sweep=None, profile_ops=False)
    assert healthy.findings[0].cost_fraction < top.cost_fraction


@pytest.mark.slow
def test_collective_probe_on_gloo_ranks():
    from gpt2_harness_b200.perf.diagnose import collective_probe
    out = collective_probe(world_size=2, steps=3, warmup=1, backend="gloo", timeout_s=300)
    for arm in ("manual_allreduce", "ddp_default_buckets", "ddp_small_buckets"):
        assert 0.0 <= out[arm]["overlap_fraction"] <= 1.0
        assert out[arm]["step_s"] > 0
    assert out["backend"] == "gloo" and out["grad_bytes"] > 0
