"""Per-strategy roofline arithmetic (CPU)."""

import pytest

from gpt2_harness_b200.config import gpt2_config
from gpt2_harness_b200.perf.mfu import param_count
from gpt2_harness_b200.perf.path_roofline import LINK_GBS, nvlink_bytes, path_roofline, table


def test_ddp_bytes_are_the_allreduce_lower_bound():
    cfg = gpt2_config("gpt2")
    n = param_count(cfg)
    assert nvlink_bytes("ddp", cfg, 16, 1024, 1) == 0.0
    for p in (2, 4, 8):
        assert nvlink_bytes("ddp", cfg, 16, 1024, p) == pytest.approx(2 * (p - 1) / p * 4 * n)
        # ZeRO-2 moves the fp32 reduce-scatter plus the bf16 all-gather
        assert nvlink_bytes("zero2", cfg, 16, 1024, p) == pytest.approx((p - 1) / p * 6 * n)


def test_tp_bytes_eight_collectives_per_block():
    cfg = gpt2_config("gpt2-xl")
    got = nvlink_bytes("tp", cfg, 32, 1024, 8)
    assert got == pytest.approx(8 * 48 * 7 / 8 * 2 * 32 * 1024 * 1600)


def test_cp_and_pp_bytes():
    cfg = gpt2_config("gpt2-large", n_positions=16384)
    n = param_count(cfg)
    chunk = 1 * 16384 / 4 * 2 * 1280 * 2
    assert nvlink_bytes("cp", cfg, 1, 16384, 2) == pytest.approx(36 * 2 * 2 * chunk + 4 * n)
    # two stages: each boundary direction carries m fp32 activations
    assert nvlink_bytes("pp", cfg, 1, 16384, 2, pp=2, cp=1, micro_batches=8) == pytest.approx(
        8 * 16384 * 1280 * 4)
    with pytest.raises(ValueError):
        nvlink_bytes("pp", cfg, 1, 16384, 4, pp=2, cp=1, micro_batches=8)


def test_fraction_and_bound():
    cfg = gpt2_config("gpt2-xl")
    r = path_roofline("tp", cfg, 32, 1024, 8, 200.0, peak_tflops=1000.0)
    assert r.bound == "NVLink"
    assert r.t_comm_ms == pytest.approx(nvlink_bytes("tp", cfg, 32, 1024, 8) / (LINK_GBS * 1e9) * 1e3, rel=1e-3)
    assert r.fraction == pytest.approx(r.t_roof_ms / 200.0, rel=1e-3)
    r1 = path_roofline("ddp", gpt2_config("gpt2"), 16, 1024, 1, 20.0, peak_tflops=1000.0)
    assert r1.bound == "compute" and r1.t_comm_ms == 0.0
    with pytest.raises(ValueError):
        path_roofline("ulysses", cfg, 1, 1024, 2, 1.0)


def test_measured_table_is_well_formed():
    rows = table()
    assert rows and all(0 < r["fraction"] <= 1.5 for r in rows)
