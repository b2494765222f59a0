"""Collective benchmark math and gloo sweep, fabric model, cgroup reader."""

import math

import pytest

from gpt2_harness_b200.cluster import cgroups, collbench, fabric


def test_bus_factors_and_fit():
    assert collbench.bus_factor("all_reduce", 8) == pytest.approx(1.75)
    assert collbench.bus_factor("all_gather", 4) == pytest.approx(0.75)
    assert collbench.bus_bandwidth("all_reduce", 1e9, 1.0, 1) == 0.0
    with pytest.raises(ValueError):
        collbench.bus_factor("broadcast", 2)
    xs = [1e3, 1e6, 1e7, 1e8]
    ys = [10e-6 + x / 100e9 for x in xs]  # 10 us + bytes / (100 GB/s raw)
    f = collbench.fit_link_model(xs, ys, 2, "all_reduce")
    assert f["latency_us"] == pytest.approx(10.0, rel=1e-6)
    assert f["bandwidth_gbytes_per_s"] == pytest.approx(100.0 * 1.0, rel=1e-6)  # factor 1 at n=2
    assert f["r_squared"] == pytest.approx(1.0)


@pytest.mark.slow
def test_collbench_gloo_sweep():
    res = collbench.run((2,), sizes=[1 << 12, 1 << 16, 1 << 20], repeats=2, warmup=1, backend="gloo", p2p=False)
    assert res["backend"] == "gloo" and len(res["results"]) == 9
    assert {f["op"] for f in res["fits"]} == set(collbench.OPS)
    assert all(r["median_s"] > 0 for r in res["results"])


def test_fabric_ring_times_and_measured_links():
    link = fabric.LINKS["nvlink5"]
    t2 = fabric.all_reduce_time(1e9, 2, link)
    t8 = fabric.all_reduce_time(1e9, 8, link)
    assert t8 > t2 and fabric.all_reduce_time(1e9, 1, link) == 0.0
    meas = fabric.LINKS["nvlink5_measured_ar"]
    assert meas.efficiency_applied and meas.measured
    # a measured link is not derated again
    assert fabric.p2p_time(725e9, meas) == pytest.approx(1.0 + meas.latency_us * 1e-6)
    fit = {"latency_us": 28.0, "bandwidth_gbytes_per_s": 700.0, "r_squared": 0.999}
    ml = fabric.link_from_measurement("x", fit, 8)
    assert ml.latency_us == pytest.approx(2.0)  # 28 us over 14 ring hops


def test_fabric_step_costs_and_crossover():
    cfg = fabric.ParallelConfig(tp=8)
    c = fabric.step_costs(fabric.GPT2_XL, cfg, "nvlink5")
    assert c["tp"] > 0 and c["ddp"] == 0.0 and c["pp"] == 0.0
    slow = fabric.step_costs(fabric.GPT2_XL, cfg, "roce200")["tp"]
    assert slow > 10 * c["tp"]
    assert fabric.crossover_ranks(fabric.LLAMA70B, "roce200") is not None
    nv = fabric.crossover_ranks(fabric.LLAMA70B, "nvlink5")
    ro = fabric.crossover_ranks(fabric.LLAMA70B, "roce200")
    assert nv is None or nv > ro
    assert "MODELLED" in fabric.format_report()


def test_cgroups_on_a_fake_tree(tmp_path):
    root = tmp_path / "cg"
    root.mkdir()
    (root / "cgroup.controllers").write_text("cpu memory pids")
    (root / "memory.max").write_text(str(8 << 30))
    (root / "memory.current").write_text(str(6 << 30))
    (root / "memory.swap.max").write_text("0")
    (root / "memory.events").write_text("low 0\nhigh 3\nmax 1\noom 1\noom_kill 2\n")
    (root / "cpu.max").write_text("150000 100000")
    (root / "cpu.stat").write_text("usage_usec 10\nnr_throttled 5\nthrottled_usec 1200")
    info = cgroups.read_cgroup(root)
    assert info.available and info.events()["oom_kill"] == 2
    txt = cgroups.report(root)
    assert "1.50 CPUs" in txt and "OOM kill" in txt and "2048 MiB" in txt and "quota is being hit" in txt
    assert not cgroups.read_cgroup(tmp_path / "missing").available
    (tmp_path / "v1").mkdir()
    assert "v1" in cgroups.read_cgroup(tmp_path / "v1").reason
