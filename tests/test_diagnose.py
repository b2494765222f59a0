"""Step diagnosis arithmetic (CPU): minimum statistics, severity bands, the
collective finding reading the arm it is given, ranking and serialisation.

Reference coverage: tests/test_perf.py of gpt2-harness (step breakdown
reports the minimum, loader stall found, quiet when the loader keeps up,
collective finding reads the given arm, findings ranked by share, JSON).
"""

import json

import pytest

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.perf.diagnose import (SEVERITY_BANDS, StepBreakdown, SyntheticLoader, diagnose,
                                             measure_step_breakdown, severity)
from gpt2_harness_b200.perf.roofline import MachinePeak

PEAK = MachinePeak("cpu", "float32", 1e11, 1e10, 10.0)
CFG = GPTConfig(vocab_size=128, n_positions=32, n_layer=1, n_head=2, n_embd=32)


def test_severity_bands():
    hi, mid, lo = SEVERITY_BANDS
    assert severity(hi) == "critical" and severity(hi - 1e-9) != "critical"
    assert severity(mid) != severity(lo) != severity(0.0)
    assert severity(0.0) == "healthy"


def test_breakdown_reports_the_minimum():
    bd = StepBreakdown(3, fetch_s=[0.3, 0.1, 0.2], compute_s=[1.0, 2.0, 0.5])
    assert bd.best_fetch_s == 0.1 and bd.best_compute_s == 0.5 and bd.best_step_s == pytest.approx(0.6)
    assert bd.stall_fraction == pytest.approx(0.1 / 0.6)
    d = bd.to_dict()
    assert d["statistic"].startswith("minimum") and d["median_compute_s"] == 1.0


def test_measure_breakdown_counts_steps_and_sees_the_stall():
    calls = []
    loader = SyntheticLoader(128, 2, 8, stall_s=0.02)
    bd = measure_step_breakdown(lambda x, y: calls.append(x.shape), loader, steps=3, warmup=1)
    assert len(calls) == 4 and bd.steps == 3 and len(bd.fetch_s) == 3
    assert bd.best_fetch_s >= 0.02 and bd.stall_fraction > 0.5


def _arm(exposed, overlap):
    return {"exposed_fraction_of_step": exposed, "overlap_fraction": overlap, "step_s": 1.0,
            "step_without_comm_s": 1.0 - exposed, "exposed_comm_s": exposed, "standalone_comm_s": 0.5}


def test_collective_finding_reads_the_given_arm_and_ranks():
    colls = {"ddp_default_buckets": _arm(0.4, 0.2), "ddp_small_buckets": _arm(0.05, 0.9)}
    rep = diagnose(PEAK, CFG, batch=2, seq=16, steps=2, warmup=1, batch_sweep=None, profile_ops=False,
                   collectives=colls)
    names = [f.name for f in rep.findings]
    assert "exposed collective time (ddp_default_buckets)" in names
    top = rep.findings[0]
    assert top.name.startswith("exposed collective") and top.cost_fraction == 0.4
    assert top.severity == "critical" and "backward hooks" in top.recommendation
    other = diagnose(PEAK, CFG, batch=2, seq=16, steps=2, warmup=1, batch_sweep=None, profile_ops=False,
                     collectives=colls, collective_arm="ddp_small_buckets")
    f = next(x for x in other.findings if x.name.startswith("exposed collective"))
    assert f.cost_fraction == 0.05 and "already overlaps" in f.recommendation
    fr = [x.cost_fraction for x in rep.findings]
    assert fr == sorted(fr, reverse=True)
    json.dumps(rep.to_dict())
    assert "ranked findings" in rep.text()


def test_throughput_fields_are_consistent():
    rep = diagnose(PEAK, CFG, batch=2, seq=16, steps=2, warmup=1, batch_sweep=None, profile_ops=False)
    t = rep.throughput
    assert t["tokens_per_s"] == pytest.approx(2 * 16 / t["step_s"])
    assert t["mfu_end_to_end"] <= t["mfu_compute_only"]
    assert 0 < t["roofline_ceiling_mfu"] <= 1.0
