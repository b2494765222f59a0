"""User-facing runners: strategy driver, results gate, preflight, cluster and
experiment runners (CPU)."""

import json
from types import SimpleNamespace

import pytest


def test_compare_results_gate(tmp_path):
    from gpt2_harness_b200.compare_results import compare, load_tree
    base, cur = tmp_path / "a", tmp_path / "b"
    for d in (base, cur):
        d.mkdir()
    doc = {"checks": [{"name": "ddp", "measured": 228096, "predicted": 228096, "ok": True}],
           "equivalence": {"ddp": {"max_grad_error": 1e-7}}, "step_s": 0.5}
    (base / "p.json").write_text(json.dumps(doc))
    doc2 = json.loads(json.dumps(doc))
    doc2["step_s"] = 0.25
    doc2["equivalence"]["ddp"]["max_grad_error"] = 3e-7
    (cur / "p.json").write_text(json.dumps(doc2))
    rep = compare(load_tree(base), load_tree(cur))
    assert rep["ok"] and rep["timings"][0]["ratio"] == 0.5 and len(rep["exact_held"]) >= 2
    doc2["checks"][0]["measured"] = 228100
    doc2["equivalence"]["ddp"]["max_grad_error"] = 2e-5
    (cur / "p.json").write_text(json.dumps(doc2))
    rep = compare(load_tree(base), load_tree(cur))
    assert not rep["ok"] and rep["exact_broken"] and rep["tolerant_broken"]


def test_preflight_dry_run_and_refusals():
    from gpt2_harness_b200.preflight import run
    rep = run(dry_run=True, stub_gpus=8, world_sizes=[1, 2, 4, 8])
    assert rep["ok"] and rep["decisions"]["backend"] == "nccl" and rep["decisions"]["native_kernels"]
    bad = run(dry_run=True, stub_gpus=4, world_sizes=[8])
    assert not bad["ok"] and "exceeds" in bad["decisions"]["problems"][0]
    assert bad["arithmetic"]["gpt2"]["params"] == 124_439_808


@pytest.mark.slow
def test_run_parallel_driver_all_checks_pass(tmp_path):
    from gpt2_harness_b200.parallel.run_parallel import main
    out = tmp_path / "pc.json"
    assert main(["--world-size", "2", "--pipeline-stages", "2", "--steps", "2", "--out", str(out)]) == 0
    res = json.loads(out.read_text())
    names = {c["name"] for c in res["checks"]}
    assert {"data_parallel.all_reduce", "zero_3.total", "tensor_parallel.all_reduce", "cp_ring.send"} <= names


def test_cluster_runner_pieces(tmp_path):
    from gpt2_harness_b200.cluster.run_cluster import measure_resharding, model_the_fabric
    r = measure_resharding(tmp_path)
    assert all(v["bitwise_identical"] for v in r["reshards"].values())
    assert r["reshards"]["2->4"]["files_read_per_rank"] == [1, 1, 1, 1]
    assert "MODELLED" in model_the_fabric()["report"]


def test_experiments_kv_and_verification(tmp_path):
    from gpt2_harness_b200.experiments import main
    assert main(["kv_cache", "--quick", "--out", str(tmp_path), "--device", "cpu"]) == 0
    kv = json.loads((tmp_path / "kv_cache.json").read_text())
    assert {r["arm"] for r in kv["rows"]} >= {"cached", "uncached"}
    assert main(["verification", "--quick", "--out", str(tmp_path), "--device", "cpu"]) == 0
    v = json.loads((tmp_path / "verification.json").read_text())
    assert v["logits_ok"] and v["all_generations_match"]
    assert main(["figures", "--out", str(tmp_path), "--figures", str(tmp_path / "fig")]) == 0
    assert (tmp_path / "fig" / "kv_cache.svg").exists()
