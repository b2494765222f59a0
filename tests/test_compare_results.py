"""The results gate (CPU): which leaves are exact invariants, which are
tolerant, which are timings, how list rows are keyed, and the exit status.

Reference coverage: tests/test_compare_results.py of gpt2-harness.
"""

import json
import subprocess

from gpt2_harness_b200.compare_results import EQUIVALENCE_TOLERANCE, compare, flatten, load_tree, main


def _tree(tmp_path, name, doc):
    d = tmp_path / name
    d.mkdir(exist_ok=True)
    (d / "r.json").write_text(json.dumps(doc))
    return d


DOC = {"comms": [{"op": "all_reduce", "payload_bytes": 228096, "calls": 1}],
       "equivalence": {"zero3": {"max_grad_error": 1e-6}}, "wall_clock": 3.0, "notes": {"lr": 3e-4}}


def test_unchanged_run_holds_every_invariant(tmp_path):
    a, b = _tree(tmp_path, "a", DOC), _tree(tmp_path, "b", DOC)
    rep = compare(load_tree(a), load_tree(b))
    assert rep["ok"] and not rep["moved"] and not rep["missing"] and not rep["new"]
    assert len(rep["exact_held"]) == 2 and len(rep["tolerant_held"]) == 1


def test_tolerance_boundary_is_absolute_not_a_ratio(tmp_path):
    a = _tree(tmp_path, "a", DOC)
    for err, ok in ((EQUIVALENCE_TOLERANCE, True), (EQUIVALENCE_TOLERANCE * 1.01, False), (1e-9, True)):
        doc = json.loads(json.dumps(DOC))
        doc["equivalence"]["zero3"]["max_grad_error"] = err
        rep = compare(load_tree(a), load_tree(_tree(tmp_path, "b", doc)))
        assert rep["ok"] is ok, err


def test_bytes_and_calls_may_not_move_but_timings_may(tmp_path):
    a = _tree(tmp_path, "a", DOC)
    doc = json.loads(json.dumps(DOC))
    doc["wall_clock"] = 30.0
    rep = compare(load_tree(a), load_tree(_tree(tmp_path, "b", doc)))
    assert rep["ok"] and rep["timings"][0]["ratio"] == 10.0
    doc["comms"][0]["calls"] = 2
    rep = compare(load_tree(a), load_tree(_tree(tmp_path, "c", doc)))
    assert not rep["ok"] and rep["exact_broken"][0]["path"].endswith(".calls")
    doc = json.loads(json.dumps(DOC))
    doc["notes"]["lr"] = 6e-4
    rep = compare(load_tree(a), load_tree(_tree(tmp_path, "d", doc)))
    assert rep["ok"] and rep["moved"][0]["path"].endswith("notes.lr")


def test_list_rows_are_keyed_by_name():
    rows = [{"name": "ddp", "v": 1}, {"name": "zero", "v": 2}]
    flat = flatten({"x": rows})
    assert "x[ddp].v" in flat and "x[zero].v" in flat
    ins = flatten({"x": [{"name": "tp", "v": 0}] + rows})
    assert ins["x[ddp].v"] == 1 and ins["x[zero].v"] == 2
    coll = flatten({"x": [{"name": "a", "v": 1}, {"name": "a", "v": 2}]})
    assert coll["x[0].v"] == 1 and coll["x[1].v"] == 2  # colliding names fall back to indices
    ops = flatten({"c": [{"op": "all_reduce", "world_size": 2, "b": 1}, {"op": "all_reduce", "world_size": 4, "b": 2}]})
    assert ops["c[all_reduce@2].b"] == 1 and ops["c[all_reduce@4].b"] == 2


def test_main_exit_status(tmp_path):
    a = _tree(tmp_path, "a", DOC)
    assert main(["--baseline", str(a), "--current", str(a)]) == 0
    doc = json.loads(json.dumps(DOC))
    doc["comms"][0]["payload_bytes"] += 4
    b = _tree(tmp_path, "b", doc)
    out = tmp_path / "rep.json"
    assert main(["--baseline", str(a), "--current", str(b), "--json", str(out)]) == 1
    assert json.loads(out.read_text())["exact_broken"]


def test_git_baseline_reads_the_committed_tree(tmp_path, monkeypatch):
    repo = tmp_path / "repo"
    (repo / "results").mkdir(parents=True)
    (repo / "results" / "r.json").write_text(json.dumps(DOC))
    run = lambda *c: subprocess.run(c, cwd=repo, check=True, capture_output=True)
    run("git", "init", "-q")
    run("git", "-c", "user.email=a@b", "-c", "user.name=t", "add", ".")
    run("git", "-c", "user.email=a@b", "-c", "user.name=t", "commit", "-qm", "x")
    doc = json.loads(json.dumps(DOC))
    doc["comms"][0]["calls"] = 5
    (repo / "results" / "r.json").write_text(json.dumps(doc))
    monkeypatch.chdir(repo)
    assert main(["--baseline-git", "HEAD", "--current", "results"]) == 1
