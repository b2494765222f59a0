"""Deploy recipes parse, and the job entry point resolves checkpoints."""

import ast
import subprocess
from pathlib import Path

import yaml

ROOT = Path(__file__).resolve().parents[1]


def test_shell_recipes_parse():
    for f in ("deploy/run_on_gpu.sh", "deploy/slurm_train.sbatch", "deploy/cgroups_demo.sh"):
        assert subprocess.run(["bash", "-n", str(ROOT / f)]).returncode == 0, f


def test_k8s_and_ci_yaml():
    for f in ("deploy/k8s/job-indexed.yaml", "deploy/k8s/statefulset.yaml"):
        docs = list(yaml.safe_load_all((ROOT / f).read_text()))
        kinds = {d["kind"] for d in docs}
        assert "Service" in kinds and ("Job" in kinds or "StatefulSet" in kinds)
        pod = [d for d in docs if d["kind"] != "Service"][0]["spec"]["template"]["spec"]
        c = pod["containers"][0]
        assert c["resources"]["limits"]["nvidia.com/gpu"] == 8
        assert "IPC_LOCK" in c["securityContext"]["capabilities"]["add"]
        assert "gpt2_harness_b200.launch" in " ".join(c["args"])
    ci = yaml.safe_load((ROOT / ".github/workflows/ci.yml").read_text())
    assert {"cpu", "build"} <= set(ci["jobs"])


def test_ray_recipe_is_valid_python():
    ast.parse((ROOT / "deploy/ray_train.py").read_text())


def test_latest_checkpoint(tmp_path):
    from gpt2_harness_b200.launch import latest_checkpoint
    assert latest_checkpoint(tmp_path / "none") is None
    for s in (500, 1000, 1500):
        (tmp_path / f"step_{s}").mkdir()
    (tmp_path / "step_500" / "index.json").write_text("{}")
    (tmp_path / "step_1000" / "index.json").write_text("{}")
    assert latest_checkpoint(tmp_path).name == "step_1000"  # step_1500 is incomplete
