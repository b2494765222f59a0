"""The distributed job entry point on one GPU: train, checkpoint, resume."""

import json
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


def _run(tmp_path, steps, log):
    cmd = [sys.executable, "-m", "gpt2_harness_b200.launch", "--model", "gpt2", "--batch", "4", "--seq", "256",
           "--steps", str(steps), "--warmup", "2", "--ckpt-dir", str(tmp_path / "ck"), "--ckpt-every", "10",
           "--log", str(log)]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=600)


def test_train_checkpoint_resume(tmp_path):
    r1 = _run(tmp_path, 20, tmp_path / "a.jsonl")
    assert r1.returncode == 0, r1.stderr[-2000:]
    assert (tmp_path / "ck" / "step_20" / "index.json").exists()
    r2 = _run(tmp_path, 30, tmp_path / "b.jsonl")
    assert r2.returncode == 0, r2.stderr[-2000:]
    steps = [json.loads(l)["step"] for l in (tmp_path / "b.jsonl").read_text().splitlines()]
    assert steps[0] > 20 and steps[-1] == 30  # resumed, not restarted
    assert (tmp_path / "ck" / "step_30" / "index.json").exists()
