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


RESUME = r'''
import json, sys
from gpt2_harness_b200 import launch
launch.LOSSES = []
launch.main(sys.argv[1:])
print("LOSSES " + json.dumps(launch.LOSSES))
'''


def _losses(tmp_path, ckpt, extra):
    base = ["--model", "gpt2", "--config",
            '{"vocab_size": 1024, "n_positions": 256, "n_layer": 2, "n_head": 4, "n_embd": 256}',
            "--batch", "4", "--seq", "256", "--warmup", "1", "--lr", "1e-3", "--steps", "8",
            "--ckpt-dir", str(tmp_path / ckpt)]
    r = subprocess.run([sys.executable, "-c", RESUME, *base, *extra], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("LOSSES ")][-1]
    return json.loads(line[7:])


def test_resume_is_bit_exact(tmp_path):
    """A run pre-empted after step 4 and resumed from its checkpoint gives the
    uninterrupted run's losses bit for bit: every kernel of the step sums in a
    fixed order (split-K and bias reductions, LayerNorm partials, the token
    embedding gradient), and the checkpoint carries weights, AdamW moments,
    the step count and the data stream position."""
    whole = _losses(tmp_path, "a", ["--ckpt-every", "100"])
    first = _losses(tmp_path, "b", ["--ckpt-every", "2", "--stop-at", "4"])
    rest = _losses(tmp_path, "b", ["--ckpt-every", "100"])
    assert len(whole) == 8 and len(first) == 4 and len(rest) == 4
    assert first == whole[:4]
    assert rest == whole[4:]
