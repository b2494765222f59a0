"""The benchmark's output contract on CPU: with the native ops replaced by
their torch contracts (tests/native_fake.py) and CUDA timing emulated on the
host, `bench.py` must print exactly one JSON line with every key the driver
reads, for the default data-parallel arm and the pipeline arm."""

import json
import sys
import time

import pytest
import torch
import torch.distributed as dist

import native_fake

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
            "scaling", "vs_baseline", "dtype", "data", "config", "e2e", "gpu_launches", "clocks"}


class _TimedEvent(native_fake._Event):
    def __init__(self, *a, **k):
        self.t = None

    def record(self, *a, **k):
        self.t = time.perf_counter()

    def elapsed_time(self, other):
        return (other.t - self.t) * 1e3


@pytest.fixture
def bench_env(monkeypatch):
    with native_fake.installed(monkeypatch):
        monkeypatch.setattr(torch.cuda, "Event", _TimedEvent)
        monkeypatch.setattr(torch.Tensor, "cuda", lambda self, *a, **k: self)
        native_fake.LIB.launch_count = lambda: 0
        from gpt2_harness_b200 import trainer as trainer_mod

        for cls_name in ("Trainer", "PipelineTrainer"):
            cls = getattr(trainer_mod, cls_name)
            # the benchmark builds its trainer on the default CUDA device: run it on the host
            monkeypatch.setattr(trainer_mod, cls_name, type(cls_name, (cls,), {
                "__init__": lambda self, *a, _cls=cls, **k: _cls.__init__(self, *a, **{**k, "device": "cpu"})}))
        import bench

        yield bench


def _run(bench, capsys, monkeypatch, args):
    monkeypatch.setattr(sys, "argv", ["bench.py", *args])
    bench.main()
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_data_parallel_line(bench_env, capsys, monkeypatch):
    out = _run(bench_env, capsys, monkeypatch, ["--steps", "1", "--warmup", "3", "--batch", "1", "--seq", "64"])
    assert REQUIRED <= set(out)
    assert out["n_gpus"] == 1 and out["steps"] == 1 and out["warmup"] == 3
    assert out["value"] > 0 and out["higher_is_better"] is True and out["scaling"] == "weak"
    assert out["e2e"]["h2d_bytes_per_step"] == 2 * 64 * 8 and out["e2e"]["d2h_bytes_per_step"] == 4
    assert out["config"]["parallelism"] == "dp1" and out["dtype"] == "bf16"
    assert out["value"] == pytest.approx(64 / (out["ms_per_step"] / 1e3), rel=1e-3, abs=0.06)  # value has one decimal


def test_pipeline_line(bench_env, capsys, monkeypatch):
    dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        out = _run(bench_env, capsys, monkeypatch, ["--strategy", "pp", "--steps", "1", "--warmup", "3",
                                                    "--batch", "1", "--seq", "64", "--micro-batches", "2"])
    finally:
        dist.destroy_process_group()
    assert REQUIRED <= set(out)
    assert out["scaling"] == "strong" and out["config"]["parallelism"] == "pp1xcp1-1f1b"
    assert out["config"]["global_batch"] == 2 and out["config"]["micro_batches"] == 2


def test_reference_arm_reports_unavailable_for_the_pipeline(bench_env, capsys, monkeypatch):
    out = _run(bench_env, capsys, monkeypatch, ["--impl", "reference", "--strategy", "pp"])
    assert out["impl"] == "reference" and "unavailable" in out
