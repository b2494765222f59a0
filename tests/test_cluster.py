"""Streaming loader and failure recovery on CPU processes (no GPU is touched:
crashes are os._exit / SIGKILL of CPU ranks, hangs are a sleeping rank)."""

import numpy as np
import pytest
import torch

from gpt2_harness_b200.cluster.failure import JobSpec, make_corpus, read_log, run_with_recovery
from gpt2_harness_b200.cluster.streaming import (DelayedSource, ShardedStream, StreamState, TokenShardSource,
                                                 global_order, measure_throughput, plan_indices)


# ------------------------------------------------------------------ streaming --
def test_shards_are_disjoint_and_cover_once():
    src = list(range(103))
    seen = []
    for r in range(4):
        seen += list(ShardedStream(src, rank=r, world_size=4, seed=3).plan)
    assert sorted(seen) == sorted(range(103)) or len(set(seen)) == len(seen)
    assert len(set(seen)) == 103


def test_order_depends_only_on_seed_and_epoch():
    a = global_order(50, 1, 2, True)
    assert np.array_equal(a, global_order(50, 1, 2, True))
    assert not np.array_equal(a, global_order(50, 1, 3, True))


def test_mid_epoch_resume_same_world():
    src = list(range(40))
    s = ShardedStream(src, rank=1, world_size=2, seed=5)
    it = iter(s)
    first = [next(it) for _ in range(6)]
    st = StreamState.from_dict(s.state_dict([6, 6]))
    s2 = ShardedStream(src, rank=1, world_size=2, state=st)
    rest = list(s2)
    assert first + rest == [src[i] for i in s.plan]


def test_elastic_resume_consumes_exactly_the_rest():
    src = list(range(60))
    streams = [ShardedStream(src, rank=r, world_size=3, seed=2) for r in range(3)]
    used = []
    for s in streams:
        it = iter(s)
        used += [next(it) for _ in range(5)]
    st = StreamState.from_dict(streams[0].state_dict([5, 5, 5]))
    rest = []
    for r in range(2):  # resume on 2 ranks
        rest += list(ShardedStream(src, rank=r, world_size=2, state=st))
    assert sorted(used + rest) == list(range(60))


def test_prefetch_does_not_skip_unconsumed():
    src = list(range(30))
    s = ShardedStream(src, rank=0, world_size=1, prefetch=8, shuffle=False)
    it = iter(s)
    got = [next(it) for _ in range(4)]
    del it
    assert s.position == 4 and got == [0, 1, 2, 3]


def test_token_source_windows_and_pinned_batches(tmp_path):
    toks = np.arange(1000) % 97
    p = TokenShardSource.write(tmp_path / "t.bin", toks)
    src = TokenShardSource(p, block_size=16)
    x, y = src[2]
    assert torch.equal(y[:-1], x[1:]) and int(x[0]) == toks[32]
    s = ShardedStream(src, rank=0, world_size=1, shuffle=False)
    bx, by = next(s.batches(4))
    assert bx.shape == (4, 16) and s.position == 4


def test_prefetch_overlaps_slow_reads():
    slow = DelayedSource(list(range(40)), 0.004)
    t0 = measure_throughput(slow, 30, prefetch=0, work_s=0.004)
    t8 = measure_throughput(slow, 30, prefetch=8, work_s=0.004)
    assert t8 > 1.3 * t0


# ------------------------------------------------------------------- failure --
def _spec(tmp_path, **kw):
    data = make_corpus(tmp_path / "corpus.bin", n_tokens=30_000, vocab=128, seed=0)
    base = dict(data_path=str(data), ckpt_dir=str(tmp_path / "ckpt"), log_path=str(tmp_path / "log.jsonl"),
                steps=14, ckpt_every=5, micro_batch=4, block_size=32)
    base.update(kw)
    return JobSpec(**base)


def _losses(path):
    out = {}
    for r in read_log(path):
        if r.get("event") == "step":
            out[r["step"]] = r["loss"]
    return out


@pytest.mark.slow
def test_kill_a_rank_and_resume_bit_exact(tmp_path):
    clean = _spec(tmp_path / "clean")
    rep0 = run_with_recovery(2, clean)
    assert rep0.launches == 1
    crashed = _spec(tmp_path / "crash")
    rep = run_with_recovery(2, crashed, kill_rank_at_step=(1, 12))
    assert rep.launches == 2 and rep.resumed_from_step == 10
    a, b = _losses(clean.log_path), _losses(crashed.log_path)
    assert set(range(1, 15)) <= set(b)
    assert max(abs(a[s] - b[s]) for s in range(1, 15)) == 0.0
    assert rep.time_to_recover_s is not None and rep.time_to_recover_s > 0


@pytest.mark.slow
def test_self_crash_resumes_from_checkpoint(tmp_path):
    spec = _spec(tmp_path, crash_step=8, crash_rank=1)
    rep = run_with_recovery(2, spec)
    assert rep.launches == 2 and rep.resumed_from_step == 5
    assert any(r.get("event") == "done" for r in read_log(spec.log_path))


@pytest.mark.slow
def test_hung_rank_is_detected_by_the_watchdog(tmp_path):
    spec = _spec(tmp_path, hang_step=7, hang_rank=0, heartbeat_timeout_s=4.0, pg_timeout_s=30.0)
    rep = run_with_recovery(2, spec, timeout_s=120)
    assert rep.hung_detected
    assert rep.resumed_from_step == 5 and rep.launches == 2
    assert any(r.get("event") == "done" for r in read_log(spec.log_path))
