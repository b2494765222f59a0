"""Shard planning of the native ZeRO-2 path (CPU): every bucket element is
owned by exactly one rank, slices are 64-element aligned, shard offsets are
contiguous."""

import pytest

from gpt2_harness_b200.config import gpt2_config
from gpt2_harness_b200.models.engine import ALIGN, ParamLayout
from gpt2_harness_b200.parallel.zero_native import plan_shards


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("bucket_mb", [1, 25])
def test_plan_covers_every_element_once(world, bucket_mb):
    layout = ParamLayout(gpt2_config("gpt2", n_layer=2))
    plan = plan_shards(layout, world, bucket_mb * 1024 * 1024)
    covered = []
    for r in range(world):
        offs = []
        for f0, n, off in plan.owned(r):
            assert f0 % ALIGN == 0 and n % ALIGN == 0 and off % ALIGN == 0
            if n:
                covered.append((f0, f0 + n))
            offs.append(off)
        assert offs == [row[3] for row in plan.table]
    covered.sort()
    assert covered[0][0] == 0 and covered[-1][1] == layout.total
    for (a0, a1), (b0, b1) in zip(covered, covered[1:]):
        assert a1 == b0
    # shard-sized buffers hold every slice of every bucket
    assert plan.shard_numel == sum(row[2] for row in plan.table)
    for lo, hi, s, _ in plan.table:
        assert s * world >= hi - lo
