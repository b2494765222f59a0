"""The tensor-parallel MLP expressed with DTensor, checked against the manual
Megatron layers (reference: src/transformer_internals/parallel/
dtensor_demo.py:57-138).

Three computations of proj(gelu(fc(x))) on a 1-D mesh: explicit placements
(Shard(0) fc weight, Shard(1) proj weight, Replicate input; the Partial ->
Replicate redistribute is the all-reduce), ``parallelize_module`` with
Colwise/Rowwise plans, and this package's ColumnParallelLinear /
RowParallelLinear. All three must agree with the single-process MLP.
"""

from __future__ import annotations

from typing import Any, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from gpt2_harness_b200.parallel.common import current_device, parallel_config
from gpt2_harness_b200.parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear

__all__ = ["dtensor_worker"]


def _mlp(n_embd: int, seed: int = 5):
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        fc = nn.Linear(n_embd, 4 * n_embd)
        proj = nn.Linear(4 * n_embd, n_embd)
    return fc, proj


def dtensor_worker(rank: int, world_size: int, batch: int = 4, seq: int = 8,
                   config_kwargs: Optional[dict] = None) -> dict[str, Any]:
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.tensor import Replicate, Shard, distribute_tensor
    from torch.distributed.tensor.parallel import ColwiseParallel, RowwiseParallel, parallelize_module

    cfg = parallel_config(**(config_kwargs or {}))
    dev = current_device()
    C = cfg.n_embd
    fc, proj = _mlp(C)
    fc, proj = fc.to(dev), proj.to(dev)
    torch.manual_seed(6)
    x = torch.randn(batch, seq, C).to(dev)
    ref = proj(F.gelu(fc(x)))
    mesh = DeviceMesh(dev.type, torch.arange(world_size))
    w1 = distribute_tensor(fc.weight, mesh, [Shard(0)])
    b1 = distribute_tensor(fc.bias, mesh, [Shard(0)])
    w2 = distribute_tensor(proj.weight, mesh, [Shard(1)])
    b2 = distribute_tensor(proj.bias, mesh, [Replicate()])
    dx = distribute_tensor(x, mesh, [Replicate()])
    h = F.gelu(F.linear(dx, w1, b1))
    y = F.linear(h, w2).redistribute(mesh, [Replicate()]) + b2
    dt_err = float((y.to_local() - ref).detach().abs().max())
    plan = nn.Sequential()
    plan.add_module("fc", nn.Linear(C, 4 * C))
    plan.add_module("proj", nn.Linear(4 * C, C))
    plan = plan.to(dev)
    plan.fc.load_state_dict(fc.state_dict())
    plan.proj.load_state_dict(proj.state_dict())
    parallelize_module(plan, mesh, {"fc": ColwiseParallel(), "proj": RowwiseParallel()})
    po = plan(x)
    po = po.to_local() if hasattr(po, "to_local") else po
    plan_err = float((po - proj(fc(x))).abs().max())
    man = RowParallelLinear(proj, rank, world_size)(F.gelu(ColumnParallelLinear(fc, rank, world_size)(x)))
    return {"rank": rank, "mesh": [int(v) for v in mesh.mesh.flatten()], "dtensor_error": dt_err,
            "parallelize_module_error": plan_err, "manual_error": float((man - ref).abs().max()),
            "manual_vs_dtensor": float((man - y.to_local()).abs().max()),
            "output_scale": float(ref.abs().max()),
            "local_fc_weight_shape": list(w1.to_local().shape),
            "local_proj_weight_shape": list(w2.to_local().shape)}
