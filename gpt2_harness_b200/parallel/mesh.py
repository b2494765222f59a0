"""N-D process meshes: the composition the reference only models.

The reference composes parallelisms only analytically
(``fabric.ParallelConfig(tp, pp, cp, dp)``, src/transformer_internals/cluster/
fabric.py:186-197); its DTensor mesh is 1-D. The B200 configs need real 2-D
groups: PP=4 x CP=2 for the 16k-context GPT-2 large and DP x TP. A
:class:`Mesh` lays ranks out row-major over named axes and creates one
process group per line along every axis, in the same order on every rank (a
requirement of ``dist.new_group``).

    mesh = Mesh({"pp": 4, "cp": 2})        # rank = pp_index * 2 + cp_index
    mesh.group("cp")                       # this rank's context-parallel pair
    mesh.coord("pp")                       # this rank's pipeline stage
    mesh.neighbor("pp", +1)                # global rank of the next stage
"""

from __future__ import annotations

import itertools
import math
from typing import Any, Optional

import torch.distributed as dist

__all__ = ["Mesh", "mesh_coords"]


def mesh_coords(rank: int, shape: dict[str, int]) -> dict[str, int]:
    """Row-major coordinates of `rank` over the named axes (last axis fastest)."""
    out = {}
    rem = rank
    sizes = list(shape.values())
    for i, name in enumerate(shape):
        stride = math.prod(sizes[i + 1:])
        out[name] = rem // stride
        rem %= stride
    return out


class Mesh:
    """A row-major mesh of ranks with one process group per axis line."""

    def __init__(self, shape: dict[str, int], rank: Optional[int] = None, world: Optional[int] = None,
                 backend: Optional[str] = None, create_groups: bool = True) -> None:
        self.shape = dict(shape)
        self.size = math.prod(self.shape.values())
        self.rank = dist.get_rank() if rank is None else rank
        world = dist.get_world_size() if world is None else world
        if world != self.size:
            raise ValueError(f"mesh {self.shape} needs {self.size} ranks, the job has {world}")
        self.coords = mesh_coords(self.rank, self.shape)
        self.groups: dict[str, Any] = {}
        self.group_ranks: dict[str, list[int]] = {}
        names = list(self.shape)
        for axis in names:
            others = [n for n in names if n != axis]
            for fixed in itertools.product(*[range(self.shape[n]) for n in others]):
                ranks = []
                for a in range(self.shape[axis]):
                    c = dict(zip(others, fixed))
                    c[axis] = a
                    ranks.append(self.rank_of(c))
                g = dist.new_group(ranks, backend=backend) if create_groups else None
                if self.rank in ranks:
                    self.groups[axis] = g
                    self.group_ranks[axis] = ranks

    def rank_of(self, coords: dict[str, int]) -> int:
        r = 0
        for name, size in self.shape.items():
            r = r * size + coords[name]
        return r

    def coord(self, axis: str) -> int:
        return self.coords[axis]

    def group(self, axis: str):
        return self.groups[axis]

    def axis_size(self, axis: str) -> int:
        return self.shape[axis]

    def neighbor(self, axis: str, step: int) -> Optional[int]:
        """Global rank `step` positions along `axis` (None off the end)."""
        c = dict(self.coords)
        c[axis] += step
        if not 0 <= c[axis] < self.shape[axis]:
            return None
        return self.rank_of(c)
