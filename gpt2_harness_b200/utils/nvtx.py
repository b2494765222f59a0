"""NVTX ranges around the framework's fused operations, for timeline profilers
(Nsight Systems, the torch profiler's CUDA trace).

Off by default: a disabled range is one Python attribute lookup and an empty
context manager, so the training step pays nothing measurable. Set
``G2B_NVTX=1`` in the environment (before the first import) to emit ranges:
``fwd/h.<l>``, ``bwd/h.<l>``, ``lm_head+ce``, ``optimizer``, and on the
communication side ``allreduce/bucket<i>``, ``tp/all_gather``,
``tp/reduce_scatter``, ``zero3/gather/h.<l>``, ``zero3/reduce_scatter/h.<l>``,
``cp/gather/<i>`` or ``cp/publish/<i>`` (layer-slot i) and ``cp/reduce_scatter``.
"""

from __future__ import annotations

import os

import torch

__all__ = ["ENABLED", "nvtx_range"]

ENABLED = os.environ.get("G2B_NVTX", "0") == "1"


class _Range:
    __slots__ = ("name",)

    def __init__(self, name: str) -> None:
        self.name = name

    def __enter__(self):
        torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc) -> None:
        torch.cuda.nvtx.range_pop()


class _Off:
    __slots__ = ()

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        return None


_OFF = _Off()


def nvtx_range(name: str):
    """Context manager: an NVTX range named `name` when enabled, else nothing."""
    return _Range(name) if ENABLED else _OFF
