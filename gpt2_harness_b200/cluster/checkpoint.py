"""Sharded checkpoints that reshard across world sizes.

On-disk format identical to the reference's (src/transformer_internals/
cluster/checkpoint.py:68-498) so checkpoints move between the two frameworks:

* one ``shard_{rank:04d}_of_{world:04d}.pt`` per rank holding
  ``{rank, world_size, step, tensors, extra}``, written atomically
  (``.pt.tmp`` then rename);
* rank 0 writes ``index.json`` = ``{format, world_size, step, plan,
  global_shapes, meta}`` with ``format == "transformer-internals-sharded-v1"``;
* a plan maps each tensor to a :class:`ShardSpec` (replicate, or shard along
  ``dim`` with ``sections`` fused sub-matrices split independently, e.g. QKV).

:func:`load_reshard` builds any destination rank's slice by reading only the
source shards that overlap it (``files_read`` is reported and tested).

B200 additions: :func:`gpt2_tp_plan` can pad the vocabulary (``pad_vocab``:
50257 -> 50304 rows of the tied table) so a vocab-parallel split divides any
TP degree; :func:`engine_state_dict` / :func:`load_into_engine` connect the
format to the native engine's flat buffers; :class:`AsyncCheckpointer`
snapshots device tensors into pinned host memory and serialises on a
background thread.
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Optional

import torch

__all__ = [
    "FORMAT",
    "REPLICATE",
    "AsyncCheckpointer",
    "CheckpointIndex",
    "ShardSpec",
    "engine_state_dict",
    "gpt2_tp_plan",
    "load_extra",
    "load_full",
    "load_into_engine",
    "load_reshard",
    "merge_pieces",
    "pad_vocab_rows",
    "save_sharded",
    "shard_path",
    "shard_state_dict",
    "split_tensor",
]

FORMAT = "transformer-internals-sharded-v1"


@dataclass(frozen=True)
class ShardSpec:
    """How one tensor is laid out across ranks: ``replicate`` or ``shard``
    along ``dim`` with ``sections`` fused sub-matrices (rank r owns slice r of
    every section)."""

    kind: str = "replicate"
    dim: int = 0
    sections: int = 1

    def __post_init__(self) -> None:
        if self.kind not in ("replicate", "shard"):
            raise ValueError(f"unknown shard kind {self.kind!r}")
        if self.sections < 1:
            raise ValueError(f"sections must be >= 1, got {self.sections}")

    @property
    def replicated(self) -> bool:
        return self.kind == "replicate"

    @staticmethod
    def from_dict(d: dict) -> "ShardSpec":
        return ShardSpec(kind=d["kind"], dim=int(d.get("dim", 0)), sections=int(d.get("sections", 1)))


REPLICATE = ShardSpec("replicate")


def split_tensor(tensor: torch.Tensor, spec: ShardSpec, world_size: int) -> list[torch.Tensor]:
    """The `world_size` local pieces of `tensor` under `spec` (contiguous
    clones). Uneven splits and splits across a fused section are refused."""
    if spec.replicated:
        return [tensor.clone() for _ in range(world_size)]
    size = tensor.shape[spec.dim]
    if size % spec.sections:
        raise ValueError(f"dim {spec.dim} of size {size} is not divisible into {spec.sections} sections")
    section = size // spec.sections
    if section % world_size:
        raise ValueError(f"section of size {section} does not divide evenly across world_size={world_size}; "
                         "pad the tensor (e.g. the vocabulary) at model construction instead")
    per = section // world_size
    out = []
    for r in range(world_size):
        parts = [tensor.narrow(spec.dim, s * section + r * per, per) for s in range(spec.sections)]
        out.append(torch.cat(parts, dim=spec.dim).contiguous() if len(parts) > 1 else parts[0].clone())
    return out


def merge_pieces(pieces: list[torch.Tensor], spec: ShardSpec) -> torch.Tensor:
    """Inverse of :func:`split_tensor`."""
    if spec.replicated:
        return pieces[0].clone()
    per = pieces[0].shape[spec.dim] // spec.sections
    parts = [p.narrow(spec.dim, s * per, per) for s in range(spec.sections) for p in pieces]
    return torch.cat(parts, dim=spec.dim).contiguous()


def pad_vocab_rows(t: torch.Tensor, padded: int) -> torch.Tensor:
    """Zero rows appended so dim 0 has `padded` rows (never-selected tokens)."""
    if t.shape[0] >= padded:
        return t
    return torch.cat([t, t.new_zeros((padded - t.shape[0],) + tuple(t.shape[1:]))], dim=0)


def gpt2_tp_plan(state_dict: dict, *, vocab_parallel: bool = True) -> dict[str, ShardSpec]:
    """Megatron plan for GPT-2: c_attn column-parallel with sections=3 (q, k,
    v split separately), c_fc column-parallel, both c_proj row-parallel (dim
    1; their biases replicated, added once after the reduction), wte/lm_head
    vocab-parallel on dim 0 (tied: same spec), everything else replicated."""
    plan = {}
    for name in state_dict:
        if name.endswith(("attn.c_attn.weight", "attn.c_attn.bias")):
            plan[name] = ShardSpec("shard", dim=0, sections=3)
        elif name.endswith(("attn.c_proj.weight", "mlp.c_proj.weight")):
            plan[name] = ShardSpec("shard", dim=1)
        elif name.endswith(("mlp.c_fc.weight", "mlp.c_fc.bias")) or (
                vocab_parallel and name in ("wte.weight", "lm_head.weight")):
            plan[name] = ShardSpec("shard", dim=0)
        else:
            plan[name] = REPLICATE
    return plan


def shard_state_dict(state_dict: dict, plan: dict, rank: int, world_size: int) -> dict:
    return {n: split_tensor(t, plan.get(n, REPLICATE), world_size)[rank] for n, t in state_dict.items()}


@dataclass
class CheckpointIndex:
    """The JSON that makes a directory of shard files self-describing."""

    format: str
    world_size: int
    step: int
    plan: dict
    global_shapes: dict
    meta: dict

    def to_json(self) -> str:
        return json.dumps({"format": self.format, "world_size": self.world_size, "step": self.step,
                           "plan": {k: asdict(v) for k, v in self.plan.items()},
                           "global_shapes": self.global_shapes, "meta": self.meta},
                          indent=2, sort_keys=True)

    @staticmethod
    def read(directory) -> "CheckpointIndex":
        d = json.loads((Path(directory) / "index.json").read_text())
        if d["format"] != FORMAT:
            raise ValueError(f"unknown checkpoint format {d['format']!r}")
        return CheckpointIndex(d["format"], int(d["world_size"]), int(d["step"]),
                               {k: ShardSpec.from_dict(v) for k, v in d["plan"].items()},
                               {k: list(v) for k, v in d["global_shapes"].items()}, d["meta"])


def shard_path(directory, rank: int, world_size: int) -> Path:
    return Path(directory) / f"shard_{rank:04d}_of_{world_size:04d}.pt"


def save_sharded(directory, local_state: dict, plan: dict, *, rank: int, world_size: int, step: int = 0,
                 global_shapes: Optional[dict] = None, extra: Optional[dict] = None,
                 meta: Optional[dict] = None) -> Path:
    """Write this rank's shard (and, from rank 0, the index), atomically."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    path = shard_path(directory, rank, world_size)
    payload = {"rank": rank, "world_size": world_size, "step": step,
               "tensors": {k: v.detach().cpu() if v.is_cuda else v for k, v in local_state.items()},
               "extra": extra or {}}
    tmp = path.with_suffix(".pt.tmp")
    torch.save(payload, tmp)
    tmp.replace(path)
    if rank == 0:
        if global_shapes is None:
            raise ValueError("rank 0 must pass global_shapes so the index can describe the checkpoint")
        idx = CheckpointIndex(FORMAT, world_size, step, {k: plan.get(k, REPLICATE) for k in local_state},
                              global_shapes, meta or {})
        itmp = directory / "index.json.tmp"
        itmp.write_text(idx.to_json())
        itmp.replace(directory / "index.json")
    return path


class _ShardReader:
    """Opens shard files lazily (mmap) and counts the files it touched."""

    def __init__(self, directory, world_size: int) -> None:
        self.directory, self.world_size = Path(directory), world_size
        self._cache: dict[int, dict] = {}
        self.files_read = 0

    def payload(self, rank: int) -> dict:
        if rank not in self._cache:
            p = shard_path(self.directory, rank, self.world_size)
            try:
                self._cache[rank] = torch.load(str(p), map_location="cpu", mmap=True, weights_only=False)
            except (RuntimeError, TypeError):
                self._cache[rank] = torch.load(p, map_location="cpu", weights_only=False)
            self.files_read += 1
        return self._cache[rank]

    def tensor(self, rank: int, name: str) -> torch.Tensor:
        return self.payload(rank)["tensors"][name]


def _reshard_one(reader: _ShardReader, name: str, spec: ShardSpec, global_size: int, src_world: int,
                 dst_world: int, dst_rank: int) -> torch.Tensor:
    section = global_size // spec.sections
    src_per, dst_per = section // src_world, section // dst_world
    parts = []
    for s in range(spec.sections):
        lo, hi = dst_rank * dst_per, dst_rank * dst_per + dst_per
        for r in range(lo // src_per, (hi - 1) // src_per + 1):
            src_lo = r * src_per
            a, b = max(lo, src_lo), min(hi, src_lo + src_per)
            parts.append(reader.tensor(r, name).narrow(spec.dim, s * src_per + (a - src_lo), b - a))
    return torch.cat(parts, dim=spec.dim).contiguous() if len(parts) > 1 else parts[0].clone()


def load_reshard(directory, *, rank: int, world_size: int, plan: Optional[dict] = None):
    """This rank's slice of a `world_size`-way layout, from a checkpoint saved
    at any world size. Returns (local_state, index, files_read)."""
    index = CheckpointIndex.read(directory)
    plan = plan or index.plan
    reader = _ShardReader(directory, index.world_size)
    replica_src = min(index.world_size - 1, (rank * index.world_size) // max(world_size, 1))
    out = {}
    for name, saved in index.plan.items():
        want = plan.get(name, REPLICATE)
        gsize = index.global_shapes[name][saved.dim] if not saved.replicated else 0
        if want.replicated and not saved.replicated:
            out[name] = merge_pieces([reader.tensor(r, name) for r in range(index.world_size)], saved)
        elif want.replicated:
            out[name] = reader.tensor(replica_src, name).clone()
        elif saved.replicated:
            out[name] = split_tensor(reader.tensor(replica_src, name), want, world_size)[rank]
        else:
            if (want.dim, want.sections) != (saved.dim, saved.sections):
                raise ValueError(f"{name}: cannot reshard from {saved} to {want}; the shard axis would change")
            out[name] = _reshard_one(reader, name, saved, gsize, index.world_size, world_size, rank)
    return out, index, reader.files_read


def load_full(directory):
    """The complete unsharded state dict."""
    index = CheckpointIndex.read(directory)
    state, index, _ = load_reshard(directory, rank=0, world_size=1, plan=dict.fromkeys(index.plan, REPLICATE))
    return state, index


def load_extra(directory, rank: int) -> dict:
    """The non-tensor payload (optimizer step, RNG, data position)."""
    index = CheckpointIndex.read(directory)
    src = rank if rank < index.world_size else 0
    return torch.load(shard_path(directory, src, index.world_size), map_location="cpu", weights_only=False)["extra"]


# ------------------------------------------------------------- native engine --
def engine_state_dict(engine, with_optimizer: bool = False, zero=None) -> tuple[dict, dict]:
    """(tensors, extra) of a native Engine in the reference naming (fp32);
    with_optimizer adds flat AdamW moments and step to `extra`.

    Under ZeRO-2/3 pass the engine's ``NativeZeRO``/``NativeZeRO3`` as `zero`: the master
    weights and moments are then gathered from the shards (a collective that
    every rank must enter) into the same full-vector format DDP writes, so a
    checkpoint resumes under either strategy and any world size."""
    extra: dict[str, Any] = {"optim_step": engine.step_count}
    if zero is not None:
        full = zero.full_master()
        sd = {s.name: engine.layout.view(full, s.name) for s in engine.layout.specs}
        if with_optimizer:
            m, v = zero.full_moments()
            extra["exp_avg"] = m.cpu()
            extra["exp_avg_sq"] = v.cpu()
        return sd, extra
    sd = {s.name: engine.p32(s.name).detach() for s in engine.layout.specs}
    if with_optimizer:
        extra["exp_avg"] = engine.exp_avg.detach().cpu()
        extra["exp_avg_sq"] = engine.exp_avg_sq.detach().cpu()
    return sd, extra


def load_into_engine(engine, state: dict, extra: Optional[dict] = None, zero=None) -> None:
    """Load reference-named tensors (+ optional moments) into an Engine (or,
    with `zero`, into the ZeRO-2 shards and the full bf16 parameters)."""
    if zero is not None:
        full = torch.zeros(engine.layout.total, dtype=torch.float32, device=engine.device)
        for s in engine.layout.specs:
            src = state[s.name] if s.name in state else state["lm_head.weight"]
            engine.layout.view(full, s.name).copy_(src.to(engine.device, torch.float32).view(s.shape))
        ea = eq = None
        if extra and "exp_avg" in extra:
            ea = extra["exp_avg"].to(engine.device)
            eq = extra["exp_avg_sq"].to(engine.device)
        zero.load_full(full, ea, eq)
        if extra:
            engine.step_count = int(extra.get("optim_step", engine.step_count))
        return
    engine.load_state_dict(state)
    if extra:
        if "exp_avg" in extra:
            engine.exp_avg.copy_(extra["exp_avg"].to(engine.device))
            engine.exp_avg_sq.copy_(extra["exp_avg_sq"].to(engine.device))
        engine.step_count = int(extra.get("optim_step", engine.step_count))


class AsyncCheckpointer:
    """Snapshot on the training thread, serialise on a background thread.

    Device tensors are copied into reusable pinned host buffers (the only part
    the step waits for: the optimizer will overwrite them in place); the
    ``torch.save`` happens on a writer thread. One write in flight at a time;
    a failure surfaces on the next :meth:`wait` / :meth:`save`.
    """

    def __init__(self) -> None:
        self._thread: Optional[threading.Thread] = None
        self._error: Optional[BaseException] = None
        self._pinned: dict[str, torch.Tensor] = {}
        self.last_blocking_seconds = 0.0
        self.last_write_seconds = 0.0

    def _snapshot(self, local_state: dict) -> dict:
        snap = {}
        for k, v in local_state.items():
            v = v.detach()
            if v.is_cuda:
                buf = self._pinned.get(k)
                if buf is None or buf.shape != v.shape or buf.dtype != v.dtype:
                    buf = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
                    self._pinned[k] = buf
                buf.copy_(v, non_blocking=True)
                snap[k] = buf
            else:
                snap[k] = v.clone()
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.current_stream().synchronize()
        return snap

    def save(self, directory, local_state: dict, **kwargs: Any) -> None:
        t0 = time.perf_counter()
        self.wait()
        snap = self._snapshot(local_state)
        self.last_blocking_seconds = time.perf_counter() - t0

        def run() -> None:
            w0 = time.perf_counter()
            try:
                save_sharded(directory, snap, **kwargs)
            except BaseException as exc:  # surfaced on the next wait()
                self._error = exc
            self.last_write_seconds = time.perf_counter() - w0

        self._thread = threading.Thread(target=run, name="ckpt-writer", daemon=False)
        self._thread.start()

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            err, self._error = self._error, None
            raise err
