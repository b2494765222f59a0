"""Hardware detection and placement decisions.

Same surface as the reference's ``transformer_internals.hardware``
(src/transformer_internals/hardware.py:61-506): a :class:`Capabilities`
snapshot (detected, or fabricated by :meth:`Capabilities.stub` so the CUDA
branches are testable without CUDA), pure decision functions over it
(:func:`select_backend`, :func:`select_device`, :func:`check_placement`) and a
thin impure edge (:func:`nvidia_smi`, :func:`set_visible_device`,
:func:`synchronize`).

B200 additions: :attr:`Capabilities.is_blackwell` (compute capability 10.x,
the sm_100a target of the native kernels) and :func:`native_kernels_supported`.
Nothing here changes a GPU setting; :func:`nvidia_smi` only queries.
"""

from __future__ import annotations

import os
import platform
import shutil
import subprocess
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

import torch

__all__ = [
    "BACKENDS",
    "Capabilities",
    "HardwareError",
    "check_placement",
    "describe",
    "environment_payload",
    "native_kernels_supported",
    "nvidia_smi",
    "select_backend",
    "select_device",
    "set_visible_device",
    "synchronize",
]

#: Supported process-group backends. MPI is deliberately not offered.
BACKENDS = ("nccl", "gloo")


class HardwareError(RuntimeError):
    """A requested placement or backend this machine cannot honour."""


@dataclass(frozen=True)
class Capabilities:
    """What this machine offers (or, with ``source == "stub"``, pretends to)."""

    cuda_available: bool = False
    device_count: int = 0
    nccl_available: bool = False
    gloo_available: bool = True
    mps_available: bool = False
    device_names: tuple = ()
    compute_capabilities: tuple = ()
    total_memory_bytes: tuple = ()
    driver_version: Optional[str] = None
    cuda_runtime_version: Optional[str] = None
    nccl_version: Optional[str] = None
    torch_version: str = ""
    platform: str = ""
    source: str = "detected"
    notes: tuple = field(default_factory=tuple)

    @classmethod
    def detect(cls) -> "Capabilities":
        notes: list[str] = []
        cuda = bool(torch.cuda.is_available())
        n = torch.cuda.device_count() if cuda else 0
        names, caps, mems = [], [], []
        for i in range(n):
            try:
                p = torch.cuda.get_device_properties(i)
                names.append(p.name)
                caps.append((p.major, p.minor))
                mems.append(int(p.total_memory))
            except Exception as exc:  # pragma: no cover - driver dependent
                notes.append(f"device {i}: {exc!r}")
        dist = torch.distributed
        nccl = bool(dist.is_available() and dist.is_nccl_available()) and cuda
        gloo = bool(dist.is_available() and dist.is_gloo_available())
        nccl_ver = None
        if nccl:
            try:
                v = torch.cuda.nccl.version()
                nccl_ver = ".".join(str(x) for x in v) if isinstance(v, tuple) else str(v)
            except Exception:  # pragma: no cover
                pass
        mps = bool(getattr(torch.backends, "mps", None) and torch.backends.mps.is_available())
        return cls(cuda, n, nccl, gloo, mps, tuple(names), tuple(caps), tuple(mems),
                   _driver_version(), torch.version.cuda, nccl_ver, torch.__version__,
                   platform.platform(), "detected", tuple(notes))

    @classmethod
    def stub(cls, device_count: int = 8, name: str = "NVIDIA B200",
             capability: tuple = (10, 0), total_memory_bytes: int = 183359 * 1024 * 1024,
             nccl_version: str = "2.28.9") -> "Capabilities":
        """A fabricated CUDA machine (``source == "stub"``) for dry runs/tests."""
        return cls(device_count > 0, device_count, device_count > 0, True, False,
                   tuple([name] * device_count), tuple([tuple(capability)] * device_count),
                   tuple([total_memory_bytes] * device_count), "stub", "stub", nccl_version,
                   torch.__version__, platform.platform(), "stub",
                   ("fabricated capabilities: no CUDA device was queried",))

    @property
    def bf16_supported(self) -> bool:
        """bf16 tensor cores on every visible device (compute capability >= 8)."""
        return self.device_count > 0 and all(c[0] >= 8 for c in self.compute_capabilities)

    @property
    def is_blackwell(self) -> bool:
        """Every visible device is compute capability 10.x (B200 / sm_100)."""
        return self.device_count > 0 and all(c[0] == 10 for c in self.compute_capabilities)

    @property
    def accelerator(self) -> str:
        if self.cuda_available and self.device_count:
            return "cuda"
        return "mps" if self.mps_available else "cpu"

    def to_dict(self) -> dict[str, Any]:
        d = asdict(self)
        d["bf16_supported"] = self.bf16_supported
        d["is_blackwell"] = self.is_blackwell
        d["accelerator"] = self.accelerator
        return d


def _driver_version() -> Optional[str]:
    out = nvidia_smi("--query-gpu=driver_version", "--format=csv,noheader")
    return out.splitlines()[0].strip() if out else None


def native_kernels_supported(caps: Optional[Capabilities] = None) -> bool:
    """Whether the sm_100a native library can run here (a B200-class GPU)."""
    caps = caps or Capabilities.detect()
    return caps.is_blackwell


def select_backend(caps: Capabilities, requested: Optional[str] = None) -> str:
    """NCCL when CUDA+NCCL exist, gloo otherwise; an explicit request that the
    machine cannot honour is refused rather than silently downgraded."""
    if requested in (None, "auto"):
        return "nccl" if (caps.cuda_available and caps.nccl_available and caps.device_count) else "gloo"
    if requested not in BACKENDS:
        raise HardwareError(f"unknown backend {requested!r}; expected one of {BACKENDS} or 'auto'")
    if requested == "nccl":
        if not caps.cuda_available or caps.device_count <= 0:
            raise HardwareError("backend 'nccl' was requested but no CUDA device is visible; "
                                "use --backend auto to run on gloo, or fix CUDA_VISIBLE_DEVICES")
        if not caps.nccl_available:
            raise HardwareError("backend 'nccl' was requested but this torch build has no NCCL")
        return "nccl"
    if not caps.gloo_available:
        raise HardwareError("backend 'gloo' was requested but this torch build has no gloo")
    return "gloo"


def select_device(caps: Capabilities, rank: int, backend: str) -> str:
    """``cuda:<rank % device_count>`` under NCCL, ``cpu`` under gloo."""
    if backend != "nccl":
        return "cpu"
    if caps.device_count <= 0:
        raise HardwareError("backend 'nccl' with zero visible CUDA devices")
    return f"cuda:{rank % caps.device_count}"


def check_placement(caps: Capabilities, world_size: int, backend: str,
                    allow_oversubscribe: bool = False) -> list[str]:
    """Validate a world size against the machine and return per-rank devices.

    More NCCL ranks than GPUs is refused unless asked for: ranks sharing a GPU
    serialise on it, so every timing taken that way measures contention.
    """
    if world_size < 1:
        raise HardwareError(f"world_size must be at least 1, got {world_size}")
    if backend == "nccl":
        if caps.device_count <= 0:
            raise HardwareError("backend 'nccl' with zero visible CUDA devices "
                                "(an empty CUDA_VISIBLE_DEVICES hides every GPU)")
        if world_size > caps.device_count and not allow_oversubscribe:
            raise HardwareError(
                f"world size {world_size} exceeds the {caps.device_count} visible CUDA device(s); "
                "ranks sharing a GPU serialise on it. Reduce the world size or allow "
                "oversubscription for correctness-only runs.")
    return [select_device(caps, r, backend) for r in range(world_size)]


def describe(caps: Capabilities, topology: Optional[str] = None) -> str:
    """Human-readable summary of the machine (and its NVLink topology)."""
    lines = [f"torch {caps.torch_version}, CUDA {caps.cuda_runtime_version}, "
             f"driver {caps.driver_version}, NCCL {caps.nccl_version} [{caps.source}]"]
    for i, (n, c, m) in enumerate(zip(caps.device_names, caps.compute_capabilities,
                                      caps.total_memory_bytes)):
        lines.append(f"  cuda:{i} {n} sm_{c[0]}{c[1]} {m / 2**30:.1f} GiB")
    if not caps.device_count:
        lines.append(f"  no CUDA devices; accelerator={caps.accelerator}")
    if topology:
        lines.append(topology)
    return "\n".join(lines)


def environment_payload(caps: Optional[Capabilities] = None, topology: bool = True) -> dict[str, Any]:
    """Machine description to embed in every result JSON."""
    caps = caps or Capabilities.detect()
    out = {"capabilities": caps.to_dict(),
           "env": {k: os.environ[k] for k in ("CUDA_VISIBLE_DEVICES", "NCCL_DEBUG", "NCCL_NVLS_ENABLE",
                                              "WORLD_SIZE") if k in os.environ}}
    if topology and caps.source == "detected" and caps.device_count:
        out["topology"] = nvidia_smi("topo", "-m")
    return out


def nvidia_smi(*args: str, timeout: float = 20.0) -> Optional[str]:
    """Run ``nvidia-smi`` with query-only arguments; None when unavailable."""
    exe = shutil.which("nvidia-smi")
    if exe is None:
        return None
    try:
        res = subprocess.run([exe, *args], capture_output=True, text=True, timeout=timeout)
    except (OSError, subprocess.TimeoutExpired):
        return None
    return res.stdout if res.returncode == 0 else None


def set_visible_device(device: str) -> torch.device:
    """Bind this process to ``device`` BEFORE any process group is opened (so
    NCCL does not guess); returns the torch device."""
    dev = torch.device(device)
    if dev.type == "cuda":
        if not torch.cuda.is_available():
            raise HardwareError(f"asked for {device} but CUDA is unavailable")
        torch.cuda.set_device(dev)
    return dev


def synchronize(device) -> None:
    dev = torch.device(device)
    if dev.type == "cuda" and torch.cuda.is_available():
        torch.cuda.synchronize(dev)
