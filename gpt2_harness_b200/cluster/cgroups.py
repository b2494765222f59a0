"""cgroup v2 limits of this process, and what each does to a training job.

Reference: src/transformer_internals/cluster/cgroups.py:106-232. Reads
``memory.max/high/current/swap.max/events``, ``cpu.max/stat`` and
``pids.max`` under the process's cgroup (never raising), and explains: the
memory.max wall is a SIGKILL from the cgroup OOM killer (the rank vanishes
with exit -9; ``memory.events`` oom_kill tells it from a hardware fault),
memory.high throttles into reclaim (slow steps, no crash), swap lets a rank
page while the others wait at the next collective, cpu.max throttles (looks
like a slow loader). The root directory is a parameter so tests can point
it at a fake tree.

    python -m gpt2_harness_b200.cluster.cgroups
"""

from __future__ import annotations

import platform
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Optional

__all__ = ["CgroupInfo", "read_cgroup", "report", "CGROUP_ROOT"]

CGROUP_ROOT = Path("/sys/fs/cgroup")


@dataclass
class CgroupInfo:
    available: bool
    reason: str = ""
    path: Optional[str] = None
    memory_max: Optional[str] = None
    memory_high: Optional[str] = None
    memory_current: Optional[str] = None
    memory_swap_max: Optional[str] = None
    memory_events: Optional[str] = None
    cpu_max: Optional[str] = None
    cpu_stat: Optional[str] = None
    pids_max: Optional[str] = None

    def to_dict(self) -> dict:
        return asdict(self)

    def events(self) -> dict[str, int]:
        out = {}
        for line in (self.memory_events or "").splitlines():
            k, _, v = line.partition(" ")
            if v.strip().isdigit():
                out[k] = int(v)
        return out


def _read(p: Path) -> Optional[str]:
    try:
        return p.read_text().strip()
    except OSError:
        return None


def _own_path(proc_cgroup: Path = Path("/proc/self/cgroup")) -> Optional[str]:
    txt = _read(proc_cgroup)
    for line in (txt or "").splitlines():
        if line.startswith("0::"):
            return line[3:] or "/"
    return None


def read_cgroup(root: Path = CGROUP_ROOT) -> CgroupInfo:
    root = Path(root)
    if not root.exists():
        return CgroupInfo(False, f"no {root} on this host ({platform.system()}); cgroups are a Linux feature")
    if not (root / "cgroup.controllers").exists():
        return CgroupInfo(False, f"{root} has no cgroup.controllers: cgroup v1 or a hybrid mount")
    g = lambda n: _read(root / n)  # noqa: E731
    return CgroupInfo(True, "", _own_path(), g("memory.max"), g("memory.high"), g("memory.current"),
                      g("memory.swap.max"), g("memory.events"), g("cpu.max"), g("cpu.stat"), g("pids.max"))


def _bytes(v: Optional[str]) -> str:
    if v is None:
        return "unreadable"
    if v == "max":
        return "max (no limit here; an ancestor or the host is the ceiling)"
    try:
        n = int(v)
        return f"{n} bytes ({n / 2 ** 30:.2f} GiB)"
    except ValueError:
        return v


def _cpu(v: Optional[str]) -> str:
    if not v:
        return "unreadable"
    q, _, per = v.partition(" ")
    if q == "max":
        return "max (unthrottled)"
    try:
        return f"{int(q)} us per {int(per)} us = {int(q) / int(per):.2f} CPUs (over quota -> throttled, not killed)"
    except ValueError:
        return v


def report(root: Path = CGROUP_ROOT) -> str:
    info = read_cgroup(root)
    w = []
    w.append("cgroup v2 limits for this process")
    w.append("=" * 60)
    if not info.available:
        w.append(f"NOT AVAILABLE: {info.reason}")
        return "\n".join(w)
    w += [f"cgroup path     : {info.path}", f"memory.max      : {_bytes(info.memory_max)}",
          f"memory.high     : {_bytes(info.memory_high)}", f"memory.current  : {_bytes(info.memory_current)}",
          f"memory.swap.max : {_bytes(info.memory_swap_max)}", f"pids.max        : {info.pids_max or 'unreadable'}",
          f"cpu.max         : {info.cpu_max or 'unreadable'}", f"                  {_cpu(info.cpu_max)}", ""]
    ev = info.events()
    w.append("memory.events: " + (", ".join(f"{k}={v}" for k, v in ev.items()) or "unreadable"))
    if ev.get("oom_kill", 0) > 0:
        w.append(f"  !! {ev['oom_kill']} OOM kill(s) in this cgroup: a rank that exited -9 was killed by the "
                 "cgroup OOM killer, not by a hardware or network fault")
    for line in (info.cpu_stat or "").splitlines():
        if line.startswith(("nr_throttled", "throttled_usec")):
            w.append(f"cpu.stat {line}" + ("   <- the CPU quota is being hit" if not line.endswith(" 0") else ""))
    try:
        cur = int(info.memory_current or 0)
        lim = int(info.memory_max) if info.memory_max not in (None, "max") else None
    except ValueError:
        cur, lim = 0, None
    if lim:
        w.append(f"headroom        : {(lim - cur) / 2 ** 20:.0f} MiB ({100 * cur / lim:.1f}% of memory.max used)")
    swap_off = info.memory_swap_max in ("0", None)
    w += ["", "What each wall does to a training job:",
          "  memory.max   SIGKILL by the cgroup OOM killer: no traceback, the launcher sees -9",
          "  memory.high  throttled into reclaim: slower steps, no crash",
          "  swap         " + ("off: an overshoot kills rather than pages (better for collective-synchronised "
                               "jobs)" if swap_off else "on: a rank pages at disk speed while the others wait at "
                                                       "the next collective; prefer swap off"),
          "  cpu.max      throttling, visible in cpu.stat; looks like a slow data loader"]
    return "\n".join(w)


if __name__ == "__main__":
    print(report())
