"""Diff two trees of result JSON and gate on the correctness invariants.

Reference: scripts/compare_results.py:1-391. Every leaf number of every JSON
under two roots is paired by its path (list elements keyed by a name / op /
arm field when they have one, so reordering does not misalign them) and
classified:

* exact invariants (byte counts, call counts, closed-form checks, bitwise
  resharding identity): must be identical, any change is a bug;
* tolerant invariants (equivalence errors, restart loss differences): must
  stay below ``EQUIVALENCE_TOLERANCE`` (1e-5) in the current tree, because
  float reductions differ across backends;
* timings: expected to move; reported as ratios;
* everything else: listed when it moved by more than a relative threshold.

Exit status is non-zero when an invariant broke, so CI can gate on it.

    python -m gpt2_harness_b200.compare_results --baseline /tmp/before --current results
    python -m gpt2_harness_b200.compare_results --baseline-git HEAD --current results
"""

from __future__ import annotations

import argparse
import json
import re
import subprocess
import sys
import tempfile
from pathlib import Path
from typing import Any, Optional

__all__ = ["EQUIVALENCE_TOLERANCE", "EXACT_INVARIANTS", "TOLERANT_INVARIANTS", "TIMING_PATTERNS", "flatten",
           "load_tree", "compare", "main"]

EQUIVALENCE_TOLERANCE = 1e-5
EXACT_INVARIANTS = [re.compile(p) for p in (r"checks(\[[^]]*\]|\.).*(measured|predicted|ok)$", r"\.payload_bytes(_per_step)?$",
                                            r"\.calls$", r"\.bitwise_identical$", r"closed_form.*$")]
TOLERANT_INVARIANTS = [re.compile(p) for p in (r"equivalence\..*error$", r"max_abs_loss_difference$")]
TIMING_PATTERNS = [re.compile(p) for p in (r"(seconds|_s|_ms|wall_clock|runtime|latency_us)$",
                                           r"(step_s|median_s|min_s|makespan_seconds|tokens_per_s)$")]


def _match(path: str, pats) -> bool:
    return any(p.search(path) for p in pats)


def _key(v: Any) -> Optional[str]:
    if isinstance(v, dict):
        for k in ("name", "arm", "op", "kernel", "label", "key"):
            if isinstance(v.get(k), (str, int)):
                extra = v.get("world_size", v.get("bytes", v.get("impl")))
                return f"{v[k]}" + (f"@{extra}" if extra is not None and k == "op" else "")
    return None


def flatten(obj: Any, prefix: str = "") -> dict[str, Any]:
    out: dict[str, Any] = {}
    if isinstance(obj, dict):
        for k, v in obj.items():
            out.update(flatten(v, f"{prefix}.{k}" if prefix else str(k)))
    elif isinstance(obj, list):
        keys = [_key(v) for v in obj]
        use = all(k is not None for k in keys) and len(set(keys)) == len(keys)
        for i, v in enumerate(obj):
            out.update(flatten(v, f"{prefix}[{keys[i] if use else i}]"))
    elif isinstance(obj, (int, float, bool)) or obj is None:
        out[prefix] = obj
    return out


def load_tree(root: Path) -> dict[str, Any]:
    leaves: dict[str, Any] = {}
    for f in sorted(Path(root).rglob("*.json")):
        try:
            data = json.loads(f.read_text())
        except (OSError, ValueError):
            continue
        for k, v in flatten(data).items():
            leaves[f"{f.relative_to(root)}:{k}"] = v
    return leaves


def git_baseline(ref: str, path: str) -> Path:
    """Materialise ``path`` at git ``ref`` into a temp directory."""
    tmp = Path(tempfile.mkdtemp(prefix="g2b_baseline_"))
    files = subprocess.run(["git", "ls-tree", "-r", "--name-only", ref, path], capture_output=True, text=True,
                           check=True).stdout.split()
    for f in files:
        if f.endswith(".json"):
            dst = tmp / Path(f).relative_to(path)
            dst.parent.mkdir(parents=True, exist_ok=True)
            dst.write_bytes(subprocess.run(["git", "show", f"{ref}:{f}"], capture_output=True, check=True).stdout)
    return tmp


def compare(base: dict, cur: dict, threshold: float = 0.05) -> dict[str, Any]:
    rep = {"exact_held": [], "exact_broken": [], "tolerant_held": [], "tolerant_broken": [], "timings": [],
           "moved": [], "missing": sorted(set(base) - set(cur)), "new": sorted(set(cur) - set(base))}
    for path in sorted(set(base) & set(cur)):
        a, b = base[path], cur[path]
        if _match(path, EXACT_INVARIANTS):
            (rep["exact_held"] if a == b else rep["exact_broken"]).append({"path": path, "baseline": a, "current": b})
        elif _match(path, TOLERANT_INVARIANTS):
            ok = isinstance(b, (int, float)) and b is not None and abs(b) <= EQUIVALENCE_TOLERANCE
            (rep["tolerant_held"] if ok else rep["tolerant_broken"]).append(
                {"path": path, "baseline": a, "current": b, "ratio": (b / a) if a else None})
        elif _match(path, TIMING_PATTERNS):
            if isinstance(a, (int, float)) and isinstance(b, (int, float)) and a:
                rep["timings"].append({"path": path, "baseline": a, "current": b, "ratio": b / a})
        elif isinstance(a, (int, float)) and isinstance(b, (int, float)) and not isinstance(a, bool):
            if a != b and abs(b - a) > threshold * max(abs(a), abs(b), 1e-30):
                rep["moved"].append({"path": path, "baseline": a, "current": b})
    rep["ok"] = not rep["exact_broken"] and not rep["tolerant_broken"]
    return rep


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    g = ap.add_mutually_exclusive_group(required=True)
    g.add_argument("--baseline")
    g.add_argument("--baseline-git")
    ap.add_argument("--current", default="results")
    ap.add_argument("--threshold", type=float, default=0.05)
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    base_root = Path(a.baseline) if a.baseline else git_baseline(a.baseline_git, a.current)
    rep = compare(load_tree(base_root), load_tree(Path(a.current)), a.threshold)
    print(f"CORRECTNESS INVARIANTS: {len(rep['exact_held'])} identical, {len(rep['exact_broken'])} broken; "
          f"{len(rep['tolerant_held'])} within {EQUIVALENCE_TOLERANCE:g}, {len(rep['tolerant_broken'])} over")
    for r in rep["exact_broken"] + rep["tolerant_broken"]:
        print(f"  BROKEN {r['path']}: {r['baseline']} -> {r['current']}")
    for r in sorted(rep["timings"], key=lambda r: r["ratio"])[:20]:
        print(f"  timing {r['path']}: x{r['ratio']:.3f}")
    print(f"{len(rep['moved'])} other values moved by more than {a.threshold:.0%}; "
          f"{len(rep['missing'])} missing, {len(rep['new'])} new")
    if a.json:
        Path(a.json).write_text(json.dumps(rep, indent=1, default=str))
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
