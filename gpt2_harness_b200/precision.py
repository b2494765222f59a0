"""Mixed-precision policy.

Same decision table as the reference (src/transformer_internals/precision.py:
90-307): bf16 autocast needs no loss scaler; fp16 gets a GradScaler; master
weights and optimizer state stay fp32 on every path; MPS stays fp32; requests a
device cannot honour are refused with a sentence instead of silently degraded.
The reduction dtype of a gradient collective is a separate knob
(:func:`reduce_dtype_of`).

On B200 the native engine always computes with bf16 matmul inputs, fp32
accumulation, an fp32 residual stream and fp32 master weights, i.e. the
``bf16`` policy; :func:`native_policy` states that explicitly for result files.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Any, Optional

import torch

from gpt2_harness_b200.hardware import Capabilities, HardwareError

__all__ = [
    "AMP_DTYPES",
    "REDUCE_DTYPES",
    "AmpPolicy",
    "autocast_context",
    "make_grad_scaler",
    "master_weight_report",
    "native_policy",
    "reduce_dtype_of",
    "resolve_amp",
]

AMP_DTYPES: dict[str, torch.dtype] = {"bf16": torch.bfloat16, "fp16": torch.float16}
REDUCE_DTYPES: dict[str, torch.dtype] = {"fp32": torch.float32, "bf16": torch.bfloat16,
                                         "fp16": torch.float16}


def reduce_dtype_of(name) -> torch.dtype:
    """Resolve a reduction dtype from its config spelling (None -> fp32)."""
    if name is None:
        return torch.float32
    if isinstance(name, torch.dtype):
        return name
    if name not in REDUCE_DTYPES:
        raise ValueError(f"unknown reduction dtype {name!r}; expected one of {sorted(REDUCE_DTYPES)}")
    return REDUCE_DTYPES[name]


@dataclass(frozen=True)
class AmpPolicy:
    """Resolved mixed-precision decision for one run, with its reason."""

    enabled: bool
    device_type: str
    dtype: Optional[torch.dtype]
    needs_scaler: bool
    reason: str
    master_dtype: torch.dtype = torch.float32

    @property
    def name(self) -> str:
        if not self.enabled or self.dtype is None:
            return "fp32"
        return {torch.bfloat16: "bf16", torch.float16: "fp16"}[self.dtype]

    def to_dict(self) -> dict[str, Any]:
        return {"enabled": self.enabled, "compute_dtype": self.name,
                "master_weight_dtype": str(self.master_dtype).replace("torch.", ""),
                "device_type": self.device_type, "grad_scaler": self.needs_scaler,
                "reason": self.reason}


def resolve_amp(enabled: bool, dtype: str = "bf16", device="cpu",
                caps: Optional[Capabilities] = None) -> AmpPolicy:
    """Mixed-precision policy for `device`, or HardwareError with the fix."""
    dev = torch.device(device)
    if not enabled:
        return AmpPolicy(False, dev.type, None, False, "autocast off, everything in fp32")
    if dtype not in AMP_DTYPES:
        raise ValueError(f"unknown amp dtype {dtype!r}; expected one of {sorted(AMP_DTYPES)}")
    want = AMP_DTYPES[dtype]
    if dev.type == "mps":
        return AmpPolicy(False, "mps", None, False,
                         "MPS: autocast is refused and the run stays fp32, so it stays comparable "
                         "with its fp32 baseline")
    if dev.type == "cuda":
        if want is torch.bfloat16:
            caps = caps if caps is not None else Capabilities.detect()
            if not caps.bf16_supported:
                names = ", ".join(f"sm_{a}{b}" for a, b in caps.compute_capabilities) or "unknown"
                raise HardwareError(f"bf16 autocast needs compute capability >= 8.0; this node "
                                    f"reports {names}. Use amp_dtype='fp16' or amp=False.")
            return AmpPolicy(True, "cuda", torch.bfloat16, False,
                             "bf16 autocast, fp32 master weights, no GradScaler (bf16 has "
                             "fp32's exponent range)")
        return AmpPolicy(True, "cuda", torch.float16, True,
                         "fp16 autocast, fp32 master weights, dynamic loss scaling")
    if dev.type == "cpu":
        if want is torch.float16:
            raise HardwareError("fp16 autocast with a GradScaler is CUDA-only; use "
                                "amp_dtype='bf16' on CPU or run on a GPU")
        return AmpPolicy(True, "cpu", torch.bfloat16, False,
                         "bf16 autocast on CPU with fp32 master weights (same numerics as CUDA)")
    raise HardwareError(f"no mixed-precision policy for device type {dev.type!r}")


def native_policy() -> AmpPolicy:
    """The fixed policy of the native B200 engine."""
    return AmpPolicy(True, "cuda", torch.bfloat16, False,
                     "native engine: bf16 matmul operands, fp32 accumulation, fp32 residual "
                     "stream and LayerNorm statistics, fp32 master weights and AdamW state")


def autocast_context(policy: AmpPolicy):
    if not policy.enabled or policy.dtype is None:
        return contextlib.nullcontext()
    return torch.autocast(device_type=policy.device_type, dtype=policy.dtype)


def make_grad_scaler(policy: AmpPolicy):
    """A GradScaler when the policy needs one (fp16), else None."""
    if not policy.needs_scaler:
        return None
    return torch.amp.GradScaler(policy.device_type)


def master_weight_report(model: torch.nn.Module) -> dict[str, Any]:
    """Parameter bytes by dtype: evidence that master weights stayed fp32."""
    by: dict[str, int] = {}
    for p in model.parameters():
        k = str(p.dtype).replace("torch.", "")
        by[k] = by.get(k, 0) + p.numel() * p.element_size()
    total = sum(by.values()) or 1
    return {"bytes_by_dtype": by, "fp32_fraction": by.get("float32", 0) / total}
