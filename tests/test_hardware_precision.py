"""Placement and mixed-precision decisions on fabricated machines (CPU).

Reference behaviour: src/transformer_internals/hardware.py (stub machines,
backend selection that refuses impossible requests instead of downgrading,
no oversubscription by default) and precision.py (bf16 needs sm >= 80 and no
scaler, fp16 gets a GradScaler and is CUDA-only, MPS stays fp32, master
weights stay fp32).
"""

import pytest
import torch

from gpt2_harness_b200.hardware import (Capabilities, HardwareError, check_placement, describe,
                                        environment_payload, native_kernels_supported, select_backend,
                                        select_device)
from gpt2_harness_b200.precision import (AmpPolicy, autocast_context, make_grad_scaler,
                                         master_weight_report, native_policy, reduce_dtype_of, resolve_amp)

B200 = Capabilities.stub(8)
A100 = Capabilities.stub(4, name="NVIDIA A100", capability=(8, 0))
V100 = Capabilities.stub(2, name="Tesla V100", capability=(7, 0))
CPU_ONLY = Capabilities(cuda_available=False, device_count=0, nccl_available=False, gloo_available=True,
                        source="stub")


def test_stub_machine_properties():
    assert B200.source == "stub" and B200.device_count == 8
    assert B200.bf16_supported and B200.is_blackwell and B200.accelerator == "cuda"
    assert A100.bf16_supported and not A100.is_blackwell
    assert not V100.bf16_supported
    assert not CPU_ONLY.bf16_supported and CPU_ONLY.accelerator == "cpu"
    d = B200.to_dict()
    assert d["is_blackwell"] and d["bf16_supported"] and d["accelerator"] == "cuda"
    assert native_kernels_supported(B200) and not native_kernels_supported(A100)


def test_backend_selection_refuses_rather_than_downgrades():
    assert select_backend(B200) == "nccl"
    assert select_backend(B200, "auto") == "nccl"
    assert select_backend(CPU_ONLY) == "gloo"
    assert select_backend(B200, "gloo") == "gloo"
    with pytest.raises(HardwareError, match="no CUDA device"):
        select_backend(CPU_ONLY, "nccl")
    with pytest.raises(HardwareError, match="unknown backend"):
        select_backend(B200, "mpi")
    no_nccl = Capabilities(cuda_available=True, device_count=2, nccl_available=False,
                           compute_capabilities=((10, 0),) * 2, source="stub")
    with pytest.raises(HardwareError, match="no NCCL"):
        select_backend(no_nccl, "nccl")
    no_gloo = Capabilities(gloo_available=False, source="stub")
    with pytest.raises(HardwareError, match="no gloo"):
        select_backend(no_gloo, "gloo")


def test_placement():
    assert check_placement(B200, 8, "nccl") == [f"cuda:{r}" for r in range(8)]
    assert check_placement(B200, 3, "gloo") == ["cpu"] * 3
    with pytest.raises(HardwareError, match="exceeds the 2 visible"):
        check_placement(V100, 4, "nccl")
    assert check_placement(V100, 4, "nccl", allow_oversubscribe=True) == ["cuda:0", "cuda:1"] * 2
    with pytest.raises(HardwareError, match="zero visible"):
        check_placement(CPU_ONLY, 1, "nccl")
    with pytest.raises(HardwareError, match="at least 1"):
        check_placement(B200, 0, "nccl")
    assert select_device(B200, 11, "nccl") == "cuda:3"
    with pytest.raises(HardwareError):
        select_device(CPU_ONLY, 0, "nccl")


def test_describe_and_payload():
    text = describe(B200, topology="GPU0 NV18")
    assert "sm_100" in text and "NVIDIA B200" in text and "GPU0 NV18" in text
    assert "no CUDA devices" in describe(CPU_ONLY)
    env = environment_payload(B200)
    assert env["capabilities"]["device_count"] == 8 and "topology" not in env  # stubs are never probed


def test_amp_decision_table():
    off = resolve_amp(False, device="cuda", caps=B200)
    assert not off.enabled and off.name == "fp32" and not off.needs_scaler
    bf = resolve_amp(True, "bf16", "cuda", caps=B200)
    assert bf.enabled and bf.dtype is torch.bfloat16 and not bf.needs_scaler and bf.name == "bf16"
    fp = resolve_amp(True, "fp16", "cuda", caps=V100)
    assert fp.needs_scaler and fp.name == "fp16"
    with pytest.raises(HardwareError, match="compute capability >= 8.0"):
        resolve_amp(True, "bf16", "cuda", caps=V100)
    mps = resolve_amp(True, "bf16", "mps")
    assert not mps.enabled and mps.name == "fp32"
    cpu = resolve_amp(True, "bf16", "cpu")
    assert cpu.enabled and cpu.dtype is torch.bfloat16
    with pytest.raises(HardwareError, match="CUDA-only"):
        resolve_amp(True, "fp16", "cpu")
    with pytest.raises(ValueError):
        resolve_amp(True, "fp8", "cuda", caps=B200)
    for pol in (off, bf, fp, mps, cpu, native_policy()):
        assert pol.master_dtype is torch.float32
        assert pol.to_dict()["master_weight_dtype"] == "float32"


def test_scaler_autocast_and_reduce_dtypes():
    assert make_grad_scaler(resolve_amp(True, "bf16", "cpu")) is None
    assert make_grad_scaler(AmpPolicy(True, "cuda", torch.float16, True, "fp16")) is not None
    with autocast_context(resolve_amp(True, "bf16", "cpu")):
        y = torch.nn.Linear(4, 4)(torch.randn(2, 4))
    assert y.dtype is torch.bfloat16
    with autocast_context(resolve_amp(False)):
        y = torch.nn.Linear(4, 4)(torch.randn(2, 4))
    assert y.dtype is torch.float32
    assert reduce_dtype_of(None) is torch.float32
    assert reduce_dtype_of("bf16") is torch.bfloat16
    assert reduce_dtype_of(torch.float16) is torch.float16
    with pytest.raises(ValueError):
        reduce_dtype_of("int8")


def test_master_weight_report():
    m = torch.nn.Sequential(torch.nn.Linear(4, 4), torch.nn.Linear(4, 4).to(torch.bfloat16))
    rep = master_weight_report(m)
    assert rep["bytes_by_dtype"] == {"float32": 80, "bfloat16": 40}
    assert rep["fp32_fraction"] == pytest.approx(80 / 120)
