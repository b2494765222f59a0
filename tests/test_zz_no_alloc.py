"""The allocation-free bias-gradient entry point, called through its exported
C symbol the way a caller that cannot allocate device memory would call it,
against a plain PyTorch fp32 column sum and against the library's regular
(workspace-taking) column sum.

Collected last on purpose (file name), so a run that stops at the first
failure has already run every other test."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = -2


def _entry():
    from gpt2_harness_b200.ops import native as N

    so = ctypes.CDLL(N.lib().__file__)  # the already-loaded extension
    f = so.g2b_bias_grad_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_int, ctypes.c_void_p]
    return f, N


def test_no_alloc_bias_grad_matches_regular_entry_point():
    torch.cuda.set_device(0)
    f, N = _entry()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    M, C = 16384, 768  # GPT-2 small, 16 x 1024 tokens: 128 chunks x 768 <= 2^18 floats
    for call in range(2):  # two calls in a row share (and reuse) the scratch array
        torch.manual_seed(call)
        dy = torch.randn(M, C, device=dev).to(torch.bfloat16)
        want = torch.zeros(C, device=dev)
        ws = torch.empty(N.colsum_ws_numel(M, C), device=dev)
        N.colsum_bf16(dy, want, ws, accumulate=False)
        got = torch.full((C,), float("nan"), device=dev)
        rc = f(dy.data_ptr(), dy.stride(0), M, C, got.data_ptr(), 0, stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        err = ((got - want).abs().max() / (want.abs().max() + 1e-6)).item()
        assert err < 1e-5, (call, err)
        ref = dy.float().sum(0)  # fp32 reference of the same op
        err_ref = ((got - ref).abs().max() / (ref.abs().max() + 1e-6)).item()
        assert err_ref < 1e-5, (call, err_ref)
        # accumulate mode adds onto the existing output
        rc = f(dy.data_ptr(), dy.stride(0), M, C, got.data_ptr(), 1, stream.cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert ((got - 2 * want).abs().max() / (2 * want.abs().max() + 1e-6)).item() < 1e-5


def test_no_alloc_rejects_sizes_beyond_scratch():
    torch.cuda.set_device(0)
    f, _ = _entry()
    dev = torch.device("cuda", 0)
    dy = torch.zeros(8, 8, device=dev, dtype=torch.bfloat16)
    out = torch.full((8,), 7.0, device=dev)
    # claim a shape whose partials (ceil(M/128) * C) exceed the 2^18-float array
    rc = f(dy.data_ptr(), 4096, 1 << 20, 4096, out.data_ptr(), 0,
           torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
    torch.cuda.synchronize()
    assert torch.equal(out, torch.full((8,), 7.0, device=dev))  # nothing launched
