"""The restructured decode attention kernel (``decode_set_impl(2)``: four
cached positions a warp on 16-byte vectors) against a plain PyTorch fp32
reference of the same step and against the default kernel: the attention
output for multi-head, grouped and multi-query heads at cache lengths that
start, fill and straddle 64-position splits, and the fused key/value append.

This kernel has not yet run on a GPU; until it has, the test runs only when
G2B_DECODE_V2_GPU=1 is set, so that a default GPU-tier run never executes it
first."""

import os

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("G2B_DECODE_V2_GPU") != "1",
                                 reason="decode kernel 2: set G2B_DECODE_V2_GPU=1 to run")]

from gpt2_harness_b200.ops import native as N  # noqa: E402


def _reference(qkv, kc, vc, lens, H, Hkv, scale):
    B = qkv.shape[0]
    G = H // Hkv
    out = torch.zeros(B, H * 64)
    q = qkv[:, :H * 64].float().view(B, H, 64)
    kn = qkv[:, H * 64:(H + Hkv) * 64].float().view(B, Hkv, 64)
    vn = qkv[:, (H + Hkv) * 64:].float().view(B, Hkv, 64)
    for b in range(B):
        n = int(lens[b])
        for h in range(H):
            j = h // G
            K = torch.cat([kc[b, j, :n].float(), kn[b, j][None]], 0)
            V = torch.cat([vc[b, j, :n].float(), vn[b, j][None]], 0)
            p = torch.softmax(K @ q[b, h] * scale, 0)
            out[b, h * 64:(h + 1) * 64] = p @ V
    return out


@pytest.mark.parametrize("H,Hkv", [(12, 12), (12, 4), (12, 3), (8, 2)])
def test_decode_kernel2_matches_reference_and_kernel1(H, Hkv):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N.error_word().zero_()
    B, Tmax = 6, 300
    lens_h = torch.tensor([0, 1, 63, 64, 200, Tmax - 1], dtype=torch.int32)
    g = torch.Generator().manual_seed(H * 10 + Hkv)
    qkv = torch.randn(B, (H + 2 * Hkv) * 64, generator=g).bfloat16()
    kc0 = torch.randn(B, Hkv, Tmax, 64, generator=g).bfloat16()
    vc0 = torch.randn(B, Hkv, Tmax, 64, generator=g).bfloat16()
    scale = 0.125
    ref = _reference(qkv, kc0, vc0, lens_h, H, Hkv, scale)
    S = (Tmax + 63) // 64
    outs, caches = {}, {}
    L = N.lib()
    try:
        for impl in (1, 2):
            L.decode_set_impl(impl)
            assert L.decode_get_impl() == impl
            kc, vc = kc0.to(dev), vc0.to(dev)
            part_o = torch.empty(B * H * S * 64, device=dev)
            part_ml = torch.empty(B * H * S * 2, device=dev)
            out = torch.empty(B, H * 64, device=dev, dtype=torch.bfloat16)
            N.decode_attn(qkv.to(dev), kc, vc, lens_h.to(dev), part_o, part_ml, out, H, Hkv, scale)
            torch.cuda.synchronize()
            N.check_errors()
            outs[impl] = out.float().cpu()
            caches[impl] = (kc.cpu(), vc.cpu())
    finally:
        L.decode_set_impl(1)
    for impl in (1, 2):
        err = ((outs[impl] - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-2, (impl, err)
    # same bf16 rounding point, different fp32 summation order
    assert ((outs[2] - outs[1]).abs().max() / ref.abs().max()).item() < 1e-2
    # the append: position lens[b] of every head holds this step's k / v
    for impl in (1, 2):
        kc, vc = caches[impl]
        for b in range(B):
            n = int(lens_h[b])
            kn = qkv[b, H * 64:(H + Hkv) * 64].view(Hkv, 64)
            vn = qkv[b, (H + Hkv) * 64:].view(Hkv, 64)
            assert torch.equal(kc[b, :, n], kn) and torch.equal(vc[b, :, n], vn)
            keep = [t for t in range(Tmax) if t != n]
            assert torch.equal(kc[b, :, keep], kc0[b, :, keep])
