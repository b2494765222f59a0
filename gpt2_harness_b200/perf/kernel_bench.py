"""Per-kernel timing of the native sm_100a kernels at GPT-2 training shapes.

Each kernel is timed with CUDA events on the launching stream (warm-up, then
the mean of `iters` back-to-back launches, synchronised on both sides) and
reported against the measured peaks in MEASURED_PEAKS.json (cuBLAS bf16
GEMM burst, STREAM-style copy bandwidth): achieved TFLOP/s or GB/s and the
fraction "of measured". The same script is the small case used for ncu
captures (``--only <name> --iters 1``).

    python -m gpt2_harness_b200.perf.kernel_bench [--batch 16 --seq 1024] [--only attn_fwd]
"""

from __future__ import annotations

import argparse
import json
import math
import os
from typing import Callable

import torch

from gpt2_harness_b200.ops import native as N

__all__ = ["time_kernel", "run_suite"]


def _peaks() -> dict:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"tflops": float(d["bf16_tflops"]), "gbs": float(d["hbm_gbs"]), "label": "of measured"}
    except (OSError, KeyError, ValueError):
        return {"tflops": 1590.0, "gbs": 6650.0, "label": "of fallback"}


def time_kernel(fn: Callable[[], None], iters: int = 20, warmup: int = 3) -> float:
    """Mean milliseconds per call (CUDA events, synchronised both sides)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def run_suite(batch: int = 16, seq: int = 1024, C: int = 768, H: int = 12, V: int = 50257,
              only: str | None = None, iters: int = 20) -> list[dict]:
    dev = torch.device("cuda", torch.cuda.current_device())
    M = batch * seq
    bf = torch.bfloat16
    pk = _peaks()
    rows = []

    def add(name, fn, flops=0.0, bytes_=0.0):
        if only and only not in name:
            return
        ms = time_kernel(fn, iters=iters)
        r = {"kernel": name, "ms": round(ms, 4)}
        if flops:
            tf = flops / (ms * 1e-3) / 1e12
            r.update(tflops=round(tf, 1), frac=round(tf / pk["tflops"], 3))
        if bytes_:
            gb = bytes_ / (ms * 1e-3) / 1e9
            r.update(gbs=round(gb, 1), bw_frac=round(gb / pk["gbs"], 3))
        r["peak"] = pk["label"]
        rows.append(r)

    x = torch.randn(M, C, device=dev).to(bf)
    w_attn = (torch.randn(3 * C, C, device=dev) * 0.02).to(bf)
    w_fc = (torch.randn(4 * C, C, device=dev) * 0.02).to(bf)
    w_proj = (torch.randn(C, 4 * C, device=dev) * 0.02).to(bf)
    b3 = torch.zeros(3 * C, device=dev, dtype=bf)
    b4 = torch.zeros(4 * C, device=dev, dtype=bf)
    qkv = torch.empty(M, 3 * C, device=dev, dtype=bf)
    h4 = torch.empty(M, 4 * C, device=dev, dtype=bf)
    u4 = torch.empty(M, 4 * C, device=dev, dtype=bf)
    res = torch.randn(M, C, device=dev)
    res2 = torch.empty(M, C, device=dev)
    add("gemm_c_attn_fwd", lambda: N.gemm(x, w_attn, qkv, bias=b3), 2.0 * M * 3 * C * C)
    add("gemm_c_fc_fwd_gelu", lambda: N.gemm(x, w_fc, h4, epilogue=N.EPI_BIAS_GELU, bias=b4, aux=u4),
        2.0 * M * 4 * C * C)
    add("gemm_mlp_proj_fwd_resid", lambda: N.gemm(h4, w_proj, res2, epilogue=N.EPI_RESID_F32, aux=res),
        2.0 * M * 4 * C * C)
    dh = torch.empty(M, C, device=dev, dtype=bf)
    add("gemm_c_fc_dgrad", lambda: N.gemm(h4, w_fc, dh, b_t=True), 2.0 * M * 4 * C * C)
    add("gemm_mlp_proj_dgrad_gelu", lambda: N.gemm(x, w_proj, h4, b_t=True, epilogue=N.EPI_GELU_BWD, aux=u4),
        2.0 * M * 4 * C * C)
    gw = torch.empty(4 * C, C, device=dev)
    ws = torch.empty(16 * 4 * C * C, device=dev)
    from gpt2_harness_b200.models.engine import choose_splits
    s_fc = choose_splits(4 * C, C, M)
    add("gemm_c_fc_wgrad", lambda: N.gemm(h4, x, gw, a_t=True, b_t=True, epilogue=N.EPI_F32,
                                          splits=s_fc, workspace=ws), 2.0 * M * 4 * C * C)
    wte = (torch.randn(V, C, device=dev) * 0.02).to(bf)
    vp = (V + 63) // 64 * 64
    logits = torch.empty(M, vp, device=dev, dtype=bf)
    add("gemm_lm_head_fwd", lambda: N.gemm(x, wte, logits[:, :V]), 2.0 * M * V * C)

    # attention (causal: half the dense FLOPs)
    lse = torch.empty(batch, H, seq, device=dev)
    y = torch.empty(M, C, device=dev, dtype=bf)
    qkv.normal_()
    fl_fwd = 4.0 * batch * H * seq * seq * 64 / 2
    add("attn_fwd", lambda: N.attention_fwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], y, lse,
                                            batch, H, seq), fl_fwd)
    dy = torch.randn(M, C, device=dev).to(bf)
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(batch, H, seq, device=dev)
    add("attn_bwd", lambda: N.attention_bwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], y, dy,
                                            dqkv[:, :C], dqkv[:, C:2 * C], dqkv[:, 2 * C:], lse,
                                            delta, batch, H, seq), 2.5 * fl_fwd)
    # memory-bound kernels
    g = torch.ones(C, device=dev, dtype=bf)
    bb = torch.zeros(C, device=dev, dtype=bf)
    mean = torch.empty(M, device=dev)
    rstd = torch.empty(M, device=dev)
    add("layernorm_fwd", lambda: N.layernorm_fwd(res, g, bb, dh, mean, rstd), bytes_=M * C * (4 + 2))
    dres = torch.zeros(M, C, device=dev)
    dres16 = torch.empty(M, C, device=dev, dtype=bf)
    dg = torch.zeros(C, device=dev)
    db = torch.zeros(C, device=dev)
    parts = N.layernorm_bwd_partials(M, C, dev)
    add("layernorm_bwd", lambda: N.layernorm_bwd(dh, res, mean, rstd, g, dres, dres16, dg, db, parts, True),
        bytes_=M * C * (2 + 4 + 4 + 4 + 2))
    cws = torch.empty(N.colsum_ws_numel(M, 4 * C), device=dev)
    bg = torch.zeros(4 * C, device=dev)
    add("bias_grad_colsum", lambda: N.colsum_bf16(h4, bg, cws), bytes_=M * 4 * C * 2)
    tgt = torch.randint(0, V, (M,), device=dev)
    rows_ = torch.empty(M, device=dev)
    lo = torch.empty(2, device=dev)
    add("cross_entropy", lambda: N.cross_entropy_fwd_bwd(logits, tgt, rows_, lo, V), bytes_=3 * M * vp * 2)
    n = 124_439_808
    p = torch.zeros(n, device=dev)
    gg = torch.zeros(n, device=dev)
    m1 = torch.zeros(n, device=dev)
    v1 = torch.zeros(n, device=dev)
    pb = torch.empty(n, device=dev, dtype=bf)
    hp = torch.tensor([3e-4, 0.9, 0.95, 1e-8, 0.1, 0.1, 0.1, 1.0], device=dev)
    add("adamw", lambda: N.adamw_step(p, gg, m1, v1, pb, n, hp), bytes_=n * (4 * 7 + 2))
    N.check_errors()
    return rows


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--only", default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    rows = run_suite(a.batch, a.seq, only=a.only, iters=a.iters)
    for r in rows:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
