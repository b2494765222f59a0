"""Per-kernel timing of the native sm_100a kernels at GPT-2 training shapes.

Each kernel is timed with CUDA events on the launching stream (warm-up, then
the mean of `iters` back-to-back launches, synchronised on both sides) and
reported against the measured peaks in MEASURED_PEAKS.json (cuBLAS bf16
GEMM burst, STREAM-style copy bandwidth): achieved TFLOP/s or GB/s and the
fraction "of measured". The same script is the small case used for ncu
captures (``--only <name> --iters 1``).

    python -m gpt2_harness_b200.perf.kernel_bench [--batch 16 --seq 1024] [--only attn_fwd]
    python -m gpt2_harness_b200.perf.kernel_bench --only cp_attn   # CP gathered vs streamed K/V
    python -m gpt2_harness_b200.perf.kernel_bench --only decode_attn_v2   # restructured decode kernel
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
    tgt = torch.randint(0, V, (M,), device=dev)
    lo = torch.empty(2, device=dev)
    cews = N.CEWorkspace(M, V, dev)
    # the whole fused lm_head + cross-entropy forward (GEMM with statistics
    # epilogue, row fold, gradient pass); against gemm_lm_head_fwd + cross_entropy
    add("lm_head_ce_fused", lambda: N.lm_head_cross_entropy(x, wte, logits, tgt, cews, lo, V),
        2.0 * M * V * C)
    # its three steps on their own
    add("gemm_lm_head_ce_stats", lambda: N.gemm(x, wte, logits[:, :V], epilogue=N.EPI_CE_STATS,
                                                ce=cews, ce_targets=tgt), 2.0 * M * V * C)
    Lb = N.lib()
    _st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    add("ce_combine", lambda: Lb.ce_combine(cews.stats.data_ptr(), cews.nparts, M, tgt.data_ptr(),
                                            cews.tgt_logit.data_ptr(), cews.lse.data_ptr(),
                                            cews.loss_rows.data_ptr(), _st()),
        bytes_=cews.nparts * M * 8)
    add("ce_grad", lambda: Lb.ce_grad(logits.data_ptr(), vp, M, V, cews.lse.data_ptr(), tgt.data_ptr(),
                                      0, _st()), bytes_=2 * M * vp * 2)

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
    rows_ = torch.empty(M, device=dev)
    add("cross_entropy", lambda: N.cross_entropy_fwd_bwd(logits, tgt, rows_, lo, V), bytes_=3 * M * vp * 2)
    n = 124_439_808
    p = torch.zeros(n, device=dev)
    gg = torch.zeros(n, device=dev)
    m1 = torch.zeros(n, device=dev)
    v1 = torch.zeros(n, device=dev)
    pb = torch.empty(n, device=dev, dtype=bf)
    hp = torch.tensor([3e-4, 0.9, 0.95, 1e-8, 0.1, 0.1, 0.1, 1.0], device=dev)
    add("adamw", lambda: N.adamw_step(p, gg, m1, v1, pb, n, hp), bytes_=n * (4 * 7 + 2))
    # KV-cached decode attention: 32 sequences x H heads x 1000 cached positions
    Bd, Td, pos = 32, 1024, 1000
    qkv_d = torch.randn(Bd, 3 * H * 64, device=dev).to(bf)
    kc_d = torch.randn(Bd, H, Td, 64, device=dev).to(bf)
    vc_d = torch.randn(Bd, H, Td, 64, device=dev).to(bf)
    lens_d = torch.full((Bd,), pos, dtype=torch.int32, device=dev)
    Sd = (Td + 63) // 64
    po = torch.empty(Bd * H * Sd * 64, device=dev)
    pml = torch.empty(Bd * H * Sd * 2, device=dev)
    od = torch.empty(Bd, H * 64, device=dev, dtype=bf)
    kv_bytes = 2 * Bd * H * (pos + 1) * 64 * 2
    dec = lambda: N.decode_attn(qkv_d, kc_d, vc_d, lens_d, po, pml, od, H, H)  # noqa: E731
    add("decode_attn", dec, bytes_=kv_bytes)
    if only == "decode_attn_v2":  # the restructured kernel, timed only when named
        N.lib().decode_set_impl(2)
        try:
            add("decode_attn_v2", dec, bytes_=kv_bytes)
        finally:
            N.lib().decode_set_impl(1)
    _comm_kernels(add, dev, M, C)
    N.check_errors()
    return rows


def _comm_kernels(add, dev, M: int, C: int) -> None:
    """The peer-memory collectives at world 1 on this GPU (their handshakes
    reduce to this rank's own flags; the data path is the same code): what a
    one-GPU ncu capture of comm.cu, tp.cu and zero.cu kernels measures."""
    L = N.lib()
    err = N.error_word(dev).data_ptr()
    stream = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    epoch = [0]

    def nxt() -> int:
        epoch[0] += 1
        return epoch[0]

    ptrs = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device=dev)  # noqa: E731
    counter = torch.zeros(1, dtype=torch.int64, device=dev)
    # fused all-reduce (the wide kernel DDP uses): one 25 MiB fp32 bucket
    nb = 25 * 2**20 // 4
    bucket = torch.randn(nb, device=dev)
    cflags = torch.zeros(L.comm_flag_words(), dtype=torch.int32, device=dev)
    pb, pf = ptrs(bucket), ptrs(cflags)
    add("allreduce_p2p_w1",
        lambda: L.allreduce_p2p(pb.data_ptr(), pf.data_ptr(), 0, 1, 0, nb, 0, 1.0, nxt(),
                                counter.data_ptr(), err, 128, 2_000_000_000, -1, stream()),
        bytes_=nb * 4 * 2)
    # tensor-parallel reduce-scatter from the local inbox (+ bias + fp32 residual)
    inbox = torch.randn(M, C, device=dev).to(torch.bfloat16)
    bias = torch.zeros(C, device=dev, dtype=torch.bfloat16)
    resid = torch.randn(M, C, device=dev)
    out = torch.empty(M, C, device=dev)
    tflags = torch.zeros(L.tp_flag_words(), dtype=torch.int32, device=dev)
    pi, ptf = ptrs(inbox), ptrs(tflags)

    def tp_rs():
        L.tp_rs_rows({"peer_bufs": pi.data_ptr(), "peer_flags": ptf.data_ptr(), "rank": 0, "world": 1,
                      "rows": M, "cols": C, "nblocks": 128, "epoch": nxt(), "err": err,
                      "bias": bias.data_ptr(), "resid": resid.data_ptr(), "out_f32": out.data_ptr(),
                      "inbox": inbox.data_ptr()}, stream())

    add("tp_rs_rows_w1", tp_rs, bytes_=M * C * (2 + 4 + 4))
    # ZeRO-3 parameter gather: one GPT-2 small block (7.1M bf16 parameters)
    span = 7_087_872
    shard = torch.randn(span, device=dev).to(torch.bfloat16)
    dst = torch.empty(span, device=dev, dtype=torch.bfloat16)
    zflags = torch.zeros(L.zero_flag_words(), dtype=torch.int32, device=dev)
    ps, pzf = ptrs(shard), ptrs(zflags)
    zargs = {"peer_grad": 0, "peer_shadow": 0, "peer_flags": pzf.data_ptr(), "peer_norm": 0,
             "rank": 0, "world": 1, "buckets": 0, "nb": 0, "bucket": 0, "rs_blocks": 148, "gsh": 0,
             "master": 0, "exp_avg": 0, "exp_avg_sq": 0, "sumsq_parts": 0, "decay_ranges": 0,
             "nr": 0, "hp": 0, "max_norm": 0.0, "scale": 1.0, "epoch": 0,
             "byte_counter": counter.data_ptr(), "norm_out": 0, "err": err,
             "wait_budget_ns": 2_000_000_000, "done_handshake": 0, "peer_shard": ps.data_ptr(),
             "gather_dst": dst.data_ptr(), "ag_span": span, "ag_slice": span, "ag_offset": 0}

    def zero_ag():
        zargs["epoch"] = nxt()
        L.zero_ag(zargs, 148, stream())

    add("zero_ag_w1", zero_ag, bytes_=span * 2 * 2)


def run_cp_stream(world: int = 8, Tl: int = 2048, H: int = 20, batch: int = 1, iters: int = 20) -> list[dict]:
    """Context-parallel attention of one zig-zag rank (GPT-2 large widths,
    16k tokens over 8 ranks by default), forward and backward, with keys and
    values from a gathered natural-order buffer against streamed from their
    owners' compact buffers. The owners are emulated as separate buffers on
    this GPU, so the difference is the cost of the per-owner maps and publish
    waits, not NVLink. Run only when named (``--only cp_attn``)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    bf = torch.bfloat16
    pk = _peaks()
    C, T, h = H * 64, world * Tl, Tl // 2
    owners = [torch.randn(batch, Tl, 2 * C, device=dev).to(bf) for _ in range(world)]
    kvn = torch.empty(batch, T, 2 * C, device=dev, dtype=bf)
    for c in range(2 * world):
        q, r0 = (c, 0) if c < world else (2 * world - 1 - c, h)
        kvn[:, c * h:(c + 1) * h] = owners[q][:, r0:r0 + h]
    kvn = kvn.view(batch * T, 2 * C)
    flags = torch.ones(16, dtype=torch.int32, device=dev)
    peers = {"bases": [o.data_ptr() for o in owners], "sb": Tl * 2 * C, "st": 2 * C, "v_off": C, "Tl": Tl,
             "zigzag": 1, "flags": flags.data_ptr(), "epoch": 1}
    rank = 0
    spans = [(half * h, k * h, (k + 1) * h) for half, k in enumerate((rank, 2 * world - 1 - rank))]
    q = torch.randn(batch * Tl, C, device=dev).to(bf)
    dy = torch.randn(batch * Tl, C, device=dev).to(bf)
    o = torch.empty(batch * Tl, C, device=dev, dtype=bf)
    dq = torch.empty_like(o)
    lse = torch.empty(2, batch, H, h, device=dev)
    delta = torch.empty_like(lse)
    dkv = torch.empty(batch * T, 2 * C, device=dev, dtype=bf)
    # causal area of the two halves: queries of chunk k see keys [0, (k+1)h)
    area = sum(h * k0 + h * h / 2 for _, k0, _ in spans)
    fl = 4.0 * batch * H * area * 64

    def fwd(stream):
        for i, (r0, q0, Tk) in enumerate(spans):
            if stream:
                N.attention_fwd_peers(q[r0:], o[r0:], lse[i], batch, H, h, Tk, q0, peers, q_rows=Tl)
            else:
                N.attention_fwd(q[r0:], kvn[:, :C], kvn[:, C:], o[r0:], lse[i], batch, H, h, Tk=Tk, q_offset=q0,
                                kv_rows=T, q_rows=Tl)

    def bwd(stream):
        for i, (r0, q0, Tk) in enumerate(spans):
            if stream:
                N.attention_bwd_peers(q[r0:], o[r0:], dy[r0:], dq[r0:], dkv[:, :C], dkv[:, C:], lse[i], delta[i],
                                      batch, H, h, Tk, q0, peers, kv_rows=T, q_rows=Tl)
            else:
                N.attention_bwd(q[r0:], kvn[:, :C], kvn[:, C:], o[r0:], dy[r0:], dq[r0:], dkv[:, :C], dkv[:, C:],
                                lse[i], delta[i], batch, H, h, Tk=Tk, q_offset=q0, kv_rows=T, q_rows=Tl)

    rows = []
    for name, fn, f in (("cp_attn_fwd_gathered", lambda: fwd(False), fl),
                        ("cp_attn_fwd_streamed", lambda: fwd(True), fl),
                        ("cp_attn_bwd_gathered", lambda: bwd(False), 2.5 * fl),
                        ("cp_attn_bwd_streamed", lambda: bwd(True), 2.5 * fl)):
        ms = time_kernel(fn, iters=iters)
        tf = f / (ms * 1e-3) / 1e12
        rows.append({"kernel": name, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac": round(tf / pk["tflops"], 3), "peak": pk["label"]})
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
    if a.only and a.only.startswith("cp_attn"):
        rows = run_cp_stream(iters=a.iters)
    else:
        rows = run_suite(a.batch, a.seq, only=a.only, iters=a.iters)
    for r in rows:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
