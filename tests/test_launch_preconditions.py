"""Host-side launch preconditions of the native kernels (CPU).

Every launcher validates shapes, alignment and group sizes before anything
reaches the device and returns an error code that the binding turns into a
RuntimeError naming the op. Each case below is rejected by the launcher's
first check, so no kernel is launched (the pointers are never dereferenced)
whether or not a GPU is present.
"""

import pytest

from gpt2_harness_b200.ops import native as N

try:
    L = N.lib()
except ImportError:  # pragma: no cover - extension not built
    L = None

pytestmark = pytest.mark.skipif(L is None, reason="native extension not built")

A16 = 1 << 20  # a 16-byte-aligned address that is never dereferenced


def _rejected(fn, *args, name):
    with pytest.raises(RuntimeError, match=rf"{name} failed \(code -"):
        fn(*args)


def test_gemm_rejects_empty_and_bad_tile():
    # M = 0
    # trailing: pair, ce_stats, ce_targets, ce_tgt_logit, ce_vocab_offset, owner_out,
    # owner_rows, owner_self, err, stream
    tail = (-1, 0, 0, 0, 0, 0, 0, -1, 0, 0)
    _rejected(L.gemm, A16, 64, 0, A16, 64, 0, 0, 64, 64, 0, A16, 64, 0, 0, 0, 1.0, 0, 0, 1, 0, 256, 0,
              *tail, name="gemm_bf16")
    # unsupported N tile
    _rejected(L.gemm, A16, 64, 0, A16, 64, 0, 128, 128, 64, 0, A16, 128, 0, 0, 0, 1.0, 0, 0, 1, 0, 96,
              0, *tail, name="gemm_bf16")


def test_norm_and_embedding_shapes():
    # LayerNorm width not a multiple of 4
    # (the three zeros before the stream: no row push)
    _rejected(L.layernorm_fwd, A16, 6, A16, A16, A16, 6, A16, A16, 8, 6, 1e-5, 0, 0, 0, 0,
              name="layernorm_fwd")
    _rejected(L.layernorm_bwd, A16, A16, A16, A16, A16, A16, 0, A16, A16, A16, 0, 0, 768, 0, 0, 0,
              0, 0, 0, 0, name="layernorm_bwd")
    # embedding: position split outside the sequence, negative offsets
    _rejected(L.embedding_fwd, A16, A16, A16, A16, 2, 16, 64, 0, 17, 0, 0, name="embedding_fwd")
    _rejected(L.embedding_bwd, A16, A16, A16, A16, 2, 16, 64, 100, -1, 16, 0, 0, 0, 0,
              name="embedding_bwd")


def test_loss_and_optimizer_alignment():
    # logits row stride must keep 16-byte rows
    _rejected(L.cross_entropy, A16, 50257, A16, A16, 4, 50257, 0, 0, name="cross_entropy")
    # AdamW buffers must be 16-byte aligned
    _rejected(L.adamw, A16 + 4, A16, A16, A16, 0, 1024, 0, 0, 0, A16, 0, 0, name="adamw")


def test_collective_group_limits():
    # all-reduce over more ranks than one NVSwitch domain holds
    _rejected(L.allreduce_p2p, A16, A16, 0, 9, 0, 1024, 0, 1.0, 1, 0, 0, 64, 10**9, -1, 0,
              name="allreduce_p2p")
    # misaligned bucket start (fp32 offset of 3 elements)
    _rejected(L.allreduce_p2p, A16, A16, 0, 2, 3, 1024, 0, 1.0, 1, 0, 0, 64, 10**9, -1, 0,
              name="allreduce_p2p")
    # multimem form: no multicast address, bucket not whole 16-byte vectors
    _rejected(L.allreduce_mc, A16, A16, 0, 0, 2, 0, 1024, 0, 1.0, 1, 0, 0, 64, 10**9, -1, 0,
              name="allreduce_mc")
    _rejected(L.allreduce_mc, A16, A16, A16, 0, 2, 0, 1022, 0, 1.0, 1, 0, 0, 64, 10**9, -1, 0,
              name="allreduce_mc")
    base = {"peer_bufs": A16, "peer_flags": A16, "rank": 0, "cols": 16, "B": 1, "Tl": 2,
            "src": A16, "src_ld": 8, "out_bf16": A16}
    # context-parallel gather / reduce: group too large, odd zig-zag length,
    # zig-zag reduce without the second partial buffer
    _rejected(L.cp_kv_gather, dict(base, world=9), 0, name="cp_kv_gather")
    _rejected(L.cp_kv_gather, dict(base, world=2, Tl=3, zigzag=1), 0, name="cp_kv_gather")
    _rejected(L.cp_kv_reduce, dict(base, world=2, zigzag=1), 0, name="cp_kv_reduce")
    # streaming publish: group too large, odd zig-zag length, rows not whole 16-byte vectors
    _rejected(L.cp_kv_publish, dict(base, world=9), 0, name="cp_kv_publish")
    _rejected(L.cp_kv_publish, dict(base, world=2, Tl=3, zigzag=1), 0, name="cp_kv_publish")
    _rejected(L.cp_kv_publish, dict(base, world=2, cols=12), 0, name="cp_kv_publish")
    # tensor-parallel row gather with a row length that is not whole 16-byte vectors
    _rejected(L.tp_ag_rows, {"peer_bufs": A16, "peer_flags": A16, "rank": 0, "world": 2,
                             "rows": 4, "cols": 12}, 0, name="tp_ag_rows")


def _peer_attn_args(bases, B=1, H=2, Tq=128, Tk=256):
    # q, o, q strides, o strides, lse, B, H, Hkv, Tq, Tk, q_offset, scale,
    # owner bases, kv strides, v_off, Tl, zigzag, flags, epoch, err, stream
    return (A16, A16, 128 * 128, 128, 64, 128 * 128, 128, 64, A16, B, H, H, Tq, Tk, 128, 0.125, bases,
            128 * 256, 256, 128, 128, 0, A16, 1, 0, 0)


def test_streamed_attention_preconditions():
    # one to eight owners
    with pytest.raises(RuntimeError, match="1 to 8 owner buffers"):
        L.attn_fwd_peers(*_peer_attn_args([A16] * 9))
    with pytest.raises(RuntimeError, match="1 to 8 owner buffers"):
        L.attn_fwd_peers(*_peer_attn_args([]))
    # no mma.sync fallback for keys read from their owners
    L.attn_set_impl(1)
    try:
        _rejected(L.attn_fwd_peers, *_peer_attn_args([A16, A16]), name="attn_fwd_peers")
    finally:
        L.attn_set_impl(0)
    # empty problem
    _rejected(L.attn_fwd_peers, *_peer_attn_args([A16, A16], Tq=0), name="attn_fwd_peers")
