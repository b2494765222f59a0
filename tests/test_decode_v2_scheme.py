"""CPU check of the work split of the restructured decode attention kernel
(``decode_attn_v2_kernel`` in csrc/decode.cu), emulated lane by lane: four
warps of 32 lanes per 64-position split; lane l takes position slot l >> 3
and dims (l & 7) * 8 .. +8; warp w visits positions p0 + 4 w + slot + 16 t;
a score is folded over the 8 lanes of a slot with xor-shuffles 4, 2, 1 and
the P.V partials over the 4 slots of a warp with xor-shuffles 8, 16, then
summed over the warps. The emulation (same loop bounds, same shuffle
partners, same lanes writing) must give plain softmax attention for every
split length 1..64 and query groups of 1..4 heads: every position and every
dim is counted exactly once. It checks the scheme, not the compiled code."""

import numpy as np
import pytest

CHUNK = 64


def _shfl_xor(x, m):
    # x: [..., 32] per-lane values of one warp
    return x[..., np.arange(32) ^ m]


def _emulate_split(q, K, V, p0, p1, G):
    """One CTA: returns (m, l, o) per head of the group for positions [p0, p1)."""
    lanes = np.arange(32)
    slot, d0 = lanes >> 3, (lanes & 7) * 8
    p_s = np.zeros((G, CHUNK))
    for w in range(4):
        for pb in range(p0 + 4 * w, p1, 16):
            p = pb + slot                                   # [32]
            valid = p < p1
            kf = np.where(valid[:, None], K[np.minimum(p, p1 - 1)[:, None], d0[:, None] + np.arange(8)], 0.0)
            for g in range(G):
                s = (q[g][d0[:, None] + np.arange(8)] * kf).sum(1)   # per-lane partial over 8 dims
                for m in (4, 2, 1):
                    s = s + _shfl_xor(s, m)
                for l in lanes:
                    if valid[l] and (l & 7) == 0:
                        p_s[g, p[l] - p0] = s[l]
    n = p1 - p0
    ml = np.zeros((G, 2))
    for g in range(G):
        s = p_s[g, :n]
        m = s.max()
        e = np.exp2(s - m)
        p_s[g, :n] = e
        ml[g] = (m, e.sum())
    red = np.zeros((4, G, 64))
    for w in range(4):
        acc = np.zeros((G, 32, 8))
        for pb in range(p0 + 4 * w, p1, 16):
            p = pb + slot
            for l in lanes:
                if p[l] < p1:
                    vf = V[p[l], d0[l]:d0[l] + 8]
                    for g in range(G):
                        acc[g, l] += p_s[g, p[l] - p0] * vf
        for g in range(G):
            a = acc[g].T                                    # [8, 32]
            a = a + _shfl_xor(a, 8)
            a = a + _shfl_xor(a, 16)
            for l in lanes:
                if slot[l] == 0:
                    red[w, g, d0[l]:d0[l] + 8] = a[:, l]
    return ml, red.sum(0)


@pytest.mark.parametrize("G", [1, 2, 3, 4])
def test_work_split_is_plain_attention(G):
    rng = np.random.default_rng(G)
    T = 2 * CHUNK + 37          # three splits: full, full, 38 positions
    q = rng.standard_normal((G, 64))
    K = rng.standard_normal((T, 64))
    V = rng.standard_normal((T, 64))
    # per split, then the combine of decode_combine_kernel
    parts = []
    for p0 in range(0, T, CHUNK):
        parts.append(_emulate_split(q, K, V, p0, min(p0 + CHUNK, T), G))
    for g in range(G):
        m = max(ml[g, 0] for ml, _ in parts)
        l = sum(ml[g, 1] * np.exp2(ml[g, 0] - m) for ml, _ in parts)
        o = sum(red[g] * np.exp2(ml[g, 0] - m) for ml, red in parts) / l
        s = K @ q[g]
        p = np.exp2(s - s.max())
        want = (p / p.sum()) @ V
        assert np.allclose(o, want, rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("n", [1, 3, 8, 15, 16, 17, 33, 63, 64])
def test_every_split_length(n):
    rng = np.random.default_rng(n)
    q = rng.standard_normal((2, 64))
    K = rng.standard_normal((n, 64))
    V = rng.standard_normal((n, 64))
    ml, o = _emulate_split(q, K, V, 0, n, 2)
    for g in range(2):
        s = K @ q[g]
        e = np.exp2(s - s.max())
        assert np.isclose(ml[g, 0], s.max()) and np.isclose(ml[g, 1], e.sum())
        assert np.allclose(o[g], e @ V, rtol=1e-10, atol=1e-12)
