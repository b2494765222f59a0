"""Numerics of every native sm_100a kernel against a plain PyTorch fp32
reference of the same op (inputs rounded to bf16 first, math in fp32)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from gpt2_harness_b200.ops import native as N  # noqa: E402


def dev():
    return torch.device("cuda", 0)


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).abs().max() / (b.abs().max() + 1e-6)).item()


@pytest.fixture(autouse=True)
def _errors_clean():
    torch.cuda.set_device(0)
    N.error_word().zero_()
    yield
    torch.cuda.synchronize()
    N.check_errors()


# ------------------------------------------------------------------- GEMM --
SHAPES = [(128, 256, 64), (256, 512, 128), (200, 136, 72), (384, 768, 768), (1000, 520, 264)]


@pytest.mark.parametrize("M,Nn,K", SHAPES)
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("bn", [256, 128])
def test_gemm_layouts(M, Nn, K, a_t, b_t, bn):
    g = torch.Generator(device="cpu").manual_seed(M * 7 + Nn + K)
    A = torch.randn(M, K, generator=g).to(dev(), torch.bfloat16)
    B = torch.randn(Nn, K, generator=g).to(dev(), torch.bfloat16)
    a_in = A.t().contiguous() if a_t else A
    b_in = B.t().contiguous() if b_t else B
    out = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev())
    N.gemm(a_in, b_in, out, a_t=a_t, b_t=b_t, bn=bn)
    ref = A.float() @ B.float().t()
    assert rel_err(out, ref) < 1e-2


def test_gemm_bias_gelu_and_bwd():
    M, Nn, K = 512, 1024, 256
    A = torch.randn(M, K, device=dev()).bfloat16()
    W = (torch.randn(Nn, K, device=dev()) * 0.05).bfloat16()
    bias = torch.randn(Nn, device=dev()).bfloat16()
    pre = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev())
    act = torch.empty_like(pre)
    N.gemm(A, W, act, epilogue=N.EPI_BIAS_GELU, bias=bias, aux=pre)
    ref_pre = A.float() @ W.float().t() + bias.float()
    ref_act = 0.5 * ref_pre * (1 + torch.tanh(math.sqrt(2 / math.pi) * (ref_pre + 0.044715 * ref_pre**3)))
    assert rel_err(pre, ref_pre) < 1e-2
    assert rel_err(act, ref_act) < 1e-2
    # GELU backward epilogue: out = (G @ W2^T) * gelu'(pre)
    G = torch.randn(M, 256, device=dev()).bfloat16()
    W2 = (torch.randn(Nn, 256, device=dev()) * 0.05).bfloat16()
    dact = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev())
    N.gemm(G, W2, dact, epilogue=N.EPI_GELU_BWD, aux=pre)
    x = pre.float().requires_grad_(True)
    y = 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x**3)))
    up = G.float() @ W2.float().t()
    (gx,) = torch.autograd.grad(y, x, up)
    assert rel_err(dact, gx) < 2e-2


def test_gemm_resid_and_f32_accumulate_splitk():
    M, Nn, K = 768, 512, 2048
    A = torch.randn(M, K, device=dev()).bfloat16()
    B = torch.randn(Nn, K, device=dev()).bfloat16()
    bias = torch.randn(Nn, device=dev()).bfloat16()
    resid = torch.randn(M, Nn, device=dev())
    ref = resid + A.float() @ B.float().t() + bias.float()
    N.gemm(A, B, resid, epilogue=N.EPI_RESID_F32, bias=bias)
    assert rel_err(resid, ref) < 1e-4
    # wgrad style: both operands MN-major, fp32 out, accumulate, split-K 4
    X = torch.randn(K, M, device=dev()).bfloat16()   # [tokens, in]
    dY = torch.randn(K, Nn, device=dev()).bfloat16()  # [tokens, out]
    gw = torch.randn(Nn, M, device=dev())
    ref = gw + dY.float().t() @ X.float()
    ws = torch.empty(4 * Nn * M, device=dev())
    N.gemm(dY, X, gw, a_t=True, b_t=True, epilogue=N.EPI_F32, accumulate=True, splits=4, workspace=ws)
    assert rel_err(gw, ref) < 1e-4


def test_gemm_alpha_ptr():
    A = torch.randn(256, 128, device=dev()).bfloat16()
    B = torch.randn(256, 128, device=dev()).bfloat16()
    out = torch.empty(256, 256, device=dev())
    a = torch.tensor([0.25], device=dev())
    N.gemm(A, B, out, epilogue=N.EPI_F32, alpha=2.0, alpha_ptr=a)
    assert rel_err(out, 0.5 * (A.float() @ B.float().t())) < 1e-4


def test_gemm_large_vocab_shape():
    # lm_head-like: N not a multiple of the tile, padded row stride
    M, V, C = 512, 50257, 768
    ld = 50304
    x = torch.randn(M, C, device=dev()).bfloat16()
    w = (torch.randn(V, C, device=dev()) * 0.02).bfloat16()
    logits = torch.zeros(M, ld, dtype=torch.bfloat16, device=dev())
    N.gemm(x, w, logits[:, :V])
    ref = x.float() @ w.float().t()
    assert rel_err(logits[:, :V], ref) < 1e-2


# ------------------------------------------------- GEMM on CTA pairs (2-SM) --
PAIR_SHAPES = [(256, 256, 64), (512, 512, 128), (264, 136, 72), (768, 768, 768), (1000, 520, 264),
               (2048, 3072, 768)]


@pytest.mark.parametrize("M,Nn,K", PAIR_SHAPES)
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_pair_layouts(M, Nn, K, a_t, b_t):
    """256x256 tiles on CTA pairs (cta_group::2) against fp32 torch, and
    against the single-CTA kernel (same k order per output: equal to fp32
    rounding)."""
    g = torch.Generator(device="cpu").manual_seed(M * 5 + Nn + K)
    A = torch.randn(M, K, generator=g).to(dev(), torch.bfloat16)
    B = torch.randn(Nn, K, generator=g).to(dev(), torch.bfloat16)
    a_in = A.t().contiguous() if a_t else A
    b_in = B.t().contiguous() if b_t else B
    out = torch.empty(M, Nn, dtype=torch.float32, device=dev())
    N.gemm(a_in, b_in, out, a_t=a_t, b_t=b_t, epilogue=N.EPI_F32, pair=1)
    ref = A.float() @ B.float().t()
    assert rel_err(out, ref) < 1e-5
    single = torch.empty_like(out)
    N.gemm(a_in, b_in, single, a_t=a_t, b_t=b_t, epilogue=N.EPI_F32, pair=0)
    assert rel_err(out, single) < 1e-6


def test_gemm_pair_epilogues():
    M, Nn, K = 1280, 1024, 512
    A = torch.randn(M, K, device=dev()).bfloat16()
    W = (torch.randn(Nn, K, device=dev()) * 0.05).bfloat16()
    bias = torch.randn(Nn, device=dev()).bfloat16()
    pre = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev())
    act = torch.empty_like(pre)
    N.gemm(A, W, act, epilogue=N.EPI_BIAS_GELU, bias=bias, aux=pre, pair=1)
    ref_pre = A.float() @ W.float().t() + bias.float()
    ref_act = 0.5 * ref_pre * (1 + torch.tanh(math.sqrt(2 / math.pi) * (ref_pre + 0.044715 * ref_pre**3)))
    assert rel_err(pre, ref_pre) < 1e-2
    assert rel_err(act, ref_act) < 1e-2
    G = torch.randn(M, 256, device=dev()).bfloat16()
    W2 = (torch.randn(Nn, 256, device=dev()) * 0.05).bfloat16()
    dact = torch.empty(M, Nn, dtype=torch.bfloat16, device=dev())
    N.gemm(G, W2, dact, epilogue=N.EPI_GELU_BWD, aux=pre, pair=1)
    x = pre.float().requires_grad_(True)
    y = 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x**3)))
    (gx,) = torch.autograd.grad(y, x, G.float() @ W2.float().t())
    assert rel_err(dact, gx) < 2e-2
    resid = torch.randn(M, Nn, device=dev())
    ref = resid + A.float() @ W.float().t() + bias.float()
    N.gemm(A, W, resid, epilogue=N.EPI_RESID_F32, bias=bias, pair=1)
    assert rel_err(resid, ref) < 1e-4
    # weight-gradient form: both MN-major, accumulate, split-K 3, device alpha
    X = torch.randn(4096, 768, device=dev()).bfloat16()
    dY = torch.randn(4096, 2304, device=dev()).bfloat16()
    gw = torch.randn(2304, 768, device=dev())
    a = torch.tensor([0.5], device=dev())
    ref = gw + 0.5 * (dY.float().t() @ X.float())
    ws = torch.empty(3 * 2304 * 768, device=dev())
    N.gemm(dY, X, gw, a_t=True, b_t=True, epilogue=N.EPI_F32, accumulate=True, splits=3,
           workspace=ws, alpha_ptr=a, pair=1)
    assert rel_err(gw, ref) < 1e-4


def test_gemm_pair_lm_head_shape():
    M, V, C = 1024, 50257, 768
    x = torch.randn(M, C, device=dev()).bfloat16()
    w = (torch.randn(V, C, device=dev()) * 0.02).bfloat16()
    logits = torch.zeros(M, 50304, dtype=torch.bfloat16, device=dev())
    N.gemm(x, w, logits[:, :V], pair=1)
    assert rel_err(logits[:, :V], x.float() @ w.float().t()) < 1e-2
    assert logits[:, V:].abs().max().item() == 0.0  # the padding columns are never written


# -------------------------------------------------------------- attention --
def ref_attention(q, k, v, causal=True, q_offset=0):
    # q: [B, H, Tq, 64], k/v: [B, H, Tk, 64] fp32
    s = q @ k.transpose(-1, -2) / 8.0
    Tq, Tk = q.shape[-2], k.shape[-2]
    if causal:
        qi = torch.arange(Tq, device=q.device)[:, None] + q_offset
        kj = torch.arange(Tk, device=q.device)[None, :]
        s = s.masked_fill(kj > qi, float("-inf"))
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize("B,H,T", [(1, 1, 64), (2, 3, 128), (2, 2, 200), (1, 12, 1024)])
def test_attention_fwd_bwd(B, H, T):
    C = H * 64
    torch.manual_seed(T + H)
    qkv = torch.randn(B * T, 3 * C, device=dev()).bfloat16()
    o = torch.empty(B * T, C, dtype=torch.bfloat16, device=dev())
    lse = torch.empty(B, H, T, device=dev())
    N.attention_fwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], o, lse, B, H, T)

    def heads(x):
        return x.float().view(B, T, H, 64).transpose(1, 2)

    q, k, v = heads(qkv[:, :C]), heads(qkv[:, C:2 * C]), heads(qkv[:, 2 * C:])
    q.requires_grad_(True), k.requires_grad_(True), v.requires_grad_(True)
    ref = ref_attention(q, k, v)
    got = o.float().view(B, T, H, 64).transpose(1, 2)
    assert rel_err(got, ref.detach()) < 2e-2

    do = torch.randn(B * T, C, device=dev()).bfloat16()
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B, H, T, device=dev())
    N.attention_bwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], o, do, dqkv[:, :C],
                    dqkv[:, C:2 * C], dqkv[:, 2 * C:], lse, delta, B, H, T)
    gq, gk, gv = torch.autograd.grad(ref, (q, k, v), heads(do))
    for got_g, ref_g in ((dqkv[:, :C], gq), (dqkv[:, C:2 * C], gk), (dqkv[:, 2 * C:], gv)):
        assert rel_err(heads(got_g), ref_g) < 3e-2


@pytest.mark.parametrize("B,H,KV,T", [(2, 4, 2, 256), (2, 12, 4, 1024), (1, 8, 1, 384), (2, 6, 3, 200)])
def test_attention_grouped_kv_heads(B, H, KV, T):
    """Grouped-query (and multi-query) attention: query head h reads key/value
    head h // (H // KV) by index; dK/dV sum over the group's query heads.
    Against fp32 torch with the key/value heads repeated (reference model.py:
    272-278)."""
    C, D = H * 64, KV * 64
    torch.manual_seed(H * 7 + KV)
    qkv = torch.randn(B * T, C + 2 * D, device=dev()).bfloat16()
    q, k, v = qkv[:, :C], qkv[:, C:C + D], qkv[:, C + D:]
    o = torch.empty(B * T, C, dtype=torch.bfloat16, device=dev())
    lse = torch.empty(B, H, T, device=dev())
    N.attention_fwd(q, k, v, o, lse, B, H, T, kv_heads=KV)

    def heads(x, n):
        return x.float().view(B, T, n, 64).transpose(1, 2)

    qh = heads(q, H).requires_grad_(True)
    kh = heads(k, KV).requires_grad_(True)
    vh = heads(v, KV).requires_grad_(True)
    G = H // KV
    ref = ref_attention(qh, kh.repeat_interleave(G, 1), vh.repeat_interleave(G, 1))
    assert rel_err(heads(o, H), ref.detach()) < 2e-2

    do = torch.randn(B * T, C, device=dev()).bfloat16()
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B, H, T, device=dev())
    N.attention_bwd(q, k, v, o, do, dqkv[:, :C], dqkv[:, C:C + D], dqkv[:, C + D:], lse, delta,
                    B, H, T, kv_heads=KV)
    N.check_errors()
    gq, gk, gv = torch.autograd.grad(ref, (qh, kh, vh), heads(do, H))
    assert rel_err(heads(dqkv[:, :C], H), gq) < 3e-2
    assert rel_err(heads(dqkv[:, C:C + D], KV), gk) < 3e-2
    assert rel_err(heads(dqkv[:, C + D:], KV), gv) < 3e-2


def test_attention_q_offset():
    # context-parallel shard: 64 local queries at absolute offset 128 vs 256 keys
    B, H, Tq, Tk, off = 1, 2, 64, 256, 128
    C = H * 64
    q = torch.randn(B * Tq, C, device=dev()).bfloat16()
    kv = torch.randn(B * Tk, 2 * C, device=dev()).bfloat16()
    o = torch.empty(B * Tq, C, dtype=torch.bfloat16, device=dev())
    lse = torch.empty(B, H, Tq, device=dev())
    N.attention_fwd(q, kv[:, :C], kv[:, C:], o, lse, B, H, Tq, Tk=Tk, q_offset=off)
    qh = q.float().view(B, Tq, H, 64).transpose(1, 2)
    kh = kv[:, :C].float().view(B, Tk, H, 64).transpose(1, 2)
    vh = kv[:, C:].float().view(B, Tk, H, 64).transpose(1, 2)
    ref = ref_attention(qh, kh, vh, q_offset=off)
    assert rel_err(o.float().view(B, Tq, H, 64).transpose(1, 2), ref) < 2e-2


def test_attention_deterministic():
    B, H, T = 2, 4, 256
    C = H * 64
    qkv = torch.randn(B * T, 3 * C, device=dev()).bfloat16()
    o = torch.empty(B * T, C, dtype=torch.bfloat16, device=dev())
    lse = torch.empty(B, H, T, device=dev())
    N.attention_fwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], o, lse, B, H, T)
    do = torch.randn(B * T, C, device=dev()).bfloat16()
    outs = []
    for _ in range(2):
        d = torch.empty_like(qkv)
        delta = torch.empty(B, H, T, device=dev())
        N.attention_bwd(qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:], o, do, d[:, :C], d[:, C:2 * C],
                        d[:, 2 * C:], lse, delta, B, H, T)
        outs.append(d)
    assert torch.equal(outs[0], outs[1])


# -------------------------------------------------------------- layernorm --
@pytest.mark.parametrize("M,C", [(64, 128), (1000, 768), (300, 1600)])
def test_layernorm(M, C):
    x = torch.randn(M, C, device=dev()) * 3 + 1
    g = (1 + 0.1 * torch.randn(C, device=dev())).bfloat16()
    b = (0.1 * torch.randn(C, device=dev())).bfloat16()
    y = torch.empty(M, C, dtype=torch.bfloat16, device=dev())
    mean = torch.empty(M, device=dev())
    rstd = torch.empty(M, device=dev())
    N.layernorm_fwd(x, g, b, y, mean, rstd)
    xr = x.clone().requires_grad_(True)
    gr = g.float().requires_grad_(True)
    br = b.float().requires_grad_(True)
    ref = torch.nn.functional.layer_norm(xr, (C,), gr, br, 1e-5)
    assert rel_err(y, ref.detach()) < 1e-2
    dy = torch.randn(M, C, device=dev()).bfloat16()
    gx, gg, gb = torch.autograd.grad(ref, (xr, gr, br), dy.float())
    dres = torch.ones(M, C, device=dev())
    dres16 = torch.empty(M, C, dtype=torch.bfloat16, device=dev())
    dg = torch.zeros(C, device=dev())
    db = torch.zeros(C, device=dev())
    ds = torch.full((C,), 2.0, device=dev())
    parts = N.layernorm_bwd_partials(M, C, dev())
    N.layernorm_bwd(dy, x, mean, rstd, g, dres, dres16, dg, db, parts, accumulate_dres=True,
                    dsum=ds, accumulate_dsum=True)
    assert rel_err(dres - 1, gx) < 1e-4
    assert rel_err(dres16, gx + 1) < 1e-2
    assert rel_err(dg, gg) < 1e-4
    assert rel_err(db, gb) < 1e-4
    # dsum = 2 + column sum of the written residual gradient (gx + 1)
    assert rel_err(ds, 2 + (gx + 1).sum(0)) < 1e-4
    # deterministic: a second identical launch gives bit-identical sums
    dres2 = torch.ones(M, C, device=dev())
    dg2 = torch.zeros(C, device=dev())
    db2 = torch.zeros(C, device=dev())
    N.layernorm_bwd(dy, x, mean, rstd, g, dres2, None, dg2, db2, parts, accumulate_dres=True,
                    accumulate_params=False)
    assert torch.equal(dres2, dres) and torch.equal(dg2, dg) and torch.equal(db2, db)


def test_colsum_bf16():
    x = torch.randn(1000, 768, device=dev()).bfloat16()
    out = torch.ones(768, device=dev())
    ws = torch.empty(N.colsum_ws_numel(1000, 768), device=dev())
    N.colsum_bf16(x, out, ws, accumulate=True)
    assert rel_err(out, 1 + x.float().sum(0)) < 1e-5


# --------------------------------------------------------------- embedding --
def test_embedding():
    V, C, B, T = 1000, 128, 3, 50
    wte = torch.randn(V, C, device=dev()).bfloat16()
    wpe = torch.randn(64, C, device=dev()).bfloat16()
    idx = torch.randint(0, V, (B, T), device=dev())
    x = torch.empty(B * T, C, device=dev())
    N.embedding_fwd(idx, wte, wpe, x)
    ref = wte.float()[idx] + wpe.float()[:T][None]
    assert rel_err(x.view(B, T, C), ref) < 1e-6
    dx = torch.randn(B * T, C, device=dev())
    gw = torch.zeros(V, C, device=dev())
    gp = torch.zeros(64, C, device=dev())
    N.embedding_bwd(idx, dx, gw, gp, V)
    ref_w = torch.zeros(V, C, device=dev()).index_add_(0, idx.flatten(), dx)
    assert rel_err(gw, ref_w) < 1e-5
    assert rel_err(gp[:T], dx.view(B, T, C).sum(0)) < 1e-5


def test_embedding_two_chunks():
    """Positions from two offsets (the zig-zag context-parallel layout)."""
    V, C, B, T, split, pos0, pos1 = 1000, 128, 2, 48, 16, 8, 40
    wte = torch.randn(V, C, device=dev()).bfloat16()
    wpe = torch.randn(128, C, device=dev()).bfloat16()
    idx = torch.randint(0, V, (B, T), device=dev())
    pos = torch.cat([torch.arange(pos0, pos0 + split), torch.arange(pos1, pos1 + T - split)]).to(dev())
    x = torch.empty(B * T, C, device=dev())
    N.embedding_fwd(idx, wte, wpe, x, pos0=pos0, pos_split=split, pos1=pos1)
    assert rel_err(x.view(B, T, C), wte.float()[idx] + wpe.float()[pos][None]) < 1e-6
    dx = torch.randn(B * T, C, device=dev())
    gp = torch.zeros(128, C, device=dev())
    N.embedding_bwd(idx, dx, None, gp, V, pos0=pos0, pos_split=split, pos1=pos1)
    ref = torch.zeros(128, C, device=dev()).index_add_(0, pos, dx.view(B, T, C).sum(0))
    assert rel_err(gp, ref) < 1e-5


# ----------------------------------------------------------- cross-entropy --
def test_cross_entropy():
    M, V, ld = 300, 50257, 50304
    logits = torch.zeros(M, ld, dtype=torch.bfloat16, device=dev())
    logits[:, :V] = (torch.randn(M, V, device=dev()) * 2).bfloat16()
    tgt = torch.randint(0, V, (M,), device=dev())
    tgt[::7] = -100
    ref_in = logits[:, :V].float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(ref_in, tgt, ignore_index=-100)
    (g,) = torch.autograd.grad(ref, ref_in)
    rows = torch.empty(M, device=dev())
    out = torch.empty(2, device=dev())
    N.cross_entropy_fwd_bwd(logits, tgt, rows, out, V)
    assert abs(out[0].item() - ref.item()) < 1e-3 * abs(ref.item())
    count = (tgt != -100).sum().item()
    assert abs(out[1].item() - 1.0 / count) < 1e-9
    assert rel_err(logits[:, :V].float() * out[1], g) < 2e-2
    assert logits[:, V:].abs().max().item() == 0


@pytest.mark.parametrize("M,V,ld,pair", [(300, 50257, 50304, 0), (1000, 50257, 50304, 1),
                                          (520, 1000, 1024, 1), (264, 777, 784, 0)])
def test_lm_head_cross_entropy_fused(M, V, ld, pair):
    """GEMM epilogue statistics + log-sum-exp fold + in-place gradient against
    torch fp32 F.cross_entropy on the same bf16 logits (odd M and V, ignored
    rows, padded columns), on single CTAs and on CTA pairs."""
    C = 768
    g = torch.Generator(device="cpu").manual_seed(M + V)
    h = torch.randn(M, C, generator=g).to(dev(), torch.bfloat16)
    w = (torch.randn(V, C, generator=g) * 0.08).to(dev(), torch.bfloat16)
    tgt = torch.randint(0, V, (M,), generator=g).to(dev())
    tgt[::7] = -100
    logits = torch.full((M, ld), 7.0, dtype=torch.bfloat16, device=dev())
    ws = N.CEWorkspace(M, V, dev())
    out = torch.empty(2, device=dev())
    N.gemm(h, w, logits[:, :V], epilogue=N.EPI_CE_STATS, ce=ws, ce_targets=tgt, pair=pair)
    # the logits the epilogue stored are the bf16 GEMM result
    assert rel_err(logits[:, :V], h.float() @ w.float().t()) < 1e-2
    # fp32 cross-entropy of exactly those bf16 logits (autocast's semantics)
    ref_logits = logits[:, :V].float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(ref_logits, tgt, ignore_index=-100)
    (gref,) = torch.autograd.grad(ref, ref_logits)
    lib = N.lib()
    stream = torch.cuda.current_stream().cuda_stream
    lib.ce_combine(ws.stats.data_ptr(), ws.nparts, M, tgt.data_ptr(), ws.tgt_logit.data_ptr(),
                   ws.lse.data_ptr(), ws.loss_rows.data_ptr(), stream)
    lib.loss_reduce(ws.loss_rows.data_ptr(), tgt.data_ptr(), M, out.data_ptr(), stream)
    lse_ref = torch.logsumexp(ref_logits.detach(), -1)
    assert (ws.lse - lse_ref).abs().max().item() < 1e-4
    lib.ce_grad(logits.data_ptr(), ld, M, V, ws.lse.data_ptr(), tgt.data_ptr(), 0, stream)
    assert abs(out[0].item() - ref.item()) < 1e-3 * abs(ref.item())
    count = (tgt != -100).sum().item()
    assert abs(out[1].item() - 1.0 / count) < 1e-9
    assert rel_err(logits[:, :V].float() * out[1], gref) < 2e-2
    assert logits[:, V:].abs().max().item() == 0
    # the public entry point does the same three steps
    logits2 = torch.zeros(M, ld, dtype=torch.bfloat16, device=dev())
    out2 = torch.empty(2, device=dev())
    N.lm_head_cross_entropy(h, w, logits2, tgt, N.CEWorkspace(M, V, dev()), out2, V)
    assert abs(out2[0].item() - out[0].item()) < 1e-6 * abs(out[0].item())
    assert torch.equal(logits2, logits)


@pytest.mark.parametrize("B,T,C,V", [(16, 1024, 768, 50257), (3, 200, 1600, 777), (2, 130, 1024, 64)])
def test_embedding_bwd_deterministic(B, T, C, V):
    """Token-embedding gradient summed in a fixed order: equal to torch's fp32
    index_add within rounding, bit-identical across calls (skewed token
    frequencies: a few ids take a third of the positions), slot table left at
    -1 for the next call."""
    g = torch.Generator(device="cpu").manual_seed(B * T + V)
    idx = torch.randint(0, V, (B, T), generator=g)
    idx[:, ::3] = torch.randint(0, min(V, 5), (B, (T + 2) // 3), generator=g)
    idx = idx.to(dev())
    dx = torch.randn(B * T, C, generator=g).to(dev())
    base = torch.randn(V, C, generator=g).to(dev())
    ws = N.EmbeddingGradWorkspace(B * T, C, V, dev())
    outs = []
    for _ in range(2):
        wte_g = base.clone()
        wpe_g = torch.zeros(T, C, device=dev())
        N.embedding_bwd(idx, dx, wte_g, wpe_g, V, det=ws)
        outs.append(wte_g)
    ref = base.clone().index_add_(0, idx.reshape(-1), dx)
    assert rel_err(outs[0], ref) < 1e-5  # fp32 sums of ~1,000 rows in another order
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(ws.slots, torch.full_like(ws.slots, -1))
    assert rel_err(wpe_g, dx.view(B, T, C).sum(0)) < 1e-6


def test_exp2_fma_against_exp2():
    """The FMA-pipe 2^x that takes half of the softmax exponentials (Cody-Waite
    reduction + degree-4 fit): relative error against torch.exp2 in fp32 below
    3e-6 (its fit bound) over the range the kernels use, exact at integers."""
    x = torch.cat([torch.linspace(-125.0, 127.0, 1_000_003), torch.arange(-125.0, 128.0),
                   torch.rand(100_000) * 2 - 1]).to(dev())
    y = torch.empty_like(x)
    N.lib().exp2_fma_test(x.data_ptr(), y.data_ptr(), x.numel(), torch.cuda.current_stream().cuda_stream)
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref).abs() / ref).max().item()
    assert rel < 3e-6, rel


# ------------------------------------------------------------------- AdamW --
def test_adamw_matches_torch():
    n = 10007
    n_decay = 6000
    torch.manual_seed(0)
    p = torch.randn(n, device=dev())
    grads = [torch.randn(n, device=dev()) for _ in range(3)]
    ref_a = torch.nn.Parameter(p[:n_decay].clone())
    ref_b = torch.nn.Parameter(p[n_decay:].clone())
    opt = torch.optim.AdamW([{"params": [ref_a], "weight_decay": 0.1},
                             {"params": [ref_b], "weight_decay": 0.0}],
                            lr=3e-4, betas=(0.9, 0.95), eps=1e-8, foreach=False, fused=False)
    mine = p.clone()
    m = torch.zeros(n, device=dev())
    v = torch.zeros(n, device=dev())
    pb = torch.empty(n, dtype=torch.bfloat16, device=dev())
    for step, gr in enumerate(grads, start=1):
        ref_a.grad = gr[:n_decay].clone()
        ref_b.grad = gr[n_decay:].clone()
        opt.step()
        hp = torch.tensor([3e-4, 0.9, 0.95, 1e-8, 0.1, 1 - 0.9**step, math.sqrt(1 - 0.95**step), 1.0],
                          device=dev())
        N.adamw_step(mine, gr, m, v, pb, n_decay, hp)
    ref = torch.cat([ref_a.detach(), ref_b.detach()])
    assert (mine - ref).abs().max().item() < 1e-6
    assert torch.equal(pb, mine.bfloat16())


def test_grad_norm_clip():
    g = torch.randn(123457, device=dev())
    ws = torch.empty(1024, device=dev())
    ss = torch.empty(1, device=dev())
    clip = torch.empty(1, device=dev())
    norm = torch.empty(1, device=dev())
    N.grad_sumsq(g, ws, ss)
    N.clip_coef(ss, 1.0, clip, norm)
    ref = g.norm().item()
    assert abs(norm.item() - ref) < 1e-4 * ref
    assert abs(clip.item() - min(1.0, 1.0 / (ref + 1e-6))) < 1e-6


def test_bounded_wait_returns_error():
    """A flag nobody sets must time out in-kernel and leave the context usable."""
    flag = torch.zeros(1, dtype=torch.int32, device=dev())
    err = torch.zeros(1, dtype=torch.int32, device=dev())
    N.lib().flag_wait_test(flag.data_ptr(), 1, 200_000_000, err.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert err.item() == 1 << 3
    # the context still works
    x = torch.ones(4, device=dev())
    assert x.sum().item() == 4


@pytest.mark.parametrize("B,H,T,off,Tk", [(2, 3, 384, 0, None), (1, 2, 200, 0, None),
                                         (1, 12, 1024, 0, None), (1, 2, 128, 256, 384),
                                         (8, 12, 1024, 0, None), (3, 5, 640, 0, None)])
def test_attention_tensor_core_matches_mma_sync(B, H, T, off, Tk):
    """tcgen05 forward (default) vs the mma.sync forward on the same inputs."""
    Tk = T if Tk is None else Tk
    C = H * 64
    q = torch.randn(B * T, C, device=dev()).bfloat16()
    kv = torch.randn(B * Tk, 2 * C, device=dev()).bfloat16()
    outs = []
    L = N.lib()
    try:
        for impl in (0, 1):
            L.attn_set_impl(impl)
            o = torch.empty(B * T, C, dtype=torch.bfloat16, device=dev())
            lse = torch.empty(B, H, T, device=dev())
            N.attention_fwd(q, kv[:, :C], kv[:, C:], o, lse, B, H, T, Tk=Tk, q_offset=off)
            outs.append((o.float(), lse))
    finally:
        L.attn_set_impl(0)
    assert rel_err(outs[0][0], outs[1][0]) < 2e-2
    assert (outs[0][1] - outs[1][1]).abs().max().item() < 2e-2


def test_attention_tensor_core_lazy_rescale():
    """Keys whose scores grow along the sequence force the running row max up
    by far more than the lazy-rescale threshold several times per row."""
    B, H, T = 2, 4, 1024
    C = H * 64
    torch.manual_seed(7)
    q = torch.randn(B * T, C, device=dev())
    k = torch.randn(B * T, C, device=dev())
    grow = (1.0 + torch.arange(T, device=dev()).float() / 48.0).repeat(B)[:, None]
    k = (k * grow).bfloat16()
    q = q.bfloat16()
    v = torch.randn(B * T, C, device=dev()).bfloat16()
    outs = []
    L = N.lib()
    try:
        for impl in (0, 1):
            L.attn_set_impl(impl)
            o = torch.empty(B * T, C, dtype=torch.bfloat16, device=dev())
            lse = torch.empty(B, H, T, device=dev())
            N.attention_fwd(q, k, v, o, lse, B, H, T)
            outs.append((o.float(), lse))
    finally:
        L.attn_set_impl(0)
    assert rel_err(outs[0][0], outs[1][0]) < 2e-2
    assert (outs[0][1] - outs[1][1]).abs().max().item() < 2e-2 * outs[1][1].abs().max().item()


@pytest.mark.parametrize("B,H,T,off,Tk", [(2, 3, 384, 0, None), (1, 2, 200, 0, None),
                                         (2, 12, 1024, 0, None), (1, 2, 128, 256, 384)])
def test_attention_backward_tensor_core_matches_mma_sync(B, H, T, off, Tk):
    """tcgen05 backward (default) vs the mma.sync backward on the same inputs."""
    Tk = T if Tk is None else Tk
    C = H * 64
    torch.manual_seed(T + H)
    q = torch.randn(B * T, C, device=dev()).bfloat16()
    kv = torch.randn(B * Tk, 2 * C, device=dev()).bfloat16()
    o = torch.empty(B * T, C, dtype=torch.bfloat16, device=dev())
    lse = torch.empty(B, H, T, device=dev())
    N.attention_fwd(q, kv[:, :C], kv[:, C:], o, lse, B, H, T, Tk=Tk, q_offset=off)
    do = torch.randn(B * T, C, device=dev()).bfloat16()
    outs = []
    L = N.lib()
    try:
        for impl in (0, 1):
            L.attn_set_impl(impl)
            dq = torch.empty_like(q)
            dkv = torch.empty_like(kv)
            delta = torch.empty(B, H, T, device=dev())
            N.attention_bwd(q, kv[:, :C], kv[:, C:], o, do, dq, dkv[:, :C], dkv[:, C:], lse, delta,
                            B, H, T, Tk=Tk, q_offset=off)
            outs.append((dq.float(), dkv.float()))
    finally:
        L.attn_set_impl(0)
    assert rel_err(outs[0][0], outs[1][0]) < 2e-2
    assert rel_err(outs[0][1], outs[1][1]) < 2e-2
