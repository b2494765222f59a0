"""Torch implementations of the native-op contracts, for host-orchestration
tests on CPU.

The engine, the pipeline stage engine and the trainers drive the sm_100a
kernels through ``gpt2_harness_b200.ops.native``. :func:`install` replaces
those calls (and the CUDA stream/event/pinned-memory calls around them) with
plain torch code that follows each kernel's documented contract -- the same
output dtypes, bf16 rounding points, accumulate flags, strided views, partial
key ranges and position offsets -- so the Python that sequences the launches
(buffer wiring, accumulation, micro-batch schedules, point-to-point transfers)
can be checked on CPU against the autograd oracle. It says nothing about the
kernels themselves; their numerics are the GPU tier's job.
"""

from __future__ import annotations

import math
from contextlib import contextmanager
from types import SimpleNamespace

import torch

from gpt2_harness_b200.models import gpt as _gpt
from gpt2_harness_b200.ops import native as N

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def _gelu(z):
    return _gpt.gelu_tanh(z)


def _gelu_grad(z):
    u = _SQRT_2_OVER_PI * (z + 0.044715 * z.pow(3))
    t = torch.tanh(u)
    return 0.5 * (1 + t) + 0.5 * z * (1 - t * t) * _SQRT_2_OVER_PI * (1 + 3 * 0.044715 * z * z)


def gemm(a, b, out, *, a_t=False, b_t=False, epilogue=N.EPI_BF16, bias=None, aux=None, alpha=1.0,
         alpha_ptr=None, accumulate=False, splits=1, workspace=None, bn=256, max_ctas=0):
    A = (a.t() if a_t else a).float()
    Bm = (b.t() if b_t else b).float()
    r = A @ Bm.t() * alpha
    if alpha_ptr is not None:
        r = r * alpha_ptr.reshape(-1)[0].float()
    n = r.shape[1]
    dst = out[:, :n]
    if bias is not None and epilogue in (N.EPI_BF16, N.EPI_BIAS_GELU, N.EPI_RESID_F32):
        r = r + bias[:n].float()
    if epilogue == N.EPI_BF16:
        dst.copy_(r)
    elif epilogue == N.EPI_BIAS_GELU:
        aux[:, :n].copy_(r)
        dst.copy_(_gelu(r))
    elif epilogue == N.EPI_RESID_F32:
        src = aux if aux is not None else dst
        dst.copy_(src[:, :n].float() + r)
    elif epilogue == N.EPI_F32:
        dst.copy_(r + dst if accumulate else r)
    elif epilogue == N.EPI_GELU_BWD:
        dst.copy_(r * _gelu_grad(aux[:, :n].float()))
    else:
        raise ValueError(epilogue)
    return out


def layernorm_fwd(x, gamma, beta, y, mean, rstd, eps=1e-5):
    xf = x.float()
    mu = xf.mean(-1)
    var = ((xf - mu[:, None]) ** 2).mean(-1)
    rs = torch.rsqrt(var + eps)
    mean.copy_(mu)
    rstd.copy_(rs)
    y.copy_((xf - mu[:, None]) * rs[:, None] * gamma.float() + beta.float())
    return y


def layernorm_bwd_partials(M, C, device):
    return torch.empty(1, 3, C, dtype=torch.float32, device=device)


def layernorm_bwd(dy, x, mean, rstd, gamma, dres, dres_bf16, dgamma, dbeta, partials, accumulate_dres,
                  accumulate_params=True, dsum=None, accumulate_dsum=False):
    xhat = (x.float() - mean[:, None]) * rstd[:, None]
    g = dy.float()
    dxhat = g * gamma.float()
    dx = rstd[:, None] * (dxhat - dxhat.mean(-1, keepdim=True) - xhat * (dxhat * xhat).mean(-1, keepdim=True))
    dres.copy_(dres + dx if accumulate_dres else dx)
    if dres_bf16 is not None:
        dres_bf16.copy_(dres)
    dg, db = (g * xhat).sum(0), g.sum(0)
    dgamma.copy_(dgamma + dg if accumulate_params else dg)
    dbeta.copy_(dbeta + db if accumulate_params else db)
    if dsum is not None:
        cs = dres.sum(0)
        dsum.copy_(dsum + cs if accumulate_dsum else cs)


def colsum_bf16(x, out, ws, accumulate=True):
    s = x.float().sum(0)
    out.copy_(out + s if accumulate else s)


def _positions(T, pos0, pos_split, pos1, device):
    split = T if pos_split is None else pos_split
    t = torch.arange(T, device=device)
    return torch.where(t < split, pos0 + t, pos1 + t - split)


def embedding_fwd(idx, wte, wpe, x, pos0=0, pos_split=None, pos1=0):
    B, T = idx.shape
    pos = _positions(T, pos0, pos_split, pos1, idx.device)
    x.copy_((wte.float()[idx] + wpe.float()[pos][None]).reshape(B * T, -1))
    return x


def embedding_bwd(idx, dx, wte_grad, wpe_grad, vocab, pos0=0, pos_split=None, pos1=0):
    B, T = idx.shape
    C = dx.shape[-1]
    d = dx.reshape(B, T, C)
    if wte_grad is not None:
        flat = idx.reshape(-1)
        ok = (flat >= 0) & (flat < vocab)
        wte_grad.index_add_(0, flat[ok], dx.reshape(-1, C)[ok])
    if wpe_grad is not None:
        pos = _positions(T, pos0, pos_split, pos1, idx.device)
        wpe_grad.index_add_(0, pos, d.sum(0))


def cross_entropy_fwd_bwd(logits, targets, loss_rows, loss_out, vocab):
    lf = logits[:, :vocab].float()
    t = targets.reshape(-1)
    valid = t != -100
    tt = torch.where(valid, t, torch.zeros_like(t))
    lse = torch.logsumexp(lf, -1)
    rows = (lse - lf.gather(1, tt[:, None])[:, 0]) * valid
    loss_rows.copy_(rows)
    count = max(int(valid.sum()), 1)
    loss_out[0] = rows.sum() / count
    loss_out[1] = 1.0 / count
    grad = torch.softmax(lf, -1)
    grad[torch.arange(len(t)), tt] -= 1.0
    grad = grad * valid[:, None]
    logits[:, :vocab].copy_(grad)
    logits[:, vocab:].zero_()


def _heads(t, b, rows, T, H):
    return t[b * rows: b * rows + T].reshape(T, H, 64).float()


def attention_fwd(q, k, v, o, lse, B, H, Tq, Tk=None, q_offset=0, causal=True, scale=None,
                  kv_rows=None, q_rows=None):
    Tk = Tq if Tk is None else Tk
    qr = Tq if q_rows is None else q_rows
    kr = Tk if kv_rows is None else kv_rows
    scale = 1.0 / 8.0 if scale is None else scale
    for b in range(B):
        Q, K, V = _heads(q, b, qr, Tq, H), _heads(k, b, kr, Tk, H), _heads(v, b, kr, Tk, H)
        s = torch.einsum("thd,shd->hts", Q, K) * scale
        if causal:
            mask = torch.arange(Tk)[None, :] > (torch.arange(Tq)[:, None] + q_offset)
            s = s.masked_fill(mask[None], float("-inf"))
        lse.view(B, H, Tq)[b].copy_(torch.logsumexp(s, -1))
        o[b * qr: b * qr + Tq].copy_(torch.einsum("hts,shd->thd", torch.softmax(s, -1), V).reshape(Tq, H * 64))


def attention_bwd(q, k, v, o, dout, dq, dk, dv, lse, delta, B, H, Tq, Tk=None, q_offset=0, causal=True,
                  scale=None, kv_rows=None, q_rows=None):
    Tk = Tq if Tk is None else Tk
    qr = Tq if q_rows is None else q_rows
    kr = Tk if kv_rows is None else kv_rows
    scale = 1.0 / 8.0 if scale is None else scale
    for b in range(B):
        Q = _heads(q, b, qr, Tq, H).requires_grad_(True)
        K = _heads(k, b, kr, Tk, H).requires_grad_(True)
        V = _heads(v, b, kr, Tk, H).requires_grad_(True)
        with torch.enable_grad():
            s = torch.einsum("thd,shd->hts", Q, K) * scale
            if causal:
                mask = torch.arange(Tk)[None, :] > (torch.arange(Tq)[:, None] + q_offset)
                s = s.masked_fill(mask[None], float("-inf"))
            out = torch.einsum("hts,shd->thd", torch.softmax(s, -1), V)
            gq, gk, gv = torch.autograd.grad(out, (Q, K, V), _heads(dout, b, qr, Tq, H))
        dq[b * qr: b * qr + Tq].copy_(gq.reshape(Tq, H * 64))
        dk[b * kr: b * kr + Tk].copy_(gk.reshape(Tk, H * 64))
        dv[b * kr: b * kr + Tk].copy_(gv.reshape(Tk, H * 64))


def grad_sumsq(g, ws, out):
    out[0] = g.double().pow(2).sum().float()


def clip_coef(sumsq, max_norm, clip, norm_out=None, scale2=1.0):
    norm = math.sqrt(float(sumsq[0]) * scale2)
    clip[0] = min(max_norm / (norm + 1e-6), 1.0)
    if norm_out is not None:
        norm_out[0] = norm


def adamw_step(p, g, m, v, p_bf16, n_decay, hp, clip=None, decay_ranges=None):
    lr, b1, b2, eps, wd, bc1, bc2s, gsc = [float(x) for x in hp[:8]]
    gs = gsc * (float(clip[0]) if clip is not None else 1.0)
    decay = torch.zeros(p.numel(), dtype=torch.bool, device=p.device)
    decay[:n_decay] = True
    if decay_ranges is not None:
        r = decay_ranges.tolist()
        for lo, hi in zip(r[::2], r[1::2]):
            decay[lo:hi] = True
    gj = g * gs
    p.mul_(torch.where(decay, 1.0 - lr * wd, 1.0))
    m.add_((gj - m) * (1.0 - b1))
    v.mul_(b2).add_((1.0 - b2) * gj * gj)
    p.add_(-(lr / bc1) * (m / (v.sqrt() / bc2s + eps)))
    if p_bf16 is not None:
        p_bf16.copy_(p)


def cast_f32_bf16(x, out):
    return out.copy_(x)


class _Event:
    def record(self, *a, **k):
        pass

    def synchronize(self):
        pass

    def query(self):
        return True


OPS = {
    "gemm": gemm, "layernorm_fwd": layernorm_fwd, "layernorm_bwd": layernorm_bwd,
    "layernorm_bwd_partials": layernorm_bwd_partials, "colsum_bf16": colsum_bf16,
    "embedding_fwd": embedding_fwd, "embedding_bwd": embedding_bwd,
    "cross_entropy_fwd_bwd": cross_entropy_fwd_bwd, "attention_fwd": attention_fwd,
    "attention_bwd": attention_bwd, "grad_sumsq": grad_sumsq, "clip_coef": clip_coef,
    "adamw_step": adamw_step, "cast_f32_bf16": cast_f32_bf16,
}


@contextmanager
def installed(monkeypatch):
    """Route the native-op calls and the CUDA runtime calls around them to
    the torch versions for the duration of a test (pytest ``monkeypatch``)."""
    from gpt2_harness_b200.models import engine as engine_mod

    for name, fn in OPS.items():
        monkeypatch.setattr(N, name, fn)
    monkeypatch.setattr(N, "lib", lambda: SimpleNamespace())
    monkeypatch.setattr(N, "check_errors", lambda *a, **k: None)
    monkeypatch.setattr(engine_mod, "DEVICE_TYPES", ("cuda", "cpu"))
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self, *a, **k: self)
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "set_device", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    yield


def install_in_process() -> None:
    """The same replacements without pytest (for spawned worker processes)."""

    class _MP:
        def setattr(self, obj, name, value):
            setattr(obj, name, value)

    with installed(_MP()):
        pass
