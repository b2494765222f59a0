"""Torch implementations of the native-op contracts, for host-orchestration
tests on CPU.

The engine, the pipeline stage engine and the trainers drive the sm_100a
kernels through ``gpt2_harness_b200.ops.native``. :func:`installed` replaces
those calls (and the CUDA stream/event/pinned-memory calls around them) with
plain torch code that follows each kernel's documented contract -- the same
output dtypes, bf16 rounding points, accumulate flags, strided views, partial
key ranges and position offsets -- so the Python that sequences the launches
(buffer wiring, accumulation, micro-batch schedules, point-to-point transfers)
can be checked on CPU against the autograd oracle. It says nothing about the
kernels themselves; their numerics are the GPU tier's job.
"""

from __future__ import annotations

import ctypes
import math
import os
import tempfile
import time
from contextlib import contextmanager
from types import SimpleNamespace

import torch
import torch.distributed as dist

from gpt2_harness_b200.models import gpt as _gpt
from gpt2_harness_b200.ops import native as N

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def _gelu(z):
    return _gpt.gelu_tanh(z)


def _gelu_grad(z):
    u = _SQRT_2_OVER_PI * (z + 0.044715 * z.pow(3))
    t = torch.tanh(u)
    return 0.5 * (1 + t) + 0.5 * z * (1 - t * t) * _SQRT_2_OVER_PI * (1 + 3 * 0.044715 * z * z)


def _require(ok, what):
    """The launchers' host-side preconditions (a violation is a host bug the
    real kernel would reject)."""
    if not ok:
        raise AssertionError(f"native precondition violated: {what}")


def _row_bytes_ok(t, esz):
    return t.dim() == 2 and t.stride(1) == 1 and (t.stride(0) * esz) % 16 == 0 and t.data_ptr() % 16 == 0


def gemm(a, b, out, *, a_t=False, b_t=False, epilogue=N.EPI_BF16, bias=None, aux=None, alpha=1.0,
         alpha_ptr=None, accumulate=False, splits=1, workspace=None, bn=256, max_ctas=0, pair=-1,
         ce=None, ce_targets=None, ce_vocab_offset=0, owner_out=None):
    # operand loads are TMA: 16-byte aligned bases and row strides (csrc/gemm.cu)
    _require(a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16, "gemm operands bf16")
    _require(_row_bytes_ok(a, 2) and _row_bytes_ok(b, 2), "gemm operand alignment")
    _require(bn in (128, 256), "gemm tile width")
    _require(splits <= 1 or epilogue == N.EPI_F32, "split-K needs the fp32 epilogue")
    A = (a.t() if a_t else a).float()
    Bm = (b.t() if b_t else b).float()
    r = A @ Bm.t() * alpha
    if alpha_ptr is not None:
        r = r * alpha_ptr.reshape(-1)[0].float()
    n = r.shape[1]
    dst = out[:, :n]
    if bias is not None and epilogue in (N.EPI_BF16, N.EPI_BIAS_GELU, N.EPI_RESID_F32):
        r = r + bias[:n].float()
    if epilogue == N.EPI_BF16 and owner_out is not None:
        # row m goes to its owner's inbox: bases[m // rows] + (m % rows) * ldo
        bases, rows = owner_out[0], owner_out[1]
        ld = out.stride(0)
        for q, base in enumerate(int(b) for b in bases.reshape(-1)):
            blk = r[q * rows:(q + 1) * rows]
            if blk.shape[0] == 0:
                break
            view = _at(base, rows * ld, torch.bfloat16).view(rows, ld)[:, :n]
            view.copy_(blk)
    elif epilogue == N.EPI_BF16:
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


def _push_rows(t, push):
    """The kernels' row push: the rows of `t` also land in every peer copy."""
    if push is None:
        return
    bases, n, local = push
    _require(t.is_contiguous(), "pushed rows are contiguous")
    for base in [int(b) for b in bases.reshape(-1)[:n]]:
        _at(base + (t.data_ptr() - int(local)), t.numel(), t.dtype).copy_(t.reshape(-1))


def layernorm_fwd(x, gamma, beta, y, mean, rstd, eps=1e-5, push=None):
    _require(x.shape[-1] % 4 == 0 and x.dtype == torch.float32 and y.dtype == torch.bfloat16, "layernorm shapes")
    xf = x.float()
    mu = xf.mean(-1)
    var = ((xf - mu[:, None]) ** 2).mean(-1)
    rs = torch.rsqrt(var + eps)
    mean.copy_(mu)
    rstd.copy_(rs)
    y.copy_((xf - mu[:, None]) * rs[:, None] * gamma.float() + beta.float())
    _push_rows(y, push)
    return y


def layernorm_bwd_partials(M, C, device):
    return torch.empty(1, 3, C, dtype=torch.float32, device=device)


def layernorm_bwd(dy, x, mean, rstd, gamma, dres, dres_bf16, dgamma, dbeta, partials, accumulate_dres,
                  accumulate_params=True, dsum=None, accumulate_dsum=False, push=None):
    xhat = (x.float() - mean[:, None]) * rstd[:, None]
    g = dy.float()
    dxhat = g * gamma.float()
    dx = rstd[:, None] * (dxhat - dxhat.mean(-1, keepdim=True) - xhat * (dxhat * xhat).mean(-1, keepdim=True))
    dres.copy_(dres + dx if accumulate_dres else dx)
    if dres_bf16 is not None:
        dres_bf16.copy_(dres)
        _push_rows(dres_bf16, push)
    dg, db = (g * xhat).sum(0), g.sum(0)
    dgamma.copy_(dgamma + dg if accumulate_params else dg)
    dbeta.copy_(dbeta + db if accumulate_params else db)
    if dsum is not None:
        cs = dres.sum(0)
        dsum.copy_(dsum + cs if accumulate_dsum else cs)


def colsum_bf16(x, out, ws, accumulate=True):
    s = x.float().sum(0)
    out.copy_(out + s if accumulate else s)


def colsum_f32(x, out, accumulate=True):
    s = x.sum(0)
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


def embedding_bwd(idx, dx, wte_grad, wpe_grad, vocab, pos0=0, pos_split=None, pos1=0, det=None):
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
    _require(_row_bytes_ok(logits, 2) and logits.shape[1] % 8 == 0, "logits rows 16-byte aligned")
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


def lm_head_cross_entropy(h, w, logits, targets, ws, loss_out, vocab):
    # the fused path's contract: the GEMM, then the cross-entropy's loss and
    # in-place gradient over the whole padded buffer
    gemm(h, w, logits[:, :vocab])
    cross_entropy_fwd_bwd(logits, targets.reshape(-1), ws.loss_rows, loss_out, vocab)


def _heads(t, b, rows, T, H):
    return t[b * rows: b * rows + T].reshape(T, H, 64).float()


def attention_fwd(q, k, v, o, lse, B, H, Tq, Tk=None, q_offset=0, causal=True, scale=None,
                  kv_rows=None, q_rows=None, kv_heads=None):
    Tk = Tq if Tk is None else Tk
    qr = Tq if q_rows is None else q_rows
    kr = Tk if kv_rows is None else kv_rows
    scale = 1.0 / 8.0 if scale is None else scale
    G = H // (kv_heads or H)
    for b in range(B):
        Q = _heads(q, b, qr, Tq, H)
        K = _heads(k, b, kr, Tk, H // G).repeat_interleave(G, 1)
        V = _heads(v, b, kr, Tk, H // G).repeat_interleave(G, 1)
        s = torch.einsum("thd,shd->hts", Q, K) * scale
        if causal:
            mask = torch.arange(Tk)[None, :] > (torch.arange(Tq)[:, None] + q_offset)
            s = s.masked_fill(mask[None], float("-inf"))
        lse.view(B, H, Tq)[b].copy_(torch.logsumexp(s, -1))
        o[b * qr: b * qr + Tq].copy_(torch.einsum("hts,shd->thd", torch.softmax(s, -1), V).reshape(Tq, H * 64))


def attention_bwd(q, k, v, o, dout, dq, dk, dv, lse, delta, B, H, Tq, Tk=None, q_offset=0, causal=True,
                  scale=None, kv_rows=None, q_rows=None, kv_heads=None):
    Tk = Tq if Tk is None else Tk
    qr = Tq if q_rows is None else q_rows
    kr = Tk if kv_rows is None else kv_rows
    scale = 1.0 / 8.0 if scale is None else scale
    G = H // (kv_heads or H)
    for b in range(B):
        Q = _heads(q, b, qr, Tq, H).requires_grad_(True)
        K = _heads(k, b, kr, Tk, H // G).requires_grad_(True)
        V = _heads(v, b, kr, Tk, H // G).requires_grad_(True)
        with torch.enable_grad():
            s = torch.einsum("thd,shd->hts", Q, K.repeat_interleave(G, 1)) * scale
            if causal:
                mask = torch.arange(Tk)[None, :] > (torch.arange(Tq)[:, None] + q_offset)
                s = s.masked_fill(mask[None], float("-inf"))
            out = torch.einsum("hts,shd->thd", torch.softmax(s, -1), V.repeat_interleave(G, 1))
            gq, gk, gv = torch.autograd.grad(out, (Q, K, V), _heads(dout, b, qr, Tq, H))
        dq[b * qr: b * qr + Tq].copy_(gq.reshape(Tq, H * 64))
        dk[b * kr: b * kr + Tk].copy_(gk.reshape(Tk, H // G * 64))
        dv[b * kr: b * kr + Tk].copy_(gv.reshape(Tk, H // G * 64))


# ------------------------------------------------------------------ decode --
def decode_embed(tok, lens, wte, wpe, x):
    x.copy_(wte.float()[tok] + wpe.float()[lens.long()])


def decode_partials(B, H, Tmax, device):
    return torch.empty(1, device=device), torch.empty(1, device=device)


def decode_attn(qkv, k_cache, v_cache, lens, part_o, part_ml, out, H, Hkv, scale=None):
    """Append this step's k/v at lens[b], then attend over positions 0..lens[b]."""
    scale = 1.0 / 8.0 if scale is None else scale
    rep = H // Hkv
    for b in range(qkv.shape[0]):
        pos = int(lens[b])
        q = qkv[b, :H * 64].float().view(H, 64)
        k_cache[b, :, pos] = qkv[b, H * 64:(H + Hkv) * 64].view(Hkv, 64)
        v_cache[b, :, pos] = qkv[b, (H + Hkv) * 64:(H + 2 * Hkv) * 64].view(Hkv, 64)
        K = k_cache[b, :, :pos + 1].float().repeat_interleave(rep, 0)
        V = v_cache[b, :, :pos + 1].float().repeat_interleave(rep, 0)
        p = torch.softmax(torch.einsum("hd,htd->ht", q, K) * scale, -1)
        out[b, :H * 64] = torch.einsum("ht,htd->hd", p, V).reshape(-1)


def decode_argmax(logits, vocab, tok, lens, hist):
    a = logits[:, :vocab].float().argmax(-1)
    tok.copy_(a)
    for b in range(logits.shape[0]):
        hist[b, int(lens[b]) + 1] = a[b]
    lens += 1


def grad_sumsq(g, ws, out):
    out[0] = g.double().pow(2).sum().float()


def clip_coef(sumsq, max_norm, clip, norm_out=None, scale2=1.0):
    norm = math.sqrt(float(sumsq[0]) * scale2)
    clip[0] = min(max_norm / (norm + 1e-6), 1.0)
    if norm_out is not None:
        norm_out[0] = norm


def adamw_step(p, g, m, v, p_bf16, n_decay, hp, clip=None, decay_ranges=None):
    _require(all(t.data_ptr() % 16 == 0 for t in (p, g, m, v)), "adamw buffers 16-byte aligned")
    _require(p_bf16 is None or p_bf16.data_ptr() % 8 == 0, "adamw bf16 copy 8-byte aligned")
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


def cast_bf16_f32(x, out):
    out.copy_(x.float())
    return out


# ------------------------------------------------------ symmetric memory --
def _at(ptr: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
    """A CPU tensor aliasing ``numel`` elements at address ``ptr``."""
    esz = torch.empty((), dtype=dtype).element_size()
    return torch.frombuffer((ctypes.c_char * (numel * esz)).from_address(ptr), dtype=dtype)


def _ptr_list(ptr: int, n: int) -> list:
    return [int(x) for x in _at(ptr, n, torch.int64)]


class FakeSymmetricBuffer:
    """Equal-sized host buffers mapped into every rank's process through
    shared files: the CPU stand-in for the CUDA-IPC symmetric buffers, with
    the same attributes (peer_ptrs / peer_ptrs_dev hold this process's
    addresses of every rank's mapping)."""

    #: peer_ptrs_dev address -> buffer (to find a kernel call's process group)
    by_ptrs: dict = {}

    def __init__(self, nbytes: int, group=None, device=None) -> None:
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device("cpu")
        self.nbytes = int((nbytes + 255) // 256 * 256)
        tag = [tempfile.mkdtemp(prefix="g2b_symm_") if self.rank == 0 else None]
        dist.broadcast_object_list(tag, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        self.dir = tag[0]
        path = lambda r: os.path.join(self.dir, f"buf_{r}")
        self.local = torch.from_file(path(self.rank), shared=True, size=self.nbytes, dtype=torch.uint8)
        self.local.zero_()
        dist.barrier(group=group)
        self._maps = [self.local if r == self.rank else
                      torch.from_file(path(r), shared=True, size=self.nbytes, dtype=torch.uint8)
                      for r in range(self.world)]
        self.peer_ptrs = [m.data_ptr() for m in self._maps]
        self.ptr = self.peer_ptrs[self.rank]
        self.peer_ptrs_dev = torch.tensor(self.peer_ptrs, dtype=torch.int64)
        FakeSymmetricBuffer.by_ptrs[self.peer_ptrs_dev.data_ptr()] = self

    def view(self, dtype, numel=None, offset_bytes: int = 0):
        esz = torch.empty((), dtype=dtype).element_size()
        n = (self.nbytes - offset_bytes) // esz if numel is None else numel
        return self.local[offset_bytes:offset_bytes + n * esz].view(dtype)

    def close(self) -> None:
        self._maps = []


class FakeMulticastBuffer(FakeSymmetricBuffer):
    """The multicast form's stand-in: the same shared host buffers, and an
    ``mc_ptr`` the fake all-reduce only checks for being set."""

    def __init__(self, nbytes: int, group=None, device=None) -> None:
        super().__init__(nbytes, group, device)
        self.mc_ptr = self.ptr


def _group(flags_ptr):
    """The process group of the symmetric flag buffer a kernel call names."""
    buf = FakeSymmetricBuffer.by_ptrs.get(int(flags_ptr))
    return None if buf is None else buf.group


def _barrier(flags_ptr):
    dist.barrier(group=_group(flags_ptr))


# ---------------------------------------- context-parallel gather / reduce --
def _cp_layout(d):
    rank, world, B, Tl, cols = d["rank"], d["world"], d["B"], d["Tl"], d["cols"]
    T = world * Tl
    if d.get("zigzag", 0):
        h = Tl // 2
        segs = [(rank * h, 0, h), ((2 * world - 1 - rank) * h, h, h)]   # (global start, local start, len)
        owner = lambda k: k if k < world else 2 * world - 1 - k
        needed = [(k * h, h, owner(k)) for k in range(2 * world - rank) if k not in (rank, 2 * world - 1 - rank)]
    else:
        segs = [(rank * Tl, 0, Tl)]
        needed = [(q * Tl, Tl, q) for q in range(rank)]
    return rank, world, B, Tl, cols, T, segs, needed


def cp_kv_gather(d, stream=0):
    rank, world, B, Tl, cols, T, segs, needed = _cp_layout(d)
    C = cols // 2
    bufs = [_at(p, B * T * cols, torch.bfloat16).view(B, T, cols) for p in _ptr_list(d["peer_bufs"], world)]
    src = _at(d["src"], (B * Tl - 1) * d["src_ld"] + 3 * C, torch.bfloat16)
    rows = torch.as_strided(src, (B, Tl, cols), (Tl * d["src_ld"], d["src_ld"], 1), C)
    for g0, l0, n in segs:
        bufs[rank][:, g0:g0 + n] = rows[:, l0:l0 + n]
    dist.barrier(group=_group(d["peer_flags"]))
    for g0, n, q in needed:
        bufs[rank][:, g0:g0 + n] = bufs[q][:, g0:g0 + n]
    dist.barrier(group=_group(d["peer_flags"]))


def cp_kv_publish(d, stream=0):
    """This rank's k/v rows (local order) into its compact buffer, then the
    epoch into word ``rank`` of every peer's publish buffer."""
    rank, world, B, Tl, cols = d["rank"], d["world"], d["B"], d["Tl"], d["cols"]
    C = cols // 2
    own = _at(_ptr_list(d["peer_bufs"], world)[rank], B * Tl * cols, torch.bfloat16).view(B, Tl, cols)
    src = _at(d["src"], (B * Tl - 1) * d["src_ld"] + 3 * C, torch.bfloat16)
    own.copy_(torch.as_strided(src, (B, Tl, cols), (Tl * d["src_ld"], d["src_ld"], 1), C))
    for p in _ptr_list(d["peer_flags"], world):
        _at(p, 16, torch.int32)[rank] = int(d["epoch"])


def _owner_kv(peers, B, Tk):
    """Natural-order [B, Tk, C] keys and values rebuilt from the owners'
    compact buffers, once every owner's publish word has reached the epoch
    (bounded wait: the owners are other processes)."""
    bases, Tl, zz = peers["bases"], peers["Tl"], peers["zigzag"]
    world, C, st = len(bases), peers["v_off"], peers["st"]
    flags = _at(peers["flags"], world, torch.int32)
    deadline = time.monotonic() + 60.0
    while any(int(flags[q]) < peers["epoch"] for q in range(world)):
        if time.monotonic() > deadline:
            raise RuntimeError(f"publish words {flags.tolist()} never reached epoch {peers['epoch']}")
        time.sleep(0.001)
    bufs = [_at(b, B * peers["sb"], torch.bfloat16).view(B, Tl, st) for b in bases]
    K = torch.zeros(B, Tk, C, dtype=torch.bfloat16)
    V = torch.zeros(B, Tk, C, dtype=torch.bfloat16)
    span = Tl // 2 if zz else Tl
    for k0 in range(0, Tk, span):
        c = k0 // span
        if zz:
            q, r0 = (c, 0) if c < world else (2 * world - 1 - c, span)
        else:
            q, r0 = c, 0
        n = min(span, Tk - k0)
        K[:, k0:k0 + n] = bufs[q][:, r0:r0 + n, :C]
        V[:, k0:k0 + n] = bufs[q][:, r0:r0 + n, C:2 * C]
    return K.reshape(B * Tk, C), V.reshape(B * Tk, C)


def attention_fwd_peers(q, o, lse, B, H, Tq, Tk, q_offset, peers, q_rows=None, kv_heads=None, scale=None):
    K, V = _owner_kv(peers, B, Tk)
    attention_fwd(q, K, V, o, lse, B, H, Tq, Tk=Tk, q_offset=q_offset, scale=scale, q_rows=q_rows,
                  kv_heads=kv_heads)


def attention_bwd_peers(q, o, dout, dq, dk, dv, lse, delta, B, H, Tq, Tk, q_offset, peers, kv_rows=None,
                        q_rows=None, kv_heads=None, scale=None):
    K, V = _owner_kv(peers, B, Tk)
    kr = Tk if kv_rows is None else kv_rows
    # the kernels write dK / dV at their natural rows of a kr-row buffer
    gk = torch.zeros(B * Tk, dk.shape[-1], dtype=dk.dtype)
    gv = torch.zeros_like(gk)
    attention_bwd(q, K, V, o, dout, dq, gk, gv, lse, delta, B, H, Tq, Tk=Tk, q_offset=q_offset, scale=scale,
                  q_rows=q_rows, kv_heads=kv_heads)
    for b in range(B):
        dk[b * kr: b * kr + Tk].copy_(gk[b * Tk:(b + 1) * Tk])
        dv[b * kr: b * kr + Tk].copy_(gv[b * Tk:(b + 1) * Tk])


def cp_kv_reduce(d, stream=0):
    rank, world, B, Tl, cols, T, segs, _ = _cp_layout(d)
    C = cols // 2
    dist.barrier(group=_group(d["peer_flags"]))
    parts1 = [_at(p, B * T * cols, torch.bfloat16).view(B, T, cols) for p in _ptr_list(d["peer_bufs"], world)]
    parts2 = ([_at(p, B * T * cols, torch.bfloat16).view(B, T, cols) for p in _ptr_list(d["peer_bufs2"], world)]
              if d.get("zigzag", 0) else None)
    out = _at(d["out_bf16"], (B * Tl - 1) * d["src_ld"] + 3 * C, torch.bfloat16)
    dst = torch.as_strided(out, (B, Tl, cols), (Tl * d["src_ld"], d["src_ld"], 1), C)
    for g0, l0, n in segs:
        acc = torch.zeros(B, n, cols)
        for q in range(world):
            if parts2 is None:
                if q >= rank:
                    acc += parts1[q][:, g0:g0 + n].float()
                continue
            h = Tl // 2
            k = g0 // h
            if k <= q:
                acc += parts1[q][:, g0:g0 + n].float()
            if k <= 2 * world - 1 - q:
                acc += parts2[q][:, g0:g0 + n].float()
        dst[:, l0:l0 + n] = acc.to(torch.bfloat16)
    dist.barrier(group=_group(d["peer_flags"]))


# ------------------------------------------------------ fused all-reduce --
def allreduce_p2p(peer_bufs, peer_flags, rank, world, offset, n, dtype, scale, epoch, counter, err,
                  nblocks, budget_ns, count, stream):
    """Sum of every rank's [offset, offset + n) elements, times `scale`,
    left in every rank's buffer (the fused kernel's contract)."""
    if n <= 0:
        return
    dt = torch.float32 if dtype == 0 else torch.bfloat16
    esz = 4 if dtype == 0 else 2
    bufs = [_at(p + offset * esz, n, dt) for p in _ptr_list(peer_bufs, world)]
    dist.barrier(group=_group(peer_flags))
    total = sum(b.float() for b in bufs) * scale
    dist.barrier(group=_group(peer_flags))
    bufs[rank].copy_(total)
    if counter:
        c = _at(counter, 1, torch.int64)
        c += (n if count < 0 else count) * esz
    dist.barrier(group=_group(peer_flags))


allreduce_p2p_slim = allreduce_p2p  # same contract, fewer threads per CTA on the GPU


def allreduce_mc(peer_bufs, peer_flags, mc_base, rank, world, offset, n, dtype, scale, epoch, counter,
                 err, nblocks, budget_ns, count, stream):
    """The multimem form: the same result through the switch."""
    esz = 4 if dtype == 0 else 2
    if not mc_base:
        raise RuntimeError("allreduce_mc failed (code -4)")
    if (n * esz) % 16:
        raise RuntimeError("allreduce_mc failed (code -2)")
    allreduce_p2p(peer_bufs, peer_flags, rank, world, offset, n, dtype, scale, epoch, counter, err,
                  nblocks, budget_ns, count, stream)


# ------------------------------------------- tensor-parallel row collectives --
def _peers(d, key="peer_bufs"):
    return _ptr_list(d[key], d["world"])


def tp_ag_rows(d, stream=0):
    rank, world, rows, cols = d["rank"], d["world"], d["rows"], d["cols"]
    bufs = [_at(p, world * rows * cols, torch.bfloat16).view(world * rows, cols) for p in _peers(d)]
    dist.barrier(group=_group(d["peer_flags"]))
    if not d.get("pushed"):  # pushed: the producer already stored its rows everywhere
        for q in range(world):
            if q != rank:
                bufs[rank][q * rows:(q + 1) * rows] = bufs[q][q * rows:(q + 1) * rows]
    dist.barrier(group=_group(d["peer_flags"]))


def tp_rs_rows(d, stream=0):
    rank, world, rows, cols = d["rank"], d["world"], d["rows"], d["cols"]
    bufs = [_at(p, world * rows * cols, torch.bfloat16).view(world * rows, cols) for p in _peers(d)]
    dist.barrier(group=_group(d["peer_flags"]))
    acc = torch.zeros(rows, cols)
    if d.get("inbox"):  # slot q of the local inbox holds peer q's partial of these rows
        inbox = _at(d["inbox"], world * rows * cols, torch.bfloat16).view(world, rows, cols)
        for q in range(world):
            acc += inbox[q].float()
    else:
        for q in range(world):
            acc += bufs[q][rank * rows:(rank + 1) * rows].float()
    if d.get("bias"):
        acc += _at(d["bias"], cols, torch.bfloat16).float()
    if d.get("resid"):
        acc += _at(d["resid"], rows * cols, torch.float32).view(rows, cols)
    if d.get("out_f32"):
        _at(d["out_f32"], rows * cols, torch.float32).view(rows, cols).copy_(acc)
    if d.get("out_bf16"):
        _at(d["out_bf16"], rows * cols, torch.bfloat16).view(rows, cols).copy_(acc)
    dist.barrier(group=_group(d["peer_flags"]))


def tp_embed_fwd(d, stream=0):
    rank, world, rows, cols, T, vpr = d["rank"], d["world"], d["rows"], d["cols"], d["T"], d["vocab_per_rank"]
    tables = [_at(p, vpr * cols, torch.bfloat16).view(vpr, cols) for p in _peers(d)]
    idx = _at(d["idx"], world * rows, torch.int64)
    wpe = _at(d["wpe"], T * cols, torch.bfloat16).view(T, cols)
    out = _at(d["out_f32"], rows * cols, torch.float32).view(rows, cols)
    dist.barrier(group=_group(d["peer_flags"]))
    for i in range(rows):
        m = rank * rows + i
        tok = int(idx[m])
        out[i] = tables[tok // vpr][tok % vpr].float() + wpe[m % T].float()
    dist.barrier(group=_group(d["peer_flags"]))


def tp_embed_bwd(d, stream=0):
    rank, world, rows, cols, T, vpr = d["rank"], d["world"], d["rows"], d["cols"], d["T"], d["vocab_per_rank"]
    grads = [_at(p, vpr * cols, torch.float32).view(vpr, cols) for p in _peers(d)]
    idx = _at(d["idx"], world * rows, torch.int64)
    dx = _at(d["resid"], rows * cols, torch.float32).view(rows, cols)
    wpe_g = _at(d["out_f32"], T * cols, torch.float32).view(T, cols)
    dist.barrier(group=_group(d["peer_flags"]))
    for r in range(world):          # one rank at a time: the kernel's atomics
        if r == rank:
            for i in range(rows):
                m = rank * rows + i
                tok = int(idx[m])
                grads[tok // vpr][tok % vpr] += dx[i]
                wpe_g[m % T] += dx[i]
        dist.barrier(group=_group(d["peer_flags"]))


def tp_ce_stats(d, stream=0):
    rows, ld, vv, v0 = d["rows"], d["ld"], d["vocab_valid"], d["vocab_start"]
    lg = _at(d["logits"], rows * ld, torch.bfloat16).view(rows, ld)[:, :vv].float()
    tgt = _at(d["idx"], rows, torch.int64)
    st = _at(d["stats"], rows * 4, torch.float32).view(rows, 4)
    if vv == 0:   # a slice of padding only
        st.copy_(torch.tensor([float("-inf"), 0.0, 0.0, 0.0]).expand(rows, 4))
        return
    m = lg.max(-1).values
    st[:, 0] = m
    st[:, 1] = torch.exp(lg - m[:, None]).sum(-1)
    t = tgt - v0
    local = (tgt != -100) & (t >= 0) & (t < vv)
    tt = torch.where(local, t, torch.zeros_like(t))
    st[:, 2] = torch.where(local, lg.gather(1, tt[:, None])[:, 0], torch.zeros(rows))
    st[:, 3] = local.float()


def tp_ce_finish(d, stream=0):
    rows, world, ld, vv, v0 = d["rows"], d["world"], d["ld"], d["vocab_valid"], d["vocab_start"]
    stats = [_at(p, rows * 4, torch.float32).view(rows, 4) for p in _peers(d)]
    tgt = _at(d["idx"], rows, torch.int64)
    logits = _at(d["logits"], rows * ld, torch.bfloat16).view(rows, ld)
    loss_rows = _at(d["loss_rows"], rows, torch.float32)
    dist.barrier(group=_group(d["peer_flags"]))
    S = torch.stack([s.clone() for s in stats])          # [world, rows, 4]
    gm = S[:, :, 0].max(0).values
    tot = (S[:, :, 1] * torch.exp(S[:, :, 0] - gm)).sum(0)
    lse = gm + torch.log(tot)
    tl = (S[:, :, 2] * S[:, :, 3]).sum(0)
    ignore = tgt == -100
    loss_rows.copy_(torch.where(ignore, torch.zeros(rows), lse - tl))
    g = torch.exp(logits[:, :vv].float() - gm[:, None]) / tot[:, None]
    t = tgt - v0
    hit = (~ignore) & (t >= 0) & (t < vv)
    g[hit.nonzero()[:, 0], t[hit]] -= 1.0
    g[ignore] = 0.0
    logits[:, :vv] = g.to(torch.bfloat16)
    logits[:, vv:] = 0
    dist.barrier(group=_group(d["peer_flags"]))


def loss_reduce(loss_rows, targets, M, out, stream=0):
    lr = _at(loss_rows, M, torch.float32)
    tg = _at(targets, M, torch.int64)
    o = _at(out, 2, torch.float32)
    count = max(int((tg != -100).sum()), 1)
    o[0] = lr.sum() / count
    o[1] = 1.0 / count


# ---------------------------------------------------------------- ZeRO-2/3 --
def _zero_table(d):
    t = _at(d["buckets"], 4 * d["nb"], torch.int64).view(d["nb"], 4)
    return [tuple(int(x) for x in row) for row in t]


def _zero_slice(row, rank):
    lo, hi, s, off = row
    f0 = lo + rank * s
    return f0, max(0, min(hi, f0 + s) - f0), off


def _bump(counter, nbytes):
    if counter:
        c = _at(counter, 1, torch.int64)
        c += int(nbytes)


def zero_rs(d, stream=0):
    """This rank's slice of bucket `bucket`, summed over the ranks in rank
    order and scaled, into its gradient shard; per-bucket sum of squares."""
    rank, world = d["rank"], d["world"]
    tab = _zero_table(d)
    ext = max(r[1] for r in tab)
    wire16 = bool(d.get("peer_grad16"))
    grads = ([_at(p, ext, torch.bfloat16) for p in _ptr_list(d["peer_grad16"], world)] if wire16
             else [_at(p, ext, torch.float32) for p in _ptr_list(d["peer_grad"], world)])
    b = d["bucket"]
    f0, n, off = _zero_slice(tab[b], rank)
    dist.barrier(group=_group(d["peer_flags"]))
    parts = (_at(d["sumsq_parts"], d["nb"] * d["rs_blocks"], torch.float32) if d.get("sumsq_parts")
             else None)
    if parts is not None:
        parts[b * d["rs_blocks"]:(b + 1) * d["rs_blocks"]] = 0
    if n:
        acc = torch.zeros(n)
        for q in range(world):
            acc += grads[q][f0:f0 + n].float()
        acc *= d["scale"]
        _at(d["gsh"], off + n, torch.float32)[off:off + n] = acc
        if parts is not None:
            parts[b * d["rs_blocks"]] = (acc * acc).sum()
    _bump(d.get("byte_counter"), (tab[b][1] - tab[b][0]) * (2 if wire16 else 4))
    dist.barrier(group=_group(d["peer_flags"]))


def zero_adamw_ag(d, nblocks, stream=0):
    """Global norm from every rank's sums of squares, clip, AdamW on the
    owned slices, the bf16 result written into every rank's parameters."""
    rank, world = d["rank"], d["world"]
    tab = _zero_table(d)
    ext = max(r[1] for r in tab)
    shard = max(off + s for (_, _, s, off) in tab)
    local = _at(d["sumsq_parts"], d["nb"] * d["rs_blocks"], torch.float32).sum().reshape(1)
    allss = [torch.zeros(1) for _ in range(world)]
    dist.all_gather(allss, local, group=_group(d["peer_flags"]))
    norm = math.sqrt(float(sum(float(x) for x in allss)))
    clip = min(d["max_norm"] / (norm + 1e-6), 1.0) if d["max_norm"] > 0 else 1.0
    if d.get("norm_out"):
        _at(d["norm_out"], 1, torch.float32)[0] = norm
    hp = _at(d["hp"], 8, torch.float32)
    master, gsh = _at(d["master"], shard, torch.float32), _at(d["gsh"], shard, torch.float32)
    m, v = _at(d["exp_avg"], shard, torch.float32), _at(d["exp_avg_sq"], shard, torch.float32)
    ranges = _at(d["decay_ranges"], 2 * d["nr"], torch.int64).tolist() if d["nr"] else []
    shadows = [_at(p, ext, torch.bfloat16) for p in _ptr_list(d["peer_shadow"], world)]
    dist.barrier(group=_group(d["peer_flags"]))
    for row in tab:
        f0, n, off = _zero_slice(row, rank)
        if not n:
            continue
        sl = slice(off, off + n)
        decay = torch.zeros(n, dtype=torch.bool)
        for lo, hi in zip(ranges[::2], ranges[1::2]):
            a, b = max(lo, f0), min(hi, f0 + n)
            if a < b:
                decay[a - f0:b - f0] = True
        lr, b1, b2, eps, wd, bc1, bc2s, gsc = [float(hp[i]) for i in range(8)]
        gj = gsh[sl] * (gsc * clip)
        pm, mm, vv = master[sl], m[sl], v[sl]
        pm.mul_(torch.where(decay, 1.0 - lr * wd, 1.0))
        mm.add_((gj - mm) * (1.0 - b1))
        vv.mul_(b2).add_((1.0 - b2) * gj * gj)
        pm.add_(-(lr / bc1) * (mm / (vv.sqrt() / bc2s + eps)))
        for r in range(world):
            shadows[r][f0:f0 + n] = master[sl].to(torch.bfloat16)
    _bump(d.get("byte_counter"), sum(r[1] - r[0] for r in tab) * 2 + 4)
    dist.barrier(group=_group(d["peer_flags"]))


def zero_ag(d, nblocks, stream=0):
    world, span, slc, off = d["world"], d["ag_span"], d["ag_slice"], d["ag_offset"]
    shards = [_at(p + off * 2, slc, torch.bfloat16) for p in _ptr_list(d["peer_shard"], world)]
    dst = _at(d["gather_dst"], span, torch.bfloat16)
    dist.barrier(group=_group(d["peer_flags"]))
    for e0 in range(0, span, slc):
        n = min(slc, span - e0)
        dst[e0:e0 + n] = shards[e0 // slc][:n]
    _bump(d.get("byte_counter"), span * 2)
    dist.barrier(group=_group(d["peer_flags"]))


class _Stream:
    cuda_stream = 0

    def __init__(self, *a, **k):
        pass

    def wait_event(self, ev):
        pass

    def wait_stream(self, other):
        pass


@contextmanager
def _stream_ctx(s):
    yield


class _Event:
    def record(self, *a, **k):
        pass

    def synchronize(self):
        pass

    def query(self):
        return True


OPS = {
    "gemm": gemm, "layernorm_fwd": layernorm_fwd, "layernorm_bwd": layernorm_bwd,
    "layernorm_bwd_partials": layernorm_bwd_partials, "colsum_bf16": colsum_bf16, "colsum_f32": colsum_f32,
    "embedding_fwd": embedding_fwd, "embedding_bwd": embedding_bwd,
    "cross_entropy_fwd_bwd": cross_entropy_fwd_bwd, "lm_head_cross_entropy": lm_head_cross_entropy,
    "attention_fwd": attention_fwd,
    "attention_bwd": attention_bwd, "attention_fwd_peers": attention_fwd_peers,
    "attention_bwd_peers": attention_bwd_peers, "grad_sumsq": grad_sumsq, "clip_coef": clip_coef,
    "adamw_step": adamw_step, "cast_f32_bf16": cast_f32_bf16, "cast_bf16_f32": cast_bf16_f32, "decode_embed": decode_embed,
    "decode_partials": decode_partials, "decode_attn": decode_attn, "decode_argmax": decode_argmax,
}

LIB = SimpleNamespace(zero_rs=zero_rs, zero_adamw_ag=zero_adamw_ag, zero_ag=zero_ag,
                      zero_flag_words=lambda: 16, zero_norm_words=lambda: 16, zero_max_blocks=lambda: 160,
                      cp_kv_gather=cp_kv_gather, cp_kv_reduce=cp_kv_reduce, tp_flag_words=lambda: 16,
                      cp_kv_publish=cp_kv_publish, kv_publish_words=lambda: 16,
                      allreduce_p2p=allreduce_p2p, allreduce_p2p_slim=allreduce_p2p_slim, allreduce_mc=allreduce_mc, comm_flag_words=lambda: 16, tp_ag_rows=tp_ag_rows,
                      tp_rs_rows=tp_rs_rows, tp_embed_fwd=tp_embed_fwd, tp_embed_bwd=tp_embed_bwd,
                      tp_ce_stats=tp_ce_stats, tp_ce_finish=tp_ce_finish, loss_reduce=loss_reduce,
                      embedding_wte_det_chunks=lambda M: -(-M // 128))


@contextmanager
def installed(monkeypatch):
    """Route the native-op calls and the CUDA runtime calls around them to
    the torch versions for the duration of a test (pytest ``monkeypatch``)."""
    from gpt2_harness_b200.models import engine as engine_mod

    for name, fn in OPS.items():
        monkeypatch.setattr(N, name, fn)
    from gpt2_harness_b200.parallel import cp_native, ddp_native, symm, tp_native, zero3_native, zero_native

    monkeypatch.setattr(N, "lib", lambda: LIB)
    monkeypatch.setattr(N, "check_errors", lambda *a, **k: None)
    monkeypatch.setattr(N, "error_word", lambda *a, **k: torch.zeros(1, dtype=torch.int32))
    monkeypatch.setattr(cp_native, "SymmetricBuffer", FakeSymmetricBuffer)
    monkeypatch.setattr(ddp_native, "SymmetricBuffer", FakeSymmetricBuffer)
    monkeypatch.setattr(ddp_native, "MulticastBuffer", FakeMulticastBuffer)
    monkeypatch.setattr(symm, "SymmetricBuffer", FakeSymmetricBuffer)
    monkeypatch.setattr(tp_native, "SymmetricBuffer", FakeSymmetricBuffer)
    monkeypatch.setattr(zero_native, "SymmetricBuffer", FakeSymmetricBuffer)
    monkeypatch.setattr(zero3_native, "SymmetricBuffer", FakeSymmetricBuffer)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())
    monkeypatch.setattr(torch.cuda, "Stream", _Stream)
    monkeypatch.setattr(torch.cuda, "stream", _stream_ctx)
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
