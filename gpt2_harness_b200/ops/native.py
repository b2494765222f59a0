"""Loader and thin, validated Python wrappers over the sm_100a native library.

The shared object ``gpt2_harness_b200/_C*.so`` is built in-tree by
``python setup.py build_ext --inplace`` (or ``__graft_entry__.build()``). On a
machine with a CUDA device the library MUST load: :func:`lib` raises instead of
silently falling back to PyTorch, so a test that passes has run our kernels.

Every wrapper checks shapes, dtypes, contiguity and alignment on the host and
then passes raw device addresses plus the current CUDA stream to the launcher,
so the launch itself is one pybind call and is capturable in a CUDA graph.
"""

from __future__ import annotations

import importlib
import math
from typing import Optional

import torch

__all__ = [
    "lib",
    "available",
    "error_word",
    "check_errors",
    "EPI_BF16",
    "EPI_BIAS_GELU",
    "EPI_RESID_F32",
    "EPI_F32",
    "EPI_GELU_BWD",
    "gemm",
    "linear_fwd",
    "attention_fwd",
    "attention_bwd",
    "attention_fwd_peers",
    "attention_bwd_peers",
    "layernorm_fwd",
    "layernorm_bwd",
    "colsum_bf16",
    "embedding_fwd",
    "embedding_bwd",
    "cross_entropy_fwd_bwd",
    "CEWorkspace",
    "lm_head_cross_entropy",
    "EmbeddingGradWorkspace",
    "adamw_step",
]

EPI_BF16, EPI_BIAS_GELU, EPI_RESID_F32, EPI_F32, EPI_GELU_BWD, EPI_CE_STATS = 0, 1, 2, 3, 4, 5

_LIB = None
_LOAD_ERROR: Optional[BaseException] = None
_ERR_WORDS: dict[int, torch.Tensor] = {}

ERROR_NAMES = {
    1 << 0: "GEMM producer wait timed out",
    1 << 1: "GEMM MMA wait timed out",
    1 << 2: "GEMM epilogue wait timed out",
    1 << 3: "peer flag wait timed out",
    1 << 4: "bad shape",
    1 << 5: "attention pipeline wait timed out",
}


def lib():
    """The native module. Raises ImportError with the build hint if absent."""
    global _LIB, _LOAD_ERROR
    if _LIB is None:
        try:
            _LIB = importlib.import_module("gpt2_harness_b200._C")
        except BaseException as exc:  # pragma: no cover - depends on the build
            _LOAD_ERROR = exc
            raise ImportError(
                "gpt2_harness_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"(original error: {exc!r})"
            ) from exc
    return _LIB


def available() -> bool:
    """True when the native library imports and a CUDA device is present."""
    if not torch.cuda.is_available():
        return False
    try:
        lib()
    except ImportError:
        return False
    return True


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def error_word(device: Optional[torch.device] = None) -> torch.Tensor:
    """Per-device uint32 word the kernels OR their error codes into."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in _ERR_WORDS:
        _ERR_WORDS[key] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
    return _ERR_WORDS[key]


def _err_ptr() -> int:
    return error_word().data_ptr()


def check_errors(device: Optional[torch.device] = None, reset: bool = True) -> None:
    """Raise RuntimeError if any kernel on `device` recorded an error (syncs)."""
    w = error_word(device)
    val = int(w.item())
    if val:
        if reset:
            w.zero_()
        names = [n for bit, n in ERROR_NAMES.items() if val & bit]
        raise RuntimeError(f"native kernel error 0x{val:x}: {', '.join(names) or 'unknown'}")


def _ptr(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.data_ptr()


def _row_stride(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"expected a 2-D row-major view, got shape {tuple(t.shape)} strides {t.stride()}")
    return t.stride(0)


def _check_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("native ops need CUDA tensors")


# ---------------------------------------------------------------------- GEMM --
def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    a_t: bool = False,
    b_t: bool = False,
    epilogue: int = EPI_BF16,
    bias: Optional[torch.Tensor] = None,
    aux: Optional[torch.Tensor] = None,
    alpha: float = 1.0,
    alpha_ptr: Optional[torch.Tensor] = None,
    accumulate: bool = False,
    splits: int = 1,
    workspace: Optional[torch.Tensor] = None,
    bn: int = 256,
    max_ctas: int = 0,
    pair: int = -1,
    ce: Optional["CEWorkspace"] = None,
    ce_targets: Optional[torch.Tensor] = None,
    ce_vocab_offset: int = 0,
    owner_out: Optional[tuple] = None,
) -> torch.Tensor:
    """out[M,N] (epilogue) = op(a) @ op(b)^T on the tcgen05 tensor cores.

    ``a`` is [M, K] (or [K, M] with ``a_t``), ``b`` is [N, K] (or [K, N] with
    ``b_t``), both bf16 row-major views. ``a_t``/``b_t`` select the MN-major
    operand layout in the kernel: no transpose is ever materialised.
    ``pair`` = 1 runs 256x256 tiles on pairs of CTAs (one cta_group::2 MMA per
    pair), 0 one CTA per 128 x ``bn`` tile, -1 the library's default.
    ``EPI_CE_STATS`` (the lm_head forward) also needs ``ce`` (a
    :class:`CEWorkspace`) and the int64 ``ce_targets``.
    ``owner_out = (bases, rows[, self])`` stores row m of the (bf16) result at
    bases[m // rows] + (m % rows) * ldo instead of into ``out``: tensor
    parallelism's GEMM -> reduce-scatter, each partial row written straight
    into its owner's inbox. With ``self``, ``out`` is this GPU's inbox and the
    tiles of its own rows keep the TMA-store path.
    """
    _check_cuda(a, b, out, bias, aux, alpha_ptr, workspace)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("gemm operands must be bf16")
    M, K = (a.shape[1], a.shape[0]) if a_t else (a.shape[0], a.shape[1])
    if b_t:
        N, Kb = b.shape[1], b.shape[0]
    else:
        N, Kb = b.shape[0], b.shape[1]
    if K != Kb:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    if out.shape[0] != M or out.shape[1] < N:
        raise ValueError(f"out shape {tuple(out.shape)} cannot hold [{M}, {N}]")
    want = torch.float32 if epilogue in (EPI_RESID_F32, EPI_F32) else torch.bfloat16
    if out.dtype != want:
        raise TypeError(f"epilogue {epilogue} writes {want}, out is {out.dtype}")
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() < N):
        raise TypeError("bias must be bf16 with at least N elements")
    if epilogue in (EPI_BIAS_GELU, EPI_GELU_BWD) and (aux is None or aux.dtype != torch.bfloat16):
        raise TypeError("this epilogue needs a bf16 aux tensor")
    if epilogue == EPI_RESID_F32 and aux is not None and aux.dtype != torch.float32:
        raise TypeError("the residual epilogue's source (aux) must be fp32")
    if splits > 1:
        if epilogue != EPI_F32:
            raise ValueError("split-K needs the fp32 epilogue")
        if workspace is None or workspace.numel() < splits * M * N:
            raise ValueError("split-K workspace too small")
    ce_ptrs = (0, 0, 0)
    if epilogue == EPI_CE_STATS:
        if ce is None or ce_targets is None or ce_targets.dtype != torch.int64:
            raise TypeError("EPI_CE_STATS needs a CEWorkspace and int64 targets")
        if ce.M != M or ce.nparts < CEWorkspace.parts(N) or ce_targets.numel() != M:
            raise ValueError("CEWorkspace / targets do not match the GEMM shape")
        if bias is not None or splits > 1:
            raise ValueError("EPI_CE_STATS takes no bias and no split-K")
        bn = 256
        ce_ptrs = (ce.stats.data_ptr(), ce_targets.data_ptr(), ce.tgt_logit.data_ptr())
    lib().gemm(
        a.data_ptr(), _row_stride(a), int(a_t), b.data_ptr(), _row_stride(b), int(b_t),
        M, N, K, epilogue, out.data_ptr(), _row_stride(out), _ptr(aux),
        0 if aux is None else _row_stride(aux), _ptr(bias), float(alpha), _ptr(alpha_ptr),
        int(accumulate), int(splits), _ptr(workspace), int(bn), int(max_ctas), int(pair),
        ce_ptrs[0], ce_ptrs[1], ce_ptrs[2], int(ce_vocab_offset),
        0 if owner_out is None else owner_out[0].data_ptr(),
        0 if owner_out is None else int(owner_out[1]),
        -1 if owner_out is None or len(owner_out) < 3 else int(owner_out[2]), _err_ptr(), _stream(),
    )
    return out


def linear_fwd(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w^T + bias with bf16 I/O (nn.Linear layout: w is [out, in])."""
    y = torch.empty(x.shape[0], w.shape[0], dtype=torch.bfloat16, device=x.device)
    return gemm(x, w, y, bias=bias)


# ----------------------------------------------------------------- attention --
def _head_strides(t: torch.Tensor, T: int, H: int):
    # t is [B*T, >=H*64] row-major; element (b,h,t,d) at b*T*ld + t*ld + h*64 + d
    ld = _row_stride(t)
    return T * ld, ld, 64


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                  lse: torch.Tensor, B: int, H: int, Tq: int, Tk: Optional[int] = None,
                  q_offset: int = 0, causal: bool = True, scale: Optional[float] = None,
                  kv_rows: Optional[int] = None, q_rows: Optional[int] = None,
                  kv_heads: Optional[int] = None) -> None:
    """Causal flash attention on head_dim 64.

    q, o: [B*Tq, ...] row-major views whose columns h*64..h*64+63 hold head h
    (e.g. the q section of the fused qkv buffer); k, v: [B*Tk, ...] likewise.
    kv_heads: key/value heads (grouped-query attention, reference model.py:
    272-278): query head h reads key/value head h // (H // kv_heads) by index,
    nothing is repeated in memory. Defaults to H.
    lse: fp32 [B, H, Tq] (log2-domain log-sum-exp, saved for backward).
    kv_rows: rows per sequence in the k/v buffers when they hold more than the
    Tk keys attended (context parallelism: a full-length key buffer of which
    a prefix is visible); defaults to Tk.
    q_rows: rows per sequence in the q/o buffers when each sequence's Tq
    queries are a slice of a longer row range (load-balanced context
    parallelism: two chunks per sequence); defaults to Tq.
    """
    Tk = Tq if Tk is None else Tk
    qr = Tq if q_rows is None else q_rows
    scale = 1.0 / math.sqrt(64) if scale is None else scale
    qsb, qst, qsh = _head_strides(q, qr, H)
    ksb, kst, ksh = _head_strides(k, Tk if kv_rows is None else kv_rows, H)
    if _head_strides(v, Tk if kv_rows is None else kv_rows, H) != (ksb, kst, ksh):
        raise ValueError("k and v must share strides")
    osb, ost, osh = _head_strides(o, qr, H)
    lib().attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), qsb, qst, qsh,
                   osb, ost, osh, lse.data_ptr(), B, H, kv_heads or H, Tq, Tk, q_offset,
                   int(causal), float(scale), ksb, kst, ksh, _err_ptr(), _stream())


def attention_bwd(q, k, v, o, dout, dq, dk, dv, lse, delta, B: int, H: int, Tq: int,
                  Tk: Optional[int] = None, q_offset: int = 0, causal: bool = True,
                  scale: Optional[float] = None, kv_rows: Optional[int] = None,
                  q_rows: Optional[int] = None, kv_heads: Optional[int] = None) -> None:
    """Deterministic flash-attention backward (dK/dV pass, then dQ pass).

    dout shares o's strides; dq shares q's layout family; dk/dv share a layout.
    delta: fp32 scratch [B, H, Tq]. kv_rows / q_rows / kv_heads as in
    :func:`attention_fwd`; with grouped heads each key/value tile sums the
    gradients of every query head of its group in one pass (no atomics).
    """
    Tk = Tq if Tk is None else Tk
    kr = Tk if kv_rows is None else kv_rows
    qr = Tq if q_rows is None else q_rows
    scale = 1.0 / math.sqrt(64) if scale is None else scale
    qsb, qst, qsh = _head_strides(q, qr, H)
    ksb, kst, ksh = _head_strides(k, kr, H)
    osb, ost, osh = _head_strides(o, qr, H)
    if _head_strides(dout, qr, H) != (osb, ost, osh):
        raise ValueError("dout must share o's strides")
    dsb, dst, dsh = _head_strides(dq, qr, H)
    dksb, dkst, dksh = _head_strides(dk, kr, H)
    if _head_strides(dv, kr, H) != (dksb, dkst, dksh):
        raise ValueError("dk and dv must share strides")
    lib().attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
                   dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), qsb, qst, qsh, osb, ost, osh,
                   dsb, dst, dsh, lse.data_ptr(), delta.data_ptr(), B, H, kv_heads or H, Tq, Tk,
                   q_offset, int(causal), float(scale), ksb, kst, ksh, dksb, dkst, dksh, _err_ptr(),
                   _stream())


def _peer_args(peers: dict) -> tuple:
    return (list(peers["bases"]), int(peers["sb"]), int(peers["st"]), int(peers["v_off"]),
            int(peers["Tl"]), int(peers["zigzag"]), int(peers["flags"]), int(peers["epoch"]) & 0xFFFFFFFF)


def attention_fwd_peers(q: torch.Tensor, o: torch.Tensor, lse: torch.Tensor, B: int, H: int, Tq: int,
                        Tk: int, q_offset: int, peers: dict, q_rows: Optional[int] = None,
                        kv_heads: Optional[int] = None, scale: Optional[float] = None) -> None:
    """Causal attention whose keys and values are read in place from their
    owners (context parallelism, streaming form): ``peers`` describes every
    rank's compact key/value buffer -- ``bases`` (this process's address of
    rank q's [B, Tl, 2C] bf16 buffer), ``sb`` / ``st`` (element strides of a
    sequence and a row), ``v_off`` (element offset of the value columns),
    ``Tl``, ``zigzag``, ``flags`` (this rank's publish words) and ``epoch``
    (the epoch the owners published these rows under). ``Tk`` counts natural
    key positions; the kernel maps each 64-key block to its owner's rows.
    Tensor-core kernel only: a layout it cannot take raises."""
    qr = Tq if q_rows is None else q_rows
    scale = 1.0 / math.sqrt(64) if scale is None else scale
    qsb, qst, qsh = _head_strides(q, qr, H)
    osb, ost, osh = _head_strides(o, qr, H)
    lib().attn_fwd_peers(q.data_ptr(), o.data_ptr(), qsb, qst, qsh, osb, ost, osh, lse.data_ptr(), B, H,
                         kv_heads or H, Tq, Tk, q_offset, float(scale), *_peer_args(peers), _err_ptr(),
                         _stream())


def attention_bwd_peers(q, o, dout, dq, dk, dv, lse, delta, B: int, H: int, Tq: int, Tk: int,
                        q_offset: int, peers: dict, kv_rows: Optional[int] = None,
                        q_rows: Optional[int] = None, kv_heads: Optional[int] = None,
                        scale: Optional[float] = None) -> None:
    """Backward of :func:`attention_fwd_peers`: keys and values read in place
    from their owners; dK / dV of every key position seen are written to
    ``dk`` / ``dv`` (natural order, ``kv_rows`` rows per sequence) as in
    :func:`attention_bwd`."""
    kr = Tk if kv_rows is None else kv_rows
    qr = Tq if q_rows is None else q_rows
    scale = 1.0 / math.sqrt(64) if scale is None else scale
    qsb, qst, qsh = _head_strides(q, qr, H)
    osb, ost, osh = _head_strides(o, qr, H)
    if _head_strides(dout, qr, H) != (osb, ost, osh):
        raise ValueError("dout must share o's strides")
    dsb, dst, dsh = _head_strides(dq, qr, H)
    dksb, dkst, dksh = _head_strides(dk, kr, H)
    if _head_strides(dv, kr, H) != (dksb, dkst, dksh):
        raise ValueError("dk and dv must share strides")
    lib().attn_bwd_peers(q.data_ptr(), o.data_ptr(), dout.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                         dv.data_ptr(), qsb, qst, qsh, osb, ost, osh, dsb, dst, dsh, lse.data_ptr(),
                         delta.data_ptr(), B, H, kv_heads or H, Tq, Tk, q_offset, float(scale), dksb, dkst,
                         dksh, *_peer_args(peers), _err_ptr(), _stream())


# ----------------------------------------------------------------- layernorm --
def _push_args(push) -> tuple:
    """(device pointer array, count, local base) of a row push, or zeros."""
    if push is None:
        return 0, 0, 0
    bases, n, local = push
    return bases.data_ptr(), int(n), int(local)


def layernorm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, y: torch.Tensor,
                  mean: torch.Tensor, rstd: torch.Tensor, eps: float = 1e-5,
                  push: Optional[tuple] = None) -> torch.Tensor:
    """y(bf16) = LN(x fp32) * gamma + beta over the last dim; saves mean/rstd.

    ``push = (bases, n, local)`` also stores every output row into n peer
    copies of the buffer (int64 device tensor of base addresses; the row at
    address a goes to bases[j] + (a - local)): the all-gather of tensor
    parallelism fused into the LayerNorm that produces the rows."""
    M, C = x.shape
    lib().layernorm_fwd(x.data_ptr(), _row_stride(x), gamma.data_ptr(), beta.data_ptr(),
                        y.data_ptr(), _row_stride(y), mean.data_ptr(), rstd.data_ptr(), M, C,
                        float(eps), *_push_args(push), _stream())
    return y


def layernorm_bwd_partials(M: int, C: int, device) -> torch.Tensor:
    """Scratch for :func:`layernorm_bwd`: one [3, C] fp32 row per CTA cluster."""
    rows = lib().layernorm_bwd_partial_rows(M)
    return torch.empty(rows, 3, C, dtype=torch.float32, device=device)


def layernorm_bwd(dy: torch.Tensor, x: torch.Tensor, mean: torch.Tensor, rstd: torch.Tensor,
                  gamma: torch.Tensor, dres: torch.Tensor, dres_bf16: Optional[torch.Tensor],
                  dgamma: torch.Tensor, dbeta: torch.Tensor, partials: torch.Tensor,
                  accumulate_dres: bool, accumulate_params: bool = True,
                  dsum: Optional[torch.Tensor] = None, accumulate_dsum: bool = False,
                  push: Optional[tuple] = None) -> None:
    """LN backward: dres (+)= dx (fp32, plus optional bf16 copy); dgamma/dbeta (+)=.

    ``push`` (see :func:`layernorm_fwd`) also stores the bf16 copy's rows
    into peer copies of its buffer.

    With ``dsum`` (fp32 [C]), also dsum (+)= the column sum of the written
    dres: the bias gradient of the projection whose output is this residual
    stream, fused here instead of a separate reduction over its bf16 copy.
    """
    M, C = x.shape
    if partials.numel() < lib().layernorm_bwd_partial_rows(M) * 3 * C:
        raise ValueError("layernorm_bwd partials too small")
    lib().layernorm_bwd(dy.data_ptr(), x.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                        gamma.data_ptr(), dres.data_ptr(), _ptr(dres_bf16), partials.data_ptr(),
                        dgamma.data_ptr(), dbeta.data_ptr(), _ptr(dsum), M, C,
                        int(accumulate_dres), int(accumulate_params), int(accumulate_dsum),
                        *_push_args(push), _stream())


def colsum_bf16(x: torch.Tensor, out: torch.Tensor, ws: torch.Tensor, accumulate: bool = True) -> None:
    """out(fp32) (+)= x.sum(0) for a bf16 [M, C] view (bias gradients)."""
    M, C = x.shape
    lib().colsum_bf16(x.data_ptr(), _row_stride(x), M, C, ws.data_ptr(), out.data_ptr(),
                      int(accumulate), _stream())


def colsum_f32(x: torch.Tensor, out: torch.Tensor, accumulate: bool = True) -> None:
    """out (+)= x.sum(0) for a contiguous fp32 [R, C] tensor (fixed order)."""
    R, C = x.shape
    if not x.is_contiguous():
        raise ValueError("colsum_f32 needs a contiguous input")
    lib().colsum_f32(x.data_ptr(), R, C, out.data_ptr(), int(accumulate), _stream())


def colsum_ws_numel(M: int, C: int) -> int:
    return ((M + 127) // 128) * C


# ----------------------------------------------------------------- embedding --
def embedding_fwd(idx: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor, x: torch.Tensor,
                  pos0: int = 0, pos_split: Optional[int] = None, pos1: int = 0) -> torch.Tensor:
    """x = wte[idx] + wpe[pos]; column t of every sequence sits at position
    pos0 + t, or pos1 + (t - pos_split) from ``pos_split`` on."""
    B, T = idx.shape
    C = wte.shape[1]
    split = T if pos_split is None else int(pos_split)
    lib().embedding_fwd(idx.data_ptr(), wte.data_ptr(), wpe.data_ptr(), x.data_ptr(), B, T, C,
                        pos0, split, pos1, _stream())
    return x


class EmbeddingGradWorkspace:
    """Buffers of the deterministic token-embedding gradient for M tokens:
    per-chunk partial rows (fp32 [M, C]) and the [chunks, V] slot table, which
    starts at -1 and is left at -1 by every call."""

    def __init__(self, M: int, C: int, vocab: int, device) -> None:
        self.part = torch.empty(M, C, dtype=torch.float32, device=device)
        chunks = lib().embedding_wte_det_chunks(M)
        self.slots = torch.full((chunks, vocab), -1, dtype=torch.int32, device=device)


def embedding_bwd(idx: torch.Tensor, dx: torch.Tensor, wte_grad: Optional[torch.Tensor],
                  wpe_grad: Optional[torch.Tensor], vocab: int, pos0: int = 0,
                  pos_split: Optional[int] = None, pos1: int = 0,
                  det: Optional[EmbeddingGradWorkspace] = None) -> None:
    """wte_grad[idx[m]] += dx[m] (token embedding) and wpe_grad[pos] += sum over
    the batch (positions), both fp32. With `det` the token sums run in a fixed
    order and are bit-reproducible; without, they use fp32 atomics."""
    B, T = idx.shape
    C = dx.shape[-1]
    split = T if pos_split is None else int(pos_split)
    lib().embedding_bwd(idx.data_ptr(), dx.data_ptr(), _ptr(wte_grad), _ptr(wpe_grad), B, T, C,
                        vocab, pos0, split, pos1, 0 if det is None else det.part.data_ptr(),
                        0 if det is None else det.slots.data_ptr(), _stream())


# --------------------------------------------------------------- cross-entropy --
def cross_entropy_fwd_bwd(logits: torch.Tensor, targets: torch.Tensor, loss_rows: torch.Tensor,
                          loss_out: torch.Tensor, vocab: int) -> None:
    """Loss + in-place dlogits (softmax - onehot) over a bf16 [M, ld] logits view.

    loss_out[0] = mean loss over non-ignored targets, loss_out[1] = 1/count
    (the scale the lm_head backward GEMMs apply through alpha_ptr).
    """
    M = logits.shape[0]
    L = lib()
    L.cross_entropy(logits.data_ptr(), _row_stride(logits), targets.data_ptr(),
                    loss_rows.data_ptr(), M, vocab, 0, _stream())
    L.loss_reduce(loss_rows.data_ptr(), targets.data_ptr(), M, loss_out.data_ptr(), _stream())


class CEWorkspace:
    """Buffers of the fused lm_head + cross-entropy for M rows: the GEMM
    epilogue's (max, sum exp) partials (2 per 256 vocabulary columns), the
    target logits, the per-row log-sum-exp and loss."""

    def __init__(self, M: int, vocab: int, device) -> None:
        self.M = M
        self.nparts = self.parts(vocab)
        self.stats = torch.empty(self.nparts * M * 2, dtype=torch.float32, device=device)
        self.tgt_logit = torch.zeros(M, dtype=torch.float32, device=device)
        self.lse = torch.empty(M, dtype=torch.float32, device=device)
        self.loss_rows = torch.empty(M, dtype=torch.float32, device=device)

    @staticmethod
    def parts(vocab: int) -> int:
        return 2 * (-(-vocab // 256))


def lm_head_cross_entropy(h: torch.Tensor, w: torch.Tensor, logits: torch.Tensor,
                          targets: torch.Tensor, ws: CEWorkspace, loss_out: torch.Tensor,
                          vocab: int) -> None:
    """Fused lm_head + cross-entropy (reference model.py:585,593-598: logits
    = ln_f(x) @ wte^T, then F.cross_entropy with ignore_index -100).

    1. ``logits[:, :vocab] = h @ w^T`` on the tcgen05 GEMM whose epilogue also
       keeps, per row, online (max, sum exp) partials of the bf16 logits and
       picks out the target logit -- no separate statistics pass;
    2. one thread per row folds the partials into log-sum-exp and the loss;
    3. one streaming pass turns the logits into softmax - onehot in place.

    loss_out[0] = mean loss over non-ignored targets, loss_out[1] = 1/count
    (the scale the lm_head backward GEMMs apply through alpha_ptr).
    """
    M = h.shape[0]
    t = targets.reshape(-1)
    gemm(h, w, logits[:, :vocab], epilogue=EPI_CE_STATS, ce=ws, ce_targets=t)
    L = lib()
    L.ce_combine(ws.stats.data_ptr(), ws.nparts, M, t.data_ptr(), ws.tgt_logit.data_ptr(),
                 ws.lse.data_ptr(), ws.loss_rows.data_ptr(), _stream())
    L.loss_reduce(ws.loss_rows.data_ptr(), t.data_ptr(), M, loss_out.data_ptr(), _stream())
    L.ce_grad(logits.data_ptr(), _row_stride(logits), M, vocab, ws.lse.data_ptr(), t.data_ptr(), 0,
              _stream())


def cast_f32_bf16(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out(bf16) = x(fp32), elementwise over contiguous buffers."""
    if x.numel() != out.numel():
        raise ValueError("cast_f32_bf16: sizes differ")
    lib().cast_f32_bf16(x.data_ptr(), out.data_ptr(), x.numel(), _stream())
    return out


def cast_bf16_f32(x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out(fp32) = x(bf16), elementwise over contiguous buffers."""
    if x.numel() != out.numel():
        raise ValueError("cast_bf16_f32: sizes differ")
    lib().cast_bf16_f32(x.data_ptr(), out.data_ptr(), x.numel(), _stream())
    return out


# ---------------------------------------------------------------- optimiser --
def adamw_step(p: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor,
               p_bf16: Optional[torch.Tensor], n_decay: int, hp: torch.Tensor,
               clip: Optional[torch.Tensor] = None,
               decay_ranges: Optional[torch.Tensor] = None) -> None:
    """Fused AdamW over flat fp32 buffers (see csrc/elementwise.cuh for hp).

    Decay applies to ``[0, n_decay)`` or, when ``decay_ranges`` (int64 device
    tensor ``[lo0, hi0, lo1, hi1, ...]``, sorted, 4-aligned) is given, inside
    those ranges.
    """
    nr = 0 if decay_ranges is None else decay_ranges.numel() // 2
    lib().adamw(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), _ptr(p_bf16), p.numel(),
                int(n_decay), _ptr(decay_ranges), nr, hp.data_ptr(), _ptr(clip), _stream())


def grad_sumsq(g: torch.Tensor, ws: torch.Tensor, out: torch.Tensor) -> None:
    lib().sumsq(g.data_ptr(), g.numel(), ws.data_ptr(), out.data_ptr(), _stream())


def clip_coef(sumsq: torch.Tensor, max_norm: float, clip: torch.Tensor,
              norm_out: Optional[torch.Tensor] = None, scale2: float = 1.0) -> None:
    lib().clip_coef(sumsq.data_ptr(), float(scale2), float(max_norm), clip.data_ptr(),
                    _ptr(norm_out), _stream())


# ------------------------------------------------------------------ decoding --
def decode_embed(tok: torch.Tensor, lens: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor,
                 x: torch.Tensor) -> None:
    """x[b] (fp32) = wte[tok[b]] + wpe[lens[b]] with bf16 tables."""
    B, C = x.shape
    lib().decode_embed(tok.data_ptr(), lens.data_ptr(), wte.data_ptr(), wpe.data_ptr(), x.data_ptr(), B, C,
                       _stream())


def decode_partials(B: int, H: int, Tmax: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    n = lib().decode_partials_numel(B, H, Tmax)
    return (torch.empty(n, dtype=torch.float32, device=device),
            torch.empty(n // 32, dtype=torch.float32, device=device))


def decode_attn(qkv: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
                part_o: torch.Tensor, part_ml: torch.Tensor, out: torch.Tensor, H: int, Hkv: int,
                scale: Optional[float] = None) -> None:
    """One decode step of attention with the KV append fused in.

    qkv: [B, (H + 2 Hkv) * 64] bf16 (this step's projections); k_cache/v_cache:
    [B, Hkv, Tmax, 64] bf16; lens: int32 [B] cached positions (the new token's
    k/v are written at lens[b]); out: [B, H * 64] bf16.
    """
    B = qkv.shape[0]
    Tmax = k_cache.shape[2]
    if k_cache.shape != (B, Hkv, Tmax, 64) or v_cache.shape != k_cache.shape:
        raise ValueError("cache must be [B, Hkv, Tmax, 64]")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("cache must be contiguous")
    scale = 1.0 / math.sqrt(64) if scale is None else scale
    lib().decode_attn(qkv.data_ptr(), _row_stride(qkv), k_cache.data_ptr(), v_cache.data_ptr(),
                      lens.data_ptr(), part_o.data_ptr(), part_ml.data_ptr(), out.data_ptr(),
                      _row_stride(out), B, H, Hkv, Tmax, float(scale), _stream())


def decode_argmax(logits: torch.Tensor, vocab: int, tok: torch.Tensor, lens: torch.Tensor,
                  hist: torch.Tensor) -> None:
    """Greedy next token per row: tok[b], hist[b, lens[b] + 1] = argmax; lens += 1."""
    B = logits.shape[0]
    lib().decode_argmax(logits.data_ptr(), _row_stride(logits), vocab, tok.data_ptr(), lens.data_ptr(),
                        hist.data_ptr(), hist.shape[1], B, _stream())
