"""Native GPT-2 training engine for one B200 (and, with a gradient hook, DDP).

The reference trains ``GPT`` through autograd with ``torch.optim.AdamW``
(src/transformer_internals/train.py:184-308, model.py:528-599). This engine
runs the same mathematics as an explicit, preplanned sequence of sm_100a
kernels with no autograd and no per-step allocation:

* **Flat parameter storage.** fp32 master weights, a bf16 shadow the kernels
  read, fp32 gradients, and AdamW moments are four flat buffers sharing one
  layout (:class:`ParamLayout`). Every tensor starts on a 64-element (128-byte)
  boundary so any view is a valid TMA base. The layout is ordered the way
  backward produces gradients (ln_f, blocks L-1 .. 0, then wte/wpe), so DDP
  buckets are contiguous ranges that complete in order.
* **Forward.** embedding -> per block: LN1 -> c_attn GEMM (+bias) -> flash
  attention straight on the fused qkv buffer -> c_proj GEMM whose epilogue adds
  bias and the fp32 residual out of place -> LN2 -> c_fc GEMM with fused
  bias+GELU (pre-activation kept) -> mlp c_proj GEMM with fused residual add ->
  ln_f -> lm_head GEMM into a padded-vocab bf16 logits buffer -> one
  cross-entropy kernel that writes the loss and overwrites the logits with
  dlogits = softmax - onehot (``fused_ce``: statistics in the GEMM epilogue,
  a row fold and one streaming gradient pass instead).
* **Backward.** dgrad GEMMs read weights MN-major (no transposes), the
  mlp dgrad fuses GELU backward, wgrad GEMMs read activations MN-major and
  split K over tokens with a deterministic reduction, LayerNorm backward adds
  into the fp32 residual gradient and emits its bf16 copy, bias gradients are
  deterministic column sums, the 1/N_tokens loss scale enters the lm_head
  GEMMs through a device scalar.
* **Optimiser.** global grad-norm, clip coefficient and AdamW (torch
  single-tensor order, decay on rank>=2 tensors) as two reductions plus one
  fused kernel that also refreshes the bf16 shadow.

Residual-stream and gradient precision follow bf16 autocast with fp32 master
weights: matmul inputs bf16, accumulation and the residual stream fp32.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch

from gpt2_harness_b200.config import GPTConfig
from gpt2_harness_b200.ops import native as N
from gpt2_harness_b200.utils.nvtx import nvtx_range

__all__ = ["ParamSpec", "ParamLayout", "qkv_width", "qkv_views", "CompactLayout", "Engine",
           "OptimConfig", "choose_splits", "init_flat_weights"]

ALIGN = 64  # elements; 128 bytes of bf16, 256 bytes of fp32
#: Device types the engine accepts. Only CUDA runs the native kernels; the
#: host-orchestration tests widen this while the ops are replaced by torch
#: implementations of the same contracts.
DEVICE_TYPES = ("cuda",)


@dataclass
class ParamSpec:
    name: str
    shape: tuple
    offset: int
    decay: bool
    group: str  # "root" or "h.<i>"

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def qkv_width(config: GPTConfig) -> int:
    """Columns of the fused c_attn output: C queries, then kv_heads x 64 keys
    and as many values (3C for multi-head attention; reference model.py:
    199-203)."""
    return config.n_embd + 2 * config.kv_heads * config.head_dim


def qkv_views(qkv: torch.Tensor, config: GPTConfig) -> tuple:
    """(q, k, v) column views of a fused [M, qkv_width] buffer."""
    C, kv = config.n_embd, config.kv_heads * config.head_dim
    return qkv[:, :C], qkv[:, C:C + kv], qkv[:, C + kv:]


class ParamLayout:
    """Flat, aligned layout of every GPT-2 parameter (tied weights once).

    Order: ln_f, h.{L-1}, ..., h.0, wte, wpe -- the order in which backward
    finishes each tensor's gradient.
    """

    def __init__(self, config: GPTConfig, align: int = ALIGN) -> None:
        if not config.tie_weights:
            raise ValueError("the native engine implements GPT-2's tied lm_head")
        if config.pos_embedding != "learned" or config.norm_position != "pre":
            raise ValueError("the native engine implements pre-LN GPT-2 with learned positions")
        if config.activation != "gelu_tanh" or config.head_dim != 64:
            raise ValueError("the native engine implements gelu_tanh, head_dim 64")
        if not (config.attn_bias and config.mlp_bias):
            raise ValueError("the native engine expects biased projections")
        self.config = config
        C, L = config.n_embd, config.n_layer
        specs: list[tuple[str, tuple, bool, str]] = [
            ("ln_f.weight", (C,), False, "root"),
            ("ln_f.bias", (C,), False, "root"),
        ]
        for i in reversed(range(L)):
            p = f"h.{i}."
            g = f"h.{i}"
            specs += [
                (p + "ln_1.weight", (C,), False, g),
                (p + "ln_1.bias", (C,), False, g),
                (p + "attn.c_attn.weight", (qkv_width(config), C), True, g),
                (p + "attn.c_attn.bias", (qkv_width(config),), False, g),
                (p + "attn.c_proj.weight", (C, C), True, g),
                (p + "attn.c_proj.bias", (C,), False, g),
                (p + "ln_2.weight", (C,), False, g),
                (p + "ln_2.bias", (C,), False, g),
                (p + "mlp.c_fc.weight", (4 * C, C), True, g),
                (p + "mlp.c_fc.bias", (4 * C,), False, g),
                (p + "mlp.c_proj.weight", (C, 4 * C), True, g),
                (p + "mlp.c_proj.bias", (C,), False, g),
            ]
        specs += [
            ("wte.weight", (config.vocab_size, C), True, "root"),
            ("wpe.weight", (config.n_positions, C), True, "root"),
        ]
        self.specs: list[ParamSpec] = []
        off = 0
        for name, shape, decay, group in specs:
            self.specs.append(ParamSpec(name, shape, off, decay, group))
            n = 1
            for s in shape:
                n *= s
            off += (n + align - 1) // align * align
        self.total = off
        self.by_name = {s.name: s for s in self.specs}

    @property
    def num_parameters(self) -> int:
        return sum(s.numel for s in self.specs)

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        s = self.by_name[name]
        return flat[s.offset : s.offset + s.numel].view(s.shape)

    def group_range(self, group: str) -> tuple[int, int]:
        specs = [s for s in self.specs if s.group == group]
        lo = specs[0].offset
        last = specs[-1]
        hi = last.offset + (last.numel + ALIGN - 1) // ALIGN * ALIGN
        return lo, hi

    def decay_segments(self) -> list[tuple[int, int, bool]]:
        return [(s.offset, s.numel, s.decay) for s in self.specs]


class CompactLayout:
    """The tensors of a :class:`ParamLayout` that `keep` selects, packed in
    the same order with the same alignment: flat storage for a subset of the
    parameters. ZeRO-3 keeps only the replicated root tensors (ln_f, wte, wpe)
    in the engine's own buffers; block tensors come from the gathered shards.

    ``segments`` lists (full_lo, full_hi, lo) for every stored tensor: its
    aligned range in the full layout and its start here."""

    def __init__(self, full: ParamLayout, keep: Callable[[ParamSpec], bool]) -> None:
        self.config = full.config
        self.full = full
        self.specs: list[ParamSpec] = []
        self.segments: list[tuple[int, int, int]] = []
        off = 0
        for s in full.specs:
            if not keep(s):
                continue
            span = (s.numel + ALIGN - 1) // ALIGN * ALIGN
            self.specs.append(ParamSpec(s.name, s.shape, off, s.decay, s.group))
            self.segments.append((s.offset, s.offset + span, off))
            off += span
        self.total = off
        self.by_name = {s.name: s for s in self.specs}

    @property
    def num_parameters(self) -> int:
        return self.full.num_parameters

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        s = self.by_name[name]
        return flat[s.offset : s.offset + s.numel].view(s.shape)

    def gather_from_full(self, full: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out[compact] = full[layout] for every stored tensor."""
        for a, b, o in self.segments:
            out[o : o + b - a].copy_(full[a:b])
        return out

    def scatter_to_full(self, compact: torch.Tensor, full: torch.Tensor) -> torch.Tensor:
        """full[layout] = compact for every stored tensor."""
        for a, b, o in self.segments:
            full[a:b].copy_(compact[o : o + b - a])
        return full


@torch.no_grad()
def init_flat_weights(layout: ParamLayout, flat: torch.Tensor, seed: int = 0) -> torch.Tensor:
    """Fill `flat` (fp32, ``layout.total`` elements, on a CUDA device) with the
    GPT-2 init in layout order from one seeded generator: the same weights for
    the same seed wherever the layout is instantiated (single GPU, data
    parallel, or sliced into tensor-parallel shards)."""
    g = torch.Generator(device=flat.device)
    g.manual_seed(seed)
    flat.zero_()
    res_std = 0.02 / math.sqrt(2 * layout.config.n_layer)
    for s in layout.specs:
        v = layout.view(flat, s.name)
        if s.name.endswith(("ln_1.weight", "ln_2.weight", "ln_f.weight")):
            v.fill_(1.0)
        elif s.name.endswith("bias"):
            v.zero_()
        elif s.name.endswith(("attn.c_proj.weight", "mlp.c_proj.weight")):
            v.normal_(0.0, res_std, generator=g)
        else:
            v.normal_(0.0, 0.02, generator=g)
    return flat


def choose_splits(m: int, n: int, k: int, bm: int = 128, bn: int = 256, sms: int = 148,
                  max_splits: int = 16, min_k: int = 1024) -> int:
    """Split-K factor for a wgrad GEMM: best wave efficiency, fewest splits."""
    tiles = -(-m // bm) * -(-n // bn)
    best, best_score = 1, -1.0
    for s in range(1, max_splits + 1):
        if s > 1 and k // s < min_k:
            break
        t = tiles * s
        eff = t / (-(-t // sms) * sms)
        score = eff - 0.015 * (s - 1)
        if score > best_score + 1e-9:
            best, best_score = s, score
    return best


@dataclass
class OptimConfig:
    lr: float = 3e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.1
    grad_clip: float = 1.0  # <= 0 disables clipping


class _Acts:
    """Activation and workspace buffers for one (B, T) shape."""

    def __init__(self, cfg: GPTConfig, B: int, T: int, dev: torch.device) -> None:
        C, L, H = cfg.n_embd, cfg.n_layer, cfg.n_head
        M = B * T
        self.B, self.T, self.M = B, T, M
        bf, f32 = torch.bfloat16, torch.float32
        self.x = [torch.empty(M, C, dtype=f32, device=dev) for _ in range(2 * L + 1)]
        self.h1 = [torch.empty(M, C, dtype=bf, device=dev) for _ in range(L)]
        W = qkv_width(cfg)
        self.qkv = [torch.empty(M, W, dtype=bf, device=dev) for _ in range(L)]
        self.y = [torch.empty(M, C, dtype=bf, device=dev) for _ in range(L)]
        self.lse = [torch.empty(B, H, T, dtype=f32, device=dev) for _ in range(L)]
        self.h2 = [torch.empty(M, C, dtype=bf, device=dev) for _ in range(L)]
        self.u = [torch.empty(M, 4 * C, dtype=bf, device=dev) for _ in range(L)]
        self.g = [torch.empty(M, 4 * C, dtype=bf, device=dev) for _ in range(L)]
        self.mu = [torch.empty(M, dtype=f32, device=dev) for _ in range(2 * L + 1)]
        self.rs = [torch.empty(M, dtype=f32, device=dev) for _ in range(2 * L + 1)]
        self.hf = torch.empty(M, C, dtype=bf, device=dev)
        vp = cfg.padded_vocab_size()
        self.logits = torch.empty(M, vp, dtype=bf, device=dev)
        self.ce = N.CEWorkspace(M, cfg.vocab_size, dev)
        # deterministic token-embedding gradient (bit-reproducible steps)
        self.emb_ws = N.EmbeddingGradWorkspace(M, C, cfg.vocab_size, dev)
        self.loss_rows = self.ce.loss_rows
        self.loss_out = torch.zeros(2, dtype=f32, device=dev)
        # backward scratch (reused across layers)
        self.dres = torch.empty(M, C, dtype=f32, device=dev)
        self.dres16 = torch.empty(M, C, dtype=bf, device=dev)
        self.dh = torch.empty(M, C, dtype=bf, device=dev)
        self.dy = torch.empty(M, C, dtype=bf, device=dev)
        self.du = torch.empty(M, 4 * C, dtype=bf, device=dev)
        self.dqkv = torch.empty(M, W, dtype=bf, device=dev)
        self.delta = torch.empty(B, H, T, dtype=f32, device=dev)
        self.ln_parts = N.layernorm_bwd_partials(M, C, dev)
        self.col_ws = torch.empty(N.colsum_ws_numel(M, 4 * C), dtype=f32, device=dev)
        # split-K plans for the four wgrad shapes
        self.splits = {
            "c_attn": choose_splits(W, C, M),
            "c_proj": choose_splits(C, C, M),
            "c_fc": choose_splits(4 * C, C, M),
            "mlp_proj": choose_splits(C, 4 * C, M),
        }
        ws = max(self.splits["c_attn"] * W * C, self.splits["c_proj"] * C * C,
                 self.splits["c_fc"] * 4 * C * C, self.splits["mlp_proj"] * 4 * C * C)
        self.splitk_ws = torch.empty(ws, dtype=f32, device=dev)


class Engine:
    """GPT-2 training engine on native kernels.

    Args:
        config: model architecture (pre-LN GPT-2 with tied embeddings).
        device: CUDA device.
        optim: AdamW / clipping settings.
        grad_buffer: optional externally owned fp32 flat gradient buffer of
            ``layout.total`` elements (DDP passes its peer-mapped buffer).
        shadow_buffer: optional externally owned bf16 flat parameter buffer
            the kernels read (ZeRO passes a peer-mapped buffer that every rank
            writes its updated slice into).
        seed: init seed for :meth:`init_weights` (ignored if weights loaded).
        optimizer_state: ``False`` skips allocating the full-size AdamW
            moments (a sharded optimiser owns them).
    """

    def __init__(self, config: GPTConfig, device: torch.device | str = "cuda", *,
                 optim: Optional[OptimConfig] = None, grad_buffer: Optional[torch.Tensor] = None,
                 shadow_buffer: Optional[torch.Tensor] = None, seed: Optional[int] = 0,
                 optimizer_state: bool = True, storage: Optional[CompactLayout] = None) -> None:
        self.config = config
        self.device = torch.device(device)
        if self.device.type not in DEVICE_TYPES:
            raise ValueError("the native engine runs on CUDA devices")
        N.lib()  # fail loudly if the extension is missing
        self.layout = ParamLayout(config)
        # the layout of the engine's own flat buffers: every tensor, or the
        # subset a parameter-sharding strategy leaves here (ZeRO-3: the root)
        self.storage = storage if storage is not None else self.layout
        self.init_seed = seed
        self.optim = optim or OptimConfig()
        n = self.storage.total
        dev = self.device
        self.master = torch.zeros(n, dtype=torch.float32, device=dev)
        if shadow_buffer is not None:
            if shadow_buffer.numel() < n or shadow_buffer.dtype != torch.bfloat16:
                raise ValueError("shadow_buffer too small or not bf16")
            self.shadow = shadow_buffer[:n]
        else:
            self.shadow = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        if grad_buffer is not None:
            if grad_buffer.numel() < n or grad_buffer.dtype != torch.float32:
                raise ValueError("grad_buffer too small or not fp32")
            self.grad = grad_buffer[:n]
        else:
            self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=dev) if optimizer_state else None
        self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=dev) if optimizer_state else None
        # A sharded optimiser replaces the update: optimizer_impl(hp) is called
        # with the device hyperparameter vector instead of the local AdamW.
        self.optimizer_impl: Optional[Callable[[torch.Tensor], None]] = None
        # Parameter sharding (ZeRO-3) supplies block parameters and gradient
        # destinations from its own buffers: param_source(name) /
        # grad_source(name) return a view or None (use the flat buffers), and
        # block_hook(phase, l) runs before block l's forward ("fwd") or
        # backward ("bwd") kernels are issued.
        self.param_source: Optional[Callable[[str], Optional[torch.Tensor]]] = None
        self.grad_source: Optional[Callable[[str], Optional[torch.Tensor]]] = None
        self.block_hook: Optional[Callable[[str, int], None]] = None
        # Context parallelism: this rank's tokens sit at positions
        # [pos0, pos0 + T) of the full sequence, and attention is delegated to
        # attn_fwd_hook(l, qkv, y, lse, B, H, T) / attn_bwd_hook(l, qkv, y, dy,
        # dqkv, lse, delta, B, H, T) when set.
        self.pos0 = 0
        # a local sequence made of two chunks of the full context (load-
        # balanced context parallelism): columns from pos_split on sit at
        # pos1 + (t - pos_split)
        self.pos_split: Optional[int] = None
        self.pos1 = 0
        self.attn_fwd_hook: Optional[Callable] = None
        self.attn_bwd_hook: Optional[Callable] = None
        # LayerNorm backward also produces the c_proj bias gradients of the
        # block that fed it (one block earlier for ln_1); a sharded gradient
        # buffer per block turns this off so each block writes only its own.
        self.fuse_bias_grad_into_ln = True
        # Cross-entropy path. Measured on B200 at 16 x 1024 tokens (CUDA
        # events, kernel bench): the lm_head GEMM with the statistics epilogue
        # + row fold + gradient pass 2.12 ms, against 1.78 ms for the plain
        # GEMM (0.98 ms) + the one-kernel cross-entropy (0.80 ms, at 0.96 of
        # the measured HBM bandwidth): the GEMM's 8 epilogue warps cannot hide
        # the per-element statistics behind the MMAs. The separate path is
        # the default; True selects the fused one.
        self.fused_ce = False
        self.step_count = 0
        self._acts: Optional[_Acts] = None
        # Hyperparameters reach the device by an async copy from pinned memory
        # each step. The host may run several steps ahead of the GPU, so the
        # pinned source rotates through a ring and a slot is reused only after
        # the copy that read it has executed.
        self._hp_ring = [torch.zeros(8, dtype=torch.float32).pin_memory() for _ in range(4)]
        self._hp_events: list = [None] * len(self._hp_ring)
        self.hp = torch.zeros(8, dtype=torch.float32, device=dev)
        self._norm_ws = torch.empty(1024, dtype=torch.float32, device=dev)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.clip = torch.ones(1, dtype=torch.float32, device=dev)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=dev)
        # Hook called after each block's gradients are final (DDP buckets);
        # signature: hook(group_name) with group in {"root_head", "h.i", "root_tail"}.
        self.grad_ready_hook: Optional[Callable[[str], None]] = None
        self.grad_scale = 1.0  # multiplies gradients inside AdamW
        # Decayed tensors (rank >= 2) are not contiguous in backward order: the
        # fused AdamW reads this table of [lo, hi) decay ranges.
        ranges = [x for lo, hi, d in self._merge_segments() if d for x in (lo, hi)]
        self.decay_ranges = torch.tensor(ranges, dtype=torch.int64, device=dev)
        if seed is not None:
            self.init_weights(seed)

    # ------------------------------------------------------------ weights --
    def _merge_segments(self):
        segs = []
        for s in self.storage.specs:
            lo = s.offset
            hi = s.offset + (s.numel + ALIGN - 1) // ALIGN * ALIGN
            if segs and segs[-1][2] == s.decay and segs[-1][1] == lo:
                segs[-1] = (segs[-1][0], hi, s.decay)
            else:
                segs.append((lo, hi, s.decay))
        return segs

    def p32(self, name: str) -> torch.Tensor:
        return self.storage.view(self.master, name)

    def p16(self, name: str) -> torch.Tensor:
        if self.param_source is not None:
            v = self.param_source(name)
            if v is not None:
                return v
        return self.storage.view(self.shadow, name)

    def g32(self, name: str) -> torch.Tensor:
        if self.grad_source is not None:
            v = self.grad_source(name)
            if v is not None:
                return v
        return self.storage.view(self.grad, name)

    @torch.no_grad()
    def init_weights(self, seed: int = 0) -> None:
        """GPT-2 init on the device: N(0, 0.02) for matmul weights and
        embeddings, N(0, 0.02/sqrt(2L)) for the two residual projections,
        zero biases, unit LayerNorm gains (reference model.py:488-518)."""
        self.init_seed = seed
        if self.storage is self.layout:
            init_flat_weights(self.layout, self.master, seed)
        else:
            # the same values as the full layout's init (one generator in
            # layout order), kept for the stored tensors only
            full = torch.empty(self.layout.total, dtype=torch.float32, device=self.device)
            self.storage.gather_from_full(init_flat_weights(self.layout, full, seed), self.master)
            del full
        self.sync_shadow()

    @torch.no_grad()
    def sync_shadow(self) -> None:
        self.shadow.copy_(self.master)

    @torch.no_grad()
    def load_state_dict(self, sd: dict) -> None:
        """Load a reference-named state dict (GPT.state_dict())."""
        for s in self.storage.specs:
            src = sd[s.name] if s.name in sd else sd.get("lm_head.weight") if s.name == "wte.weight" else None
            if src is None:
                raise KeyError(s.name)
            self.p32(s.name).copy_(src.to(self.device, torch.float32).view(s.shape))
        self.sync_shadow()

    def state_dict(self) -> dict:
        """Reference-named fp32 state dict (``lm_head.weight`` tied to wte)."""
        out = {s.name: self.p32(s.name).detach().clone() for s in self.storage.specs}
        out["lm_head.weight"] = out["wte.weight"]
        return out

    @classmethod
    def from_module(cls, model, device="cuda", **kw) -> "Engine":
        eng = cls(model.config, device, seed=None, **kw)
        eng.load_state_dict(model.state_dict())
        return eng

    # --------------------------------------------------------- activations --
    def acts(self, B: int, T: int) -> _Acts:
        if self._acts is None or (self._acts.B, self._acts.T) != (B, T):
            self._acts = None
            torch.cuda.empty_cache()
            self._acts = _Acts(self.config, B, T, self.device)
        return self._acts

    # ------------------------------------------------------------- forward --
    def forward(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Forward pass; returns the device scalar loss (loss_out[0]).
        Also leaves dlogits in the logits buffer for :meth:`backward`."""
        targets = targets.contiguous()
        A = self._forward_to_logits(idx, targets)
        return A.loss_out[0]

    @torch.no_grad()
    def logits(self, idx: torch.Tensor) -> torch.Tensor:
        """Forward without the loss: (B*T, vocab) bf16 logits (a view of the
        engine's buffer, valid until the next forward)."""
        return self._forward_to_logits(idx).logits[:, : self.config.vocab_size]

    def _forward_to_logits(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None) -> _Acts:
        """Forward to the lm_head. With `targets`, the lm_head GEMM is the
        fused cross-entropy (loss in loss_out, dlogits left in the logits
        buffer); without, the buffer holds the logits."""
        cfg = self.config
        idx = idx.contiguous()
        B, T = idx.shape
        top = self.pos0 + T if self.pos_split is None else max(self.pos0 + self.pos_split,
                                                               self.pos1 + T - self.pos_split)
        if top > cfg.n_positions:
            raise ValueError(f"positions up to {top} exceed n_positions={cfg.n_positions}")
        A = self.acts(B, T)
        C, H, L, V = cfg.n_embd, cfg.n_head, cfg.n_layer, cfg.vocab_size
        eps = cfg.layer_norm_epsilon
        p = self.p16
        N.embedding_fwd(idx, p("wte.weight"), p("wpe.weight"), A.x[0], pos0=self.pos0,
                        pos_split=self.pos_split, pos1=self.pos1)
        bh = self.block_hook
        for l in range(L):
            pre = f"h.{l}."
            if bh:
                bh("fwd", l)
            rng = nvtx_range(f"fwd/h.{l}")
            rng.__enter__()
            N.layernorm_fwd(A.x[2 * l], p(pre + "ln_1.weight"), p(pre + "ln_1.bias"), A.h1[l],
                            A.mu[2 * l], A.rs[2 * l], eps)
            N.gemm(A.h1[l], p(pre + "attn.c_attn.weight"), A.qkv[l], bias=p(pre + "attn.c_attn.bias"))
            qkv = A.qkv[l]
            if self.attn_fwd_hook is not None:
                self.attn_fwd_hook(l, qkv, A.y[l], A.lse[l], B, H, T)
            else:
                N.attention_fwd(*qkv_views(qkv, cfg), A.y[l], A.lse[l], B, H, T, kv_heads=cfg.kv_heads)
            N.gemm(A.y[l], p(pre + "attn.c_proj.weight"), A.x[2 * l + 1], epilogue=N.EPI_RESID_F32,
                   bias=p(pre + "attn.c_proj.bias"), aux=A.x[2 * l])
            N.layernorm_fwd(A.x[2 * l + 1], p(pre + "ln_2.weight"), p(pre + "ln_2.bias"), A.h2[l],
                            A.mu[2 * l + 1], A.rs[2 * l + 1], eps)
            N.gemm(A.h2[l], p(pre + "mlp.c_fc.weight"), A.g[l], epilogue=N.EPI_BIAS_GELU,
                   bias=p(pre + "mlp.c_fc.bias"), aux=A.u[l])
            N.gemm(A.g[l], p(pre + "mlp.c_proj.weight"), A.x[2 * l + 2], epilogue=N.EPI_RESID_F32,
                   bias=p(pre + "mlp.c_proj.bias"), aux=A.x[2 * l + 1])
            rng.__exit__(None, None, None)
        with nvtx_range("lm_head+ce"):
            N.layernorm_fwd(A.x[2 * L], p("ln_f.weight"), p("ln_f.bias"), A.hf, A.mu[2 * L], A.rs[2 * L],
                            eps)
            if targets is not None and self.fused_ce:
                N.lm_head_cross_entropy(A.hf, p("wte.weight"), A.logits, targets, A.ce, A.loss_out, V)
            else:
                N.gemm(A.hf, p("wte.weight"), A.logits[:, :V])
                if targets is not None:
                    N.cross_entropy_fwd_bwd(A.logits, targets.view(-1), A.loss_rows, A.loss_out, V)
        return A

    # ------------------------------------------------------------ backward --
    def backward(self, idx: torch.Tensor, accumulate: bool = False) -> None:
        """Backward of the last :meth:`forward`; gradients land in ``self.grad``
        (added to it when ``accumulate``)."""
        cfg = self.config
        A = self._acts
        B, T, M = A.B, A.T, A.M
        C, H, L, V = cfg.n_embd, cfg.n_head, cfg.n_layer, cfg.vocab_size
        p, g = self.p16, self.g32
        acc = bool(accumulate)
        inv_count = A.loss_out[1:2]
        hook = self.grad_ready_hook
        logits = A.logits[:, :V]
        # lm_head (tied): dhf = dlogits @ wte / count ; dwte = dlogits^T @ hf / count
        N.gemm(logits, p("wte.weight"), A.dh, b_t=True, alpha_ptr=inv_count)
        N.gemm(logits, A.hf, g("wte.weight"), a_t=True, b_t=True, epilogue=N.EPI_F32,
               alpha_ptr=inv_count, accumulate=acc)
        # LN backward also sums the residual gradient it writes: that column
        # sum is the bias gradient of the projection that produced the stream
        fuse = self.fuse_bias_grad_into_ln
        bh = self.block_hook
        N.layernorm_bwd(A.dh, A.x[2 * L], A.mu[2 * L], A.rs[2 * L], p("ln_f.weight"), A.dres,
                        A.dres16, g("ln_f.weight"), g("ln_f.bias"), A.ln_parts,
                        accumulate_dres=False, accumulate_params=acc,
                        dsum=g(f"h.{L - 1}.mlp.c_proj.bias") if fuse else None, accumulate_dsum=acc)
        if hook:
            hook("root_head")
        ws = A.splitk_ws
        for l in reversed(range(L)):
            pre = f"h.{l}."
            if bh:
                bh("bwd", l)
            rng = nvtx_range(f"bwd/h.{l}")
            rng.__enter__()
            # mlp.c_proj
            N.gemm(A.dres16, p(pre + "mlp.c_proj.weight"), A.du, b_t=True, epilogue=N.EPI_GELU_BWD,
                   aux=A.u[l])
            N.gemm(A.dres16, A.g[l], g(pre + "mlp.c_proj.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=A.splits["mlp_proj"], workspace=ws)
            if not fuse:
                N.colsum_bf16(A.dres16, g(pre + "mlp.c_proj.bias"), A.col_ws, accumulate=acc)
            # mlp.c_fc
            N.gemm(A.du, p(pre + "mlp.c_fc.weight"), A.dh, b_t=True)
            N.gemm(A.du, A.h2[l], g(pre + "mlp.c_fc.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=A.splits["c_fc"], workspace=ws)
            N.colsum_bf16(A.du, g(pre + "mlp.c_fc.bias"), A.col_ws, accumulate=acc)
            N.layernorm_bwd(A.dh, A.x[2 * l + 1], A.mu[2 * l + 1], A.rs[2 * l + 1],
                            p(pre + "ln_2.weight"), A.dres, A.dres16, g(pre + "ln_2.weight"),
                            g(pre + "ln_2.bias"), A.ln_parts, accumulate_dres=True,
                            accumulate_params=acc,
                            dsum=g(pre + "attn.c_proj.bias") if fuse else None,
                            accumulate_dsum=acc)
            # attn.c_proj
            N.gemm(A.dres16, p(pre + "attn.c_proj.weight"), A.dy, b_t=True)
            N.gemm(A.dres16, A.y[l], g(pre + "attn.c_proj.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=A.splits["c_proj"], workspace=ws)
            if not fuse:
                N.colsum_bf16(A.dres16, g(pre + "attn.c_proj.bias"), A.col_ws, accumulate=acc)
            # attention
            qkv, dqkv = A.qkv[l], A.dqkv
            if self.attn_bwd_hook is not None:
                self.attn_bwd_hook(l, qkv, A.y[l], A.dy, dqkv, A.lse[l], A.delta, B, H, T)
            else:
                N.attention_bwd(*qkv_views(qkv, cfg), A.y[l], A.dy, *qkv_views(dqkv, cfg), A.lse[l],
                                A.delta, B, H, T, kv_heads=cfg.kv_heads)
            # attn.c_attn
            N.gemm(dqkv, p(pre + "attn.c_attn.weight"), A.dh, b_t=True)
            N.gemm(dqkv, A.h1[l], g(pre + "attn.c_attn.weight"), a_t=True, b_t=True,
                   epilogue=N.EPI_F32, accumulate=acc, splits=A.splits["c_attn"], workspace=ws)
            N.colsum_bf16(dqkv, g(pre + "attn.c_attn.bias"), A.col_ws, accumulate=acc)
            N.layernorm_bwd(A.dh, A.x[2 * l], A.mu[2 * l], A.rs[2 * l], p(pre + "ln_1.weight"),
                            A.dres, A.dres16, g(pre + "ln_1.weight"), g(pre + "ln_1.bias"),
                            A.ln_parts, accumulate_dres=True, accumulate_params=acc,
                            dsum=g(f"h.{l - 1}.mlp.c_proj.bias") if (fuse and l > 0) else None,
                            accumulate_dsum=acc)
            rng.__exit__(None, None, None)
            if hook:
                hook(f"h.{l}")
        wpe_g = g("wpe.weight")
        if not acc:
            wpe_g.zero_()
        N.embedding_bwd(idx, A.dres, g("wte.weight"), wpe_g, V, pos0=self.pos0,
                        pos_split=self.pos_split, pos1=self.pos1, det=A.emb_ws)
        if hook:
            hook("root_tail")

    # ----------------------------------------------------------- optimiser --
    def set_lr(self, lr: float) -> None:
        self.optim.lr = lr

    def optimizer_step(self) -> None:
        """Clip (global norm) + AdamW over the whole flat buffer."""
        self.stage_hyperparams()
        with nvtx_range("optimizer"):
            self._optimizer_update()

    def stage_hyperparams(self) -> None:
        """The host half of a step: advance the step count and copy this
        step's AdamW scalars (lr, bias corrections, gradient scale) into the
        device buffer the update kernels read (stream-ordered)."""
        o = self.optim
        self.step_count += 1
        t = self.step_count
        slot = t % len(self._hp_ring)
        if self._hp_events[slot] is not None:
            self._hp_events[slot].synchronize()
        hp = self._hp_ring[slot]
        hp[0] = o.lr
        hp[1] = o.betas[0]
        hp[2] = o.betas[1]
        hp[3] = o.eps
        hp[4] = o.weight_decay
        hp[5] = 1.0 - o.betas[0] ** t
        hp[6] = math.sqrt(1.0 - o.betas[1] ** t)
        hp[7] = self.grad_scale
        self.hp.copy_(hp, non_blocking=True)
        ev = self._hp_events[slot] or torch.cuda.Event()
        ev.record()
        self._hp_events[slot] = ev

    def _optimizer_update(self) -> None:
        o = self.optim
        if self.optimizer_impl is not None:
            self.optimizer_impl(self.hp)
            return
        clip = None
        if o.grad_clip and o.grad_clip > 0:
            N.grad_sumsq(self.grad, self._norm_ws, self.sumsq)
            N.clip_coef(self.sumsq, o.grad_clip, self.clip, self.grad_norm,
                        scale2=self.grad_scale * self.grad_scale)
            clip = self.clip
        N.adamw_step(self.master, self.grad, self.exp_avg, self.exp_avg_sq, self.shadow, 0,
                     self.hp, clip, decay_ranges=self.decay_ranges)

    # ---------------------------------------------------------------- step --
    def train_step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One optimiser step on one micro-batch; returns the device loss."""
        loss = self.forward(idx, targets)
        self.backward(idx)
        self.optimizer_step()
        return loss
