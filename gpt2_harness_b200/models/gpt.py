"""GPT-2 as a plain PyTorch module: the single-process oracle.

This is the model every parallel strategy, checkpoint and science tool wraps,
and the numerical reference the native engine (:mod:`.engine`) is tested
against. Its parameter names, initialisation and forward contract are the
reference's (src/transformer_internals/model.py:57-653), so state dicts move
between the two frameworks unchanged:

* pre-LN blocks ``x + attn(ln_1(x))``, ``x + mlp(ln_2(x))`` (post-LN optional);
* fused ``c_attn`` producing q, k, v (k/v narrowed to ``n_kv_head`` heads for
  GQA/MQA); explicit softmax attention with the causal mask taken at absolute
  positions (so cached decoding agrees with full recompute); optional SDPA arm;
* tied ``lm_head`` (shares ``wte.weight``), N(0, 0.02) init with the two
  residual-writing projections at 0.02/sqrt(2 n_layer);
* ``forward`` returns a dict: ``logits`` and, on request, ``loss`` (cross
  entropy, ignore_index -100), ``attentions`` and ``taps``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from gpt2_harness_b200.config import GPTConfig

__all__ = [
    "GPT",
    "MLP",
    "Block",
    "CausalSelfAttention",
    "KVCache",
    "gelu_tanh",
    "sinusoidal_position_embeddings",
]

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """GELU with the tanh approximation GPT-2 shipped:
    ``0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))``."""
    return 0.5 * x * (1.0 + torch.tanh(_SQRT_2_OVER_PI * (x + 0.044715 * x.pow(3))))


def sinusoidal_position_embeddings(n_positions: int, n_embd: int) -> torch.Tensor:
    """Fixed (n_positions, n_embd) table: sin on even channels, cos on odd,
    frequencies 10000^(-2i/d) (Vaswani et al., 2017)."""
    pos = torch.arange(n_positions, dtype=torch.float32)[:, None]
    freq = torch.exp(torch.arange(0, n_embd, 2, dtype=torch.float32) * (-math.log(10000.0) / n_embd))
    table = torch.zeros(n_positions, n_embd)
    table[:, 0::2] = torch.sin(pos * freq)
    table[:, 1::2] = torch.cos(pos * freq)[:, : n_embd // 2]
    return table


@dataclass
class KVCache:
    """Growing per-layer key/value history for incremental decoding.

    ``keys[l]`` / ``values[l]`` are ``(B, n_kv_head, T, head_dim)`` or None.
    Attention must use :meth:`length` of its own layer: within one forward pass
    earlier layers have already appended the current step.
    """

    keys: list
    values: list

    @classmethod
    def empty(cls, n_layer: int) -> "KVCache":
        return cls(keys=[None] * n_layer, values=[None] * n_layer)

    @property
    def seq_len(self) -> int:
        return self.length(0)

    def length(self, layer: int) -> int:
        k = self.keys[layer]
        return 0 if k is None else int(k.shape[-2])

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        if self.keys[layer] is not None:
            k = torch.cat([self.keys[layer], k], dim=-2)
            v = torch.cat([self.values[layer], v], dim=-2)
        self.keys[layer], self.values[layer] = k, v
        return k, v


class CausalSelfAttention(nn.Module):
    """Multi-head (or grouped-query) causal self-attention with a fused
    q/k/v projection. ``head_mask`` (n_head,) multiplies each head's output
    before the projection (head ablation / pruning)."""

    def __init__(self, config: GPTConfig, layer_idx: int = 0) -> None:
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.n_head = config.n_head
        self.n_kv_head = config.kv_heads
        self.n_embd = config.n_embd
        self.head_dim = config.head_dim
        self.kv_dim = self.n_kv_head * self.head_dim
        self.c_attn = nn.Linear(config.n_embd, config.n_embd + 2 * self.kv_dim, bias=config.attn_bias)
        self.c_proj = nn.Linear(config.n_embd, config.n_embd, bias=config.attn_bias)
        self.attn_dropout = nn.Dropout(config.dropout)
        self.resid_dropout = nn.Dropout(config.dropout)
        self.register_buffer(
            "causal_mask",
            torch.ones(config.n_positions, config.n_positions, dtype=torch.bool).tril(),
            persistent=False,
        )
        self.head_mask: torch.Tensor | None = None

    def forward(self, x: torch.Tensor, cache: KVCache | None = None, need_weights: bool = False):
        B, T, C = x.shape
        past = cache.length(self.layer_idx) if cache is not None else 0
        q, k, v = self.c_attn(x).split([self.n_embd, self.kv_dim, self.kv_dim], dim=2)
        q = q.view(B, T, self.n_head, self.head_dim).transpose(1, 2)
        k = k.view(B, T, self.n_kv_head, self.head_dim).transpose(1, 2)
        v = v.view(B, T, self.n_kv_head, self.head_dim).transpose(1, 2)
        if cache is not None:
            k, v = cache.update(self.layer_idx, k, v)
        total = k.shape[-2]
        if self.n_kv_head != self.n_head:
            rep = self.n_head // self.n_kv_head
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
        mask = self.causal_mask[past : past + T, :total]
        weights = None
        if self.config.use_sdpa and not need_weights:
            y = F.scaled_dot_product_attention(
                q, k, v, attn_mask=mask.view(1, 1, T, total),
                dropout_p=self.config.dropout if self.training else 0.0,
            )
        else:
            scores = (q @ k.transpose(-2, -1)) / math.sqrt(self.head_dim)
            scores = scores.masked_fill(~mask.view(1, 1, T, total), float("-inf"))
            probs = F.softmax(scores, dim=-1)
            if need_weights:
                weights = probs
            y = self.attn_dropout(probs) @ v
        if self.head_mask is not None:
            # (n_head,) for every sequence, or (B, n_head) per sequence
            m = self.head_mask.to(y.device, y.dtype)
            y = y * (m.view(1, -1, 1, 1) if m.dim() == 1 else m.view(m.shape[0], -1, 1, 1))
        y = y.transpose(1, 2).contiguous().view(B, T, C)
        return self.resid_dropout(self.c_proj(y)), weights


class MLP(nn.Module):
    """4x feed-forward block; ``neuron_mask`` (4C,) multiplies hidden units."""

    def __init__(self, config: GPTConfig) -> None:
        super().__init__()
        self.config = config
        self.c_fc = nn.Linear(config.n_embd, 4 * config.n_embd, bias=config.mlp_bias)
        self.c_proj = nn.Linear(4 * config.n_embd, config.n_embd, bias=config.mlp_bias)
        self.dropout = nn.Dropout(config.dropout)
        self.neuron_mask: torch.Tensor | None = None

    def act(self, x: torch.Tensor) -> torch.Tensor:
        if self.config.activation == "gelu_tanh":
            return gelu_tanh(x)
        if self.config.activation == "gelu_exact":
            return F.gelu(x)
        return F.relu(x)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.act(self.c_fc(x))
        if self.neuron_mask is not None:
            h = h * self.neuron_mask.to(h.device, h.dtype)
        return self.dropout(self.c_proj(h))


class Block(nn.Module):
    """Transformer block, pre-LN (default) or post-LN."""

    def __init__(self, config: GPTConfig, layer_idx: int = 0) -> None:
        super().__init__()
        self.config = config
        self.ln_1 = nn.LayerNorm(config.n_embd, eps=config.layer_norm_epsilon)
        self.attn = CausalSelfAttention(config, layer_idx=layer_idx)
        self.ln_2 = nn.LayerNorm(config.n_embd, eps=config.layer_norm_epsilon)
        self.mlp = MLP(config)

    def forward(self, x, cache=None, need_weights=False, taps=None, prefix=""):
        def tap(name, t):
            if taps is not None:
                taps[prefix + name] = t

        if self.config.norm_position == "pre":
            h = self.ln_1(x)
            tap("ln_1", h)
            a, w = self.attn(h, cache=cache, need_weights=need_weights)
            tap("attn", a)
            x = x + a
            tap("resid_mid", x)
            h2 = self.ln_2(x)
            m = self.mlp(h2)
            tap("ln_2", h2)
            tap("mlp", m)
            x = x + m
        else:
            a, w = self.attn(x, cache=cache, need_weights=need_weights)
            tap("attn", a)
            x = self.ln_1(x + a)
            tap("resid_mid", x)
            m = self.mlp(x)
            tap("mlp", m)
            x = self.ln_2(x + m)
        tap("resid_out", x)
        return x, w


class GPT(nn.Module):
    """GPT-2 decoder. Module names follow the OpenAI/HF checkpoint layout."""

    def __init__(self, config: GPTConfig) -> None:
        super().__init__()
        self.config = config
        self.wte = nn.Embedding(config.vocab_size, config.n_embd)
        if config.pos_embedding == "learned":
            self.wpe: nn.Embedding | None = nn.Embedding(config.n_positions, config.n_embd)
        else:
            self.wpe = None
            self.register_buffer(
                "sinusoidal_pe",
                sinusoidal_position_embeddings(config.n_positions, config.n_embd),
                persistent=False,
            )
        self.drop = nn.Dropout(config.dropout)
        self.h = nn.ModuleList([Block(config, layer_idx=i) for i in range(config.n_layer)])
        self.ln_f = nn.LayerNorm(config.n_embd, eps=config.layer_norm_epsilon)
        self.lm_head = nn.Linear(config.n_embd, config.vocab_size, bias=False)
        if config.tie_weights:
            self.lm_head.weight = self.wte.weight
        self.apply(self._init_weights)
        if config.residual_scaled_init:
            std = 0.02 / math.sqrt(2 * config.n_layer)
            for blk in self.h:
                nn.init.normal_(blk.attn.c_proj.weight, mean=0.0, std=std)
                nn.init.normal_(blk.mlp.c_proj.weight, mean=0.0, std=std)

    @staticmethod
    def _init_weights(module: nn.Module) -> None:
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
        elif isinstance(module, nn.LayerNorm):
            nn.init.ones_(module.weight)
            nn.init.zeros_(module.bias)

    def position_embeddings(self, pos: torch.Tensor) -> torch.Tensor:
        if self.wpe is not None:
            return self.wpe(pos)
        return self.sinusoidal_pe[pos]

    def forward(self, idx, targets=None, cache=None, need_weights=False, collect_taps=False) -> dict[str, Any]:
        _, T = idx.shape
        past = cache.seq_len if cache is not None else 0
        if past + T > self.config.n_positions:
            raise ValueError(
                f"sequence of length {past + T} exceeds n_positions={self.config.n_positions}; "
                "learned position embeddings cannot extrapolate"
            )
        pos = torch.arange(past, past + T, dtype=torch.long, device=idx.device)
        x = self.drop(self.wte(idx) + self.position_embeddings(pos))
        taps: dict[str, torch.Tensor] | None = {} if collect_taps else None
        if taps is not None:
            taps["embed"] = x
        attentions = []
        for i, blk in enumerate(self.h):
            x, w = blk(x, cache=cache, need_weights=need_weights, taps=taps, prefix=f"h.{i}.")
            if w is not None:
                attentions.append(w)
        x = self.ln_f(x)
        if taps is not None:
            taps["ln_f"] = x
        logits = self.lm_head(x)
        out: dict[str, Any] = {"logits": logits}
        if taps is not None:
            taps["logits"] = logits
            out["taps"] = taps
        if need_weights:
            out["attentions"] = attentions
        if targets is not None:
            out["loss"] = F.cross_entropy(
                logits.view(-1, logits.size(-1)), targets.reshape(-1), ignore_index=-100
            )
        return out

    def num_parameters(self, non_embedding: bool = False) -> int:
        """Distinct parameter count (tied weights once); ``non_embedding``
        drops the position table (the token table still counts: it is also
        the output head)."""
        n = sum(p.numel() for p in self.parameters())
        if non_embedding and self.wpe is not None:
            n -= self.wpe.weight.numel()
        return n

    def configure_optimizers(self, weight_decay: float, lr: float, betas, eps: float = 1e-8):
        """AdamW with decay on rank>=2 tensors (matmul weights, embeddings)
        only; biases and LayerNorm gains are not decayed."""
        decay = [p for p in self.parameters() if p.requires_grad and p.dim() >= 2]
        rest = [p for p in self.parameters() if p.requires_grad and p.dim() < 2]
        groups = [{"params": decay, "weight_decay": weight_decay}, {"params": rest, "weight_decay": 0.0}]
        return torch.optim.AdamW(groups, lr=lr, betas=betas, eps=eps)
