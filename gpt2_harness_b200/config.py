"""Architecture and optimisation configuration.

Same public surface as the reference's ``transformer_internals.config``
(``GPTConfig``, ``TrainConfig``, ``GPT2_SIZES``, ``gpt2_config``; reference
src/transformer_internals/config.py:24-229), so a config written for the
reference constructs here unchanged. Additions for the B200 runs:

* ``padded_vocab_size``: the vocabulary rounded up (default to a multiple of
  64 -> 50304 for GPT-2) so that the lm_head row stride is 16-byte aligned for
  TMA and divides evenly across tensor-parallel ranks.
* :data:`BENCH_CONFIGS`: the model/batch shapes of the headline benchmarks.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any, Literal

__all__ = ["GPT2_SIZES", "GPTConfig", "TrainConfig", "gpt2_config", "BENCH_CONFIGS"]


@dataclass
class GPTConfig:
    """Decoder-only GPT-2 architecture. Defaults are GPT-2 124M exactly.

    Fields mirror the reference one for one (config.py:75-92): vocab_size,
    n_positions, n_layer, n_head, n_kv_head (GQA/MQA when set), n_embd, dropout,
    layer_norm_epsilon and the ablation switches norm_position ("pre"/"post"),
    pos_embedding ("learned"/"sinusoidal"), tie_weights, activation
    ("gelu_tanh"/"gelu_exact"/"relu"), residual_scaled_init, attn_bias,
    mlp_bias and use_sdpa.
    """

    vocab_size: int = 50257
    n_positions: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_kv_head: int | None = None
    n_embd: int = 768
    dropout: float = 0.0
    layer_norm_epsilon: float = 1e-5

    norm_position: Literal["pre", "post"] = "pre"
    pos_embedding: Literal["learned", "sinusoidal"] = "learned"
    tie_weights: bool = True
    activation: Literal["gelu_tanh", "gelu_exact", "relu"] = "gelu_tanh"
    residual_scaled_init: bool = True
    attn_bias: bool = True
    mlp_bias: bool = True
    use_sdpa: bool = False

    def __post_init__(self) -> None:
        if self.n_embd % self.n_head:
            raise ValueError(f"n_embd={self.n_embd} must be divisible by n_head={self.n_head}")
        if self.n_kv_head is not None and (self.n_kv_head < 1 or self.n_head % self.n_kv_head):
            raise ValueError(f"n_head={self.n_head} must be divisible by n_kv_head={self.n_kv_head}")
        if self.norm_position not in ("pre", "post"):
            raise ValueError(f"norm_position must be 'pre' or 'post', got {self.norm_position!r}")
        if self.pos_embedding not in ("learned", "sinusoidal"):
            raise ValueError(f"unknown pos_embedding {self.pos_embedding!r}")
        if self.activation not in ("gelu_tanh", "gelu_exact", "relu"):
            raise ValueError(f"unknown activation {self.activation!r}")

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def kv_heads(self) -> int:
        return self.n_head if self.n_kv_head is None else self.n_kv_head

    def padded_vocab_size(self, multiple: int = 64) -> int:
        """Vocabulary rounded up to ``multiple`` (50257 -> 50304 at 64)."""
        return ((self.vocab_size + multiple - 1) // multiple) * multiple

    def kv_cache_bytes_per_token(self, dtype_bytes: int = 4) -> int:
        """KV-cache bytes per token per sequence across layers:
        ``2 * n_layer * kv_heads * head_dim * dtype_bytes``."""
        return 2 * self.n_layer * self.kv_heads * self.head_dim * dtype_bytes

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


#: The four released GPT-2 sizes (reference config.py:138-143).
GPT2_SIZES: dict[str, dict[str, int]] = {
    "gpt2": {"n_layer": 12, "n_head": 12, "n_embd": 768},
    "gpt2-medium": {"n_layer": 24, "n_head": 16, "n_embd": 1024},
    "gpt2-large": {"n_layer": 36, "n_head": 20, "n_embd": 1280},
    "gpt2-xl": {"n_layer": 48, "n_head": 25, "n_embd": 1600},
}


def gpt2_config(size: str = "gpt2", **overrides: Any) -> GPTConfig:
    """Config of a released GPT-2 size, with field overrides applied on top."""
    if size not in GPT2_SIZES:
        raise ValueError(f"unknown GPT-2 size {size!r}; expected one of {sorted(GPT2_SIZES)}")
    return GPTConfig(**{**GPT2_SIZES[size], **overrides})


@dataclass
class TrainConfig:
    """Optimisation settings (reference config.py:163-229, same defaults).

    lr 3e-4 with linear warmup then cosine decay to ``lr * min_lr_ratio``;
    AdamW betas (0.9, 0.95), eps 1e-8, weight decay 0.1 on rank>=2 tensors only;
    global-norm clip 1.0; optional autocast (``amp``/``amp_dtype``).
    """

    steps: int = 600
    batch_size: int = 16
    grad_accum: int = 1
    block_size: int = 128
    lr: float = 3e-4
    min_lr_ratio: float = 0.1
    warmup_steps: int = 60
    weight_decay: float = 0.1
    grad_clip: float = 1.0
    betas: tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    seed: int = 0
    eval_interval: int = 50
    eval_batches: int = 20
    amp: bool = False
    amp_dtype: Literal["bf16", "fp16"] = "bf16"
    log_every: int = 50
    extra: dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


#: Headline benchmark shapes (model, per-GPU micro-batch, sequence length,
#: strategy). ``gpt2-small-ddp`` is the flagship ``bench.py`` default.
BENCH_CONFIGS: dict[str, dict[str, Any]] = {
    "gpt2-small-ddp": {"size": "gpt2", "batch": 16, "seq": 1024, "strategy": "ddp"},
    "gpt2-medium-zero3": {"size": "gpt2-medium", "batch": 8, "seq": 1024, "strategy": "zero3"},
    "gpt2-xl-tp8": {"size": "gpt2-xl", "global_batch": 32, "seq": 1024, "strategy": "tp"},
    "gpt2-large-pp4cp2": {"size": "gpt2-large", "micro_batch": 1, "micro_batches": 8,
                          "seq": 16384, "strategy": "pp_cp"},
    "gpt2-tiny-ddp": {"size": None, "n_layer": 8, "n_head": 4, "n_embd": 128,
                      "n_positions": 64, "batch": 4, "seq": 64, "strategy": "ddp"},
}
