"""Activation memory: measured (saved-tensor hooks) and analytic.

Reference: src/transformer_internals/perf/activation_memory.py:127-613.

* :class:`ActivationMeter` counts the distinct storages autograd saves for
  backward during a forward pass, excluding parameters/buffers and classifying
  autocast's narrow copies of weights (found by walking ``grad_fn`` through
  view/cast nodes back to a leaf) as parameter memory; a weakref finaliser
  releases each storage when the graph drops it, so ``peak_bytes`` is a live
  high-water mark.
* :func:`analytic_activation_bytes` enumerates the tensors the oracle model's
  operators save (fp32, dropout 0, explicit attention, MHA): no fitted
  constants. The tanh GELU written from primitive ops saves four 4C-wide
  tensors; cross-entropy saves one tokens x vocab log-softmax.
* The native engine's stash is a fixed, planned set of buffers;
  :func:`native_activation_bytes` reports it exactly (bf16 operands, fp32
  residual stream, per-row LSE instead of T x T probabilities).
"""

from __future__ import annotations

import weakref
from dataclasses import asdict, dataclass
from typing import Any, Iterable, Optional

import torch

from gpt2_harness_b200.config import GPTConfig

__all__ = [
    "PASSTHROUGH_NODES",
    "GELU_TANH_SAVED_TENSORS",
    "ActivationMeter",
    "ActivationReport",
    "analytic_activation_bytes",
    "measure_activation_bytes",
    "native_activation_bytes",
]

PASSTHROUGH_NODES = frozenset({
    "TBackward0", "ViewBackward0", "UnsafeViewBackward0", "ToCopyBackward0", "ExpandBackward0",
    "PermuteBackward0", "TransposeBackward0", "ReshapeAliasBackward0", "CloneBackward0",
    "DetachBackward0", "SqueezeBackward0", "UnsqueezeBackward0",
})

#: Saved 4C-wide tensors of 0.5*x*(1+tanh(k*(x+0.044715*x^3))) built from
#: primitive ops: x (pow), tanh output, 0.5*x, and 1+tanh(...).
GELU_TANH_SAVED_TENSORS = 4


def _source_leaf(t: torch.Tensor, max_depth: int = 8) -> Optional[torch.Tensor]:
    node = t.grad_fn
    for _ in range(max_depth):
        if node is None:
            return None
        name = type(node).__name__
        if name == "AccumulateGrad":
            return getattr(node, "variable", None)
        if name not in PASSTHROUGH_NODES:
            return None
        nxt = [n for n, _ in node.next_functions if n is not None]
        if len(nxt) != 1:
            return None
        node = nxt[0]
    return None


def _storage_key(t: torch.Tensor) -> int:
    try:
        return t.untyped_storage().data_ptr()
    except (RuntimeError, NotImplementedError, AttributeError):
        return -1


class ActivationMeter:
    """Context manager measuring the live saved-for-backward storage bytes."""

    def __init__(self, device=None, exclude: Optional[Iterable[torch.Tensor]] = None) -> None:
        self.device = torch.device(device) if device is not None else None
        self._excluded: set[int] = set()
        self.excluded_bytes = 0
        for t in exclude or ():
            k = _storage_key(t)
            if k >= 0 and k not in self._excluded:
                self._excluded.add(k)
                self.excluded_bytes += t.untyped_storage().nbytes()
        self._live: dict[int, list] = {}
        self._current = 0
        self.peak_bytes = 0
        self.tensors_saved = 0
        self.parameter_cast_bytes = 0
        self._cast_seen: set[int] = set()
        self.cuda_peak_allocated_bytes: Optional[int] = None
        self._cuda_base: Optional[int] = None
        self._ctx = None

    def _pack(self, t: torch.Tensor) -> torch.Tensor:
        try:
            st = t.untyped_storage()
            key, nbytes = st.data_ptr(), st.nbytes()
        except (RuntimeError, NotImplementedError):
            return t
        if nbytes == 0 or key in self._excluded:
            return t
        if self._excluded:
            leaf = _source_leaf(t)
            if leaf is not None and _storage_key(leaf) in self._excluded:
                if key not in self._cast_seen:
                    self._cast_seen.add(key)
                    self.parameter_cast_bytes += nbytes
                return t
        self.tensors_saved += 1
        ent = self._live.get(key)
        if ent is None:
            self._live[key] = [nbytes, 1]
            self._current += nbytes
            self.peak_bytes = max(self.peak_bytes, self._current)
        else:
            ent[1] += 1
        weakref.finalize(t, self._release, key)
        return t

    def _release(self, key: int) -> None:
        ent = self._live.get(key)
        if ent is None:
            return
        ent[1] -= 1
        if ent[1] <= 0:
            self._current -= ent[0]
            del self._live[key]

    @staticmethod
    def _unpack(t: torch.Tensor) -> torch.Tensor:
        return t

    def __enter__(self) -> "ActivationMeter":
        if self.device is not None and self.device.type == "cuda":
            torch.cuda.reset_peak_memory_stats(self.device)
            self._cuda_base = int(torch.cuda.memory_allocated(self.device))
        self._ctx = torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack)
        self._ctx.__enter__()
        return self

    def __exit__(self, *exc: Any) -> None:
        self._ctx.__exit__(*exc)
        self._ctx = None
        if self.device is not None and self.device.type == "cuda":
            self.cuda_peak_allocated_bytes = int(torch.cuda.max_memory_allocated(self.device)) - (self._cuda_base or 0)

    def stash_bytes(self) -> int:
        return self._current

    def snapshot(self) -> dict[str, Any]:
        return {"activation_bytes": self._current, "distinct_storages": len(self._live),
                "saved_tensor_count": self.tensors_saved,
                "parameter_cast_bytes": self.parameter_cast_bytes}

    def to_dict(self) -> dict[str, Any]:
        return {"saved_for_backward_peak_bytes": self.peak_bytes,
                "saved_tensor_count": self.tensors_saved,
                "excluded_parameter_bytes": self.excluded_bytes,
                "parameter_cast_bytes": self.parameter_cast_bytes,
                "cuda_peak_allocated_bytes": self.cuda_peak_allocated_bytes}


@dataclass
class ActivationReport:
    measured_bytes: int
    analytic_bytes: float
    batch: int
    seq: int
    detail: dict

    @property
    def ratio(self) -> float:
        return self.measured_bytes / self.analytic_bytes if self.analytic_bytes else float("nan")

    def as_dict(self) -> dict:
        d = asdict(self)
        d["ratio"] = self.ratio
        return d


def analytic_activation_bytes(cfg: GPTConfig, batch: int, seq: int, dtype_bytes: int = 4,
                              with_loss: bool = True) -> dict[str, float]:
    """Bytes the oracle model's forward saves for backward, term by term.

    Refuses configurations whose saved set it does not enumerate (dropout > 0,
    SDPA, GQA, non-fp32)."""
    if cfg.dropout > 0:
        raise ValueError("analytic count covers dropout=0 only (dropout saves a mask per site)")
    if cfg.use_sdpa:
        raise ValueError("analytic count covers the explicit attention path only")
    if cfg.n_kv_head is not None:
        raise ValueError("analytic count covers multi-head attention only")
    if dtype_bytes != 4:
        raise ValueError("analytic count covers fp32 only: autocast keeps LayerNorm and the "
                         "log-softmax in fp32, so halving every term is wrong; measure instead")
    n, c, v = float(batch * seq), float(cfg.n_embd), float(cfg.vocab_size)
    L, H, e = float(cfg.n_layer), float(cfg.n_head), float(dtype_bytes)
    act = n * c * e
    stats = 2.0 * n * 4.0
    gelu = {"gelu_tanh": float(GELU_TANH_SAVED_TENSORS), "gelu_exact": 1.0, "relu": 0.0}[cfg.activation]
    per = {
        "residual_into_the_first_sublayer": act,
        "layernorm_1_stats": stats,
        "qkv_projection_input": act,
        "score_matmul_operands_q_and_k": 2.0 * act,
        "attention_probabilities": float(batch) * H * float(seq) ** 2 * e,
        "inverted_causal_mask": float(seq) ** 2,
        "value_matmul_operand": act,
        "attention_output_projection_input": act,
        "residual_into_the_second_sublayer": act,
        "layernorm_2_stats": stats,
        "mlp_up_projection_input": act,
        "mlp_activation_intermediates": gelu * 4.0 * act,
        "mlp_down_projection_input": 4.0 * act,
    }
    root = {"final_layernorm_input": act, "final_layernorm_stats": stats, "lm_head_input": act,
            "token_ids": n * 8.0}
    if cfg.pos_embedding == "learned":
        root["position_ids"] = float(seq) * 8.0
    if with_loss:
        root["cross_entropy_log_softmax_output"] = n * v * e
        root["cross_entropy_target_ids"] = n * 8.0
        root["cross_entropy_total_weight"] = 4.0
    out = {f"per_layer.{k}": x for k, x in per.items()}
    out["per_layer_subtotal"] = sum(per.values())
    out["all_layers"] = L * out["per_layer_subtotal"]
    out.update({f"root.{k}": x for k, x in root.items()})
    out["root_subtotal"] = sum(root.values())
    out["total"] = out["all_layers"] + out["root_subtotal"]
    out["bytes_per_token"] = out["total"] / max(n, 1.0)
    return out


def measure_activation_bytes(model, inputs: torch.Tensor, targets=None, cfg: Optional[GPTConfig] = None,
                             dtype_bytes: int = 4) -> ActivationReport:
    """One forward under an ActivationMeter, read before backward, plus the
    analytic prediction for the same shape."""
    cfg = cfg if cfg is not None else model.config
    B, T = int(inputs.shape[0]), int(inputs.shape[1])
    meter = ActivationMeter(device=inputs.device, exclude=[*model.parameters(), *model.buffers()])
    with meter:
        out = model(inputs, targets=targets)
        loss = out["loss"] if targets is not None else out["logits"].float().mean()
    snap = meter.snapshot()
    loss.backward()
    terms = analytic_activation_bytes(cfg, B, T, dtype_bytes, with_loss=targets is not None)
    detail = meter.to_dict()
    detail.update(snap)
    detail["analytic_terms"] = terms
    return ActivationReport(snap["activation_bytes"], terms["total"], B, T, detail)


def native_activation_bytes(cfg: GPTConfig, batch: int, seq: int) -> dict[str, float]:
    """Exact bytes the native engine keeps between forward and backward."""
    M, C, L, H = batch * seq, cfg.n_embd, cfg.n_layer, cfg.n_head
    vp = cfg.padded_vocab_size()
    per = {
        "residual_stream_fp32": 2 * M * C * 4,  # x_in and x_mid per block
        "ln_stats_fp32": 2 * 2 * M * 4,
        "ln1_out_bf16": M * C * 2,
        "qkv_bf16": M * (C + 2 * cfg.kv_heads * cfg.head_dim) * 2,
        "attn_out_bf16": M * C * 2,
        "attn_lse_fp32": batch * H * seq * 4,
        "ln2_out_bf16": M * C * 2,
        "gelu_input_bf16": M * 4 * C * 2,
        "gelu_output_bf16": M * 4 * C * 2,
    }
    root = {"final_residual_fp32": M * C * 4, "ln_f_out_bf16": M * C * 2, "ln_f_stats": 2 * M * 4,
            "logits_bf16_padded": M * vp * 2, "loss_rows": M * 4}
    out = {f"per_layer.{k}": float(x) for k, x in per.items()}
    out["per_layer_subtotal"] = float(sum(per.values()))
    out["all_layers"] = L * out["per_layer_subtotal"]
    out.update({f"root.{k}": float(x) for k, x in root.items()})
    out["total"] = out["all_layers"] + float(sum(root.values()))
    return out
