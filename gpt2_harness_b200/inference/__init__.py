"""Inference: sampling rules, KV-cached generation (reference semantics on the
oracle model) and the B200 decode engine (preallocated KV cache, fused
append + split-K decode attention, CUDA-graph decode step)."""

from .sampling import apply_temperature, generate, top_k_filter, top_p_filter  # noqa: F401
