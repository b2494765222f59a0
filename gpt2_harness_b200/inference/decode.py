"""KV-cached decoding on B200 kernels.

The reference decodes with the eager model and a ``torch.cat``-grown cache
(src/transformer_internals/model.py:106-172, sampling.py:100-181). Here the
cache is preallocated once for ``max_len`` positions ([L, B, Hkv, Tmax, 64]
bf16) and the per-token work is a fixed sequence of launches over fixed
buffers:

* ``decode_embed``: token + position embedding, the position read from the
  device-side ``lens`` vector;
* per layer: LayerNorm (native), the q/k/v projection (a skinny cuBLAS GEMM),
  ``decode_attn`` (native: appends this token's k/v in place and runs split-K
  attention over the cache, grouped-query aware), output projection and MLP
  with fp32 residuals;
* final LayerNorm, tied head, and ``decode_argmax`` (native: greedy token,
  history append, ``lens += 1``).

Because nothing in that sequence depends on host values, one decode step is
captured once in a CUDA graph and replayed per token (greedy decoding);
sampled decoding replays the graph up to the logits and samples on the host
side with the same filters as :mod:`.sampling`.

The prompt is encoded by a prefill pass that runs the native flash-attention
forward (multi-head) or PyTorch SDPA (grouped-query) and writes K/V straight
into the cache.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from ..config import GPTConfig
from ..ops import native as N
from .sampling import sample_next

__all__ = ["DecodeEngine"]


def _bf16(t: torch.Tensor, dev) -> torch.Tensor:
    return t.detach().to(device=dev, dtype=torch.bfloat16).contiguous()


class DecodeEngine:
    """Batched incremental decoding for a GPT-2 state dict (oracle names)."""

    def __init__(self, config: GPTConfig, state_dict: dict, batch: int, max_len: Optional[int] = None,
                 device="cuda", use_graph: bool = True) -> None:
        cfg = config
        if cfg.n_embd // cfg.n_head != 64:
            raise ValueError("the decode kernels need head_dim 64")
        if cfg.norm_position != "pre" or cfg.activation != "gelu_tanh" or cfg.pos_embedding != "learned":
            raise ValueError("DecodeEngine covers the GPT-2 architecture (pre-LN, gelu_tanh, learned positions)")
        self.config = cfg
        self.device = dev = torch.device(device)
        self.B = batch
        self.Tmax = min(max_len or cfg.n_positions, cfg.n_positions)
        self.H, self.Hkv, self.C, self.L = cfg.n_head, cfg.kv_heads, cfg.n_embd, cfg.n_layer
        self.V = cfg.vocab_size
        self.Vp = (self.V + 63) // 64 * 64
        sd = {k: v for k, v in state_dict.items()}
        self.w = {}
        for k, v in sd.items():
            if k.endswith("causal_mask") or not torch.is_tensor(v) or not v.is_floating_point():
                continue
            self.w[k] = _bf16(v, dev)
        wte = self.w["wte.weight"]
        head = self.w.get("lm_head.weight", wte) if not cfg.tie_weights else wte
        self.head = torch.zeros(self.Vp, self.C, dtype=torch.bfloat16, device=dev)
        self.head[: self.V].copy_(head)
        zeros = lambda n: torch.zeros(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
        for l in range(self.L):
            for name, n in (("attn.c_attn", self.C + 2 * self.Hkv * 64), ("attn.c_proj", self.C),
                            ("mlp.c_fc", 4 * self.C), ("mlp.c_proj", self.C)):
                self.w.setdefault(f"h.{l}.{name}.bias", zeros(n))
        B, C, Tm = batch, self.C, self.Tmax
        kvd = (self.L, B, self.Hkv, Tm, 64)
        self.k_cache = torch.zeros(kvd, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros(kvd, dtype=torch.bfloat16, device=dev)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.hist = torch.zeros(B, Tm, dtype=torch.int64, device=dev)
        f32, bf = torch.float32, torch.bfloat16
        self.x = torch.zeros(B, C, dtype=f32, device=dev)
        self.h = torch.zeros(B, C, dtype=bf, device=dev)
        self.qkv = torch.zeros(B, C + 2 * self.Hkv * 64, dtype=bf, device=dev)
        self.att = torch.zeros(B, C, dtype=bf, device=dev)
        self.proj = torch.zeros(B, C, dtype=bf, device=dev)
        self.u = torch.zeros(B, 4 * C, dtype=bf, device=dev)
        self.logits = torch.zeros(B, self.Vp, dtype=bf, device=dev)
        self.mean = torch.zeros(B, dtype=f32, device=dev)
        self.rstd = torch.zeros(B, dtype=f32, device=dev)
        self.part_o, self.part_ml = N.decode_partials(B, self.H, Tm, dev)
        self.eps = cfg.layer_norm_epsilon
        self.use_graph = use_graph and dev.type == "cuda"
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self.prompt_len = 0

    @classmethod
    def from_model(cls, model, batch: int, max_len: Optional[int] = None, device="cuda", **kw) -> "DecodeEngine":
        return cls(model.config, model.state_dict(), batch, max_len, device, **kw)

    # ---------------------------------------------------------------- step --
    def _ln(self, name: str) -> None:
        N.layernorm_fwd(self.x, self.w[name + ".weight"], self.w[name + ".bias"], self.h, self.mean, self.rstd,
                        self.eps)

    def _body(self) -> None:
        """Embedding .. logits for the token in ``tok`` at position ``lens``."""
        w = self.w
        N.decode_embed(self.tok, self.lens, w["wte.weight"], w["wpe.weight"], self.x)
        for l in range(self.L):
            p = f"h.{l}."
            self._ln(p + "ln_1")
            torch.addmm(w[p + "attn.c_attn.bias"], self.h, w[p + "attn.c_attn.weight"].t(), out=self.qkv)
            N.decode_attn(self.qkv, self.k_cache[l], self.v_cache[l], self.lens, self.part_o, self.part_ml,
                          self.att, self.H, self.Hkv)
            torch.addmm(w[p + "attn.c_proj.bias"], self.att, w[p + "attn.c_proj.weight"].t(), out=self.proj)
            self.x.add_(self.proj)
            self._ln(p + "ln_2")
            torch.addmm(w[p + "mlp.c_fc.bias"], self.h, w[p + "mlp.c_fc.weight"].t(), out=self.u)
            self.u.copy_(F.gelu(self.u, approximate="tanh"))
            torch.addmm(w[p + "mlp.c_proj.bias"], self.u, w[p + "mlp.c_proj.weight"].t(), out=self.proj)
            self.x.add_(self.proj)
        self._ln("ln_f")
        torch.mm(self.h, self.head.t(), out=self.logits)

    def _greedy_step(self) -> None:
        self._body()
        N.decode_argmax(self.logits, self.V, self.tok, self.lens, self.hist)

    def step(self) -> None:
        """One greedy token for every row (graph replay after the first call)."""
        if not self.use_graph:
            self._greedy_step()
            return
        if self._graph is None:
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            snap = (self.lens.clone(), self.tok.clone(), self.hist.clone(), self.k_cache.clone(),
                    self.v_cache.clone())
            with torch.cuda.stream(s):
                self._greedy_step()  # warm-up outside capture (library handles, workspaces)
            torch.cuda.current_stream(self.device).wait_stream(s)
            self.lens.copy_(snap[0]); self.tok.copy_(snap[1]); self.hist.copy_(snap[2])  # noqa: E702
            self.k_cache.copy_(snap[3]); self.v_cache.copy_(snap[4])  # noqa: E702
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._greedy_step()
            self._graph = g
            self.lens.copy_(snap[0]); self.tok.copy_(snap[1]); self.hist.copy_(snap[2])  # noqa: E702
            self.k_cache.copy_(snap[3]); self.v_cache.copy_(snap[4])  # noqa: E702
        self._graph.replay()

    # ------------------------------------------------------------- prefill --
    @torch.no_grad()
    def prefill(self, idx: torch.Tensor) -> torch.Tensor:
        """Encode (B, T0) prompts into the cache; returns last-position logits
        (B, V) and leaves the greedy next token in ``tok``."""
        B, T0 = idx.shape
        if B != self.B or T0 < 1 or T0 >= self.Tmax:
            raise ValueError(f"prompt must be ({self.B}, 1..{self.Tmax - 1})")
        w, C, H, Hkv = self.w, self.C, self.H, self.Hkv
        idx = idx.to(self.device)
        pos = torch.arange(T0, device=self.device)
        x = (w["wte.weight"][idx].float() + w["wpe.weight"][pos].float()).reshape(B * T0, C)
        h = torch.empty(B * T0, C, dtype=torch.bfloat16, device=self.device)
        mean = torch.empty(B * T0, dtype=torch.float32, device=self.device)
        rstd = torch.empty_like(mean)
        for l in range(self.L):
            p = f"h.{l}."
            N.layernorm_fwd(x, w[p + "ln_1.weight"], w[p + "ln_1.bias"], h, mean, rstd, self.eps)
            qkv = torch.addmm(w[p + "attn.c_attn.bias"], h, w[p + "attn.c_attn.weight"].t())
            q, k, v = qkv.split([C, Hkv * 64, Hkv * 64], dim=1)
            kh = k.reshape(B, T0, Hkv, 64).transpose(1, 2)
            vh = v.reshape(B, T0, Hkv, 64).transpose(1, 2)
            self.k_cache[l, :, :, :T0].copy_(kh)
            self.v_cache[l, :, :, :T0].copy_(vh)
            if Hkv == H:
                y = torch.empty(B * T0, C, dtype=torch.bfloat16, device=self.device)
                lse = torch.empty(B, H, T0, dtype=torch.float32, device=self.device)
                N.attention_fwd(q, k, v, y, lse, B, H, T0)
            else:
                qh = q.reshape(B, T0, H, 64).transpose(1, 2)
                rep = H // Hkv
                y = F.scaled_dot_product_attention(qh, kh.repeat_interleave(rep, 1), vh.repeat_interleave(rep, 1),
                                                   is_causal=True)
                y = y.transpose(1, 2).reshape(B * T0, C)
            x = x + torch.addmm(w[p + "attn.c_proj.bias"], y, w[p + "attn.c_proj.weight"].t()).float()
            N.layernorm_fwd(x, w[p + "ln_2.weight"], w[p + "ln_2.bias"], h, mean, rstd, self.eps)
            u = F.gelu(torch.addmm(w[p + "mlp.c_fc.bias"], h, w[p + "mlp.c_fc.weight"].t()), approximate="tanh")
            x = x + torch.addmm(w[p + "mlp.c_proj.bias"], u, w[p + "mlp.c_proj.weight"].t()).float()
        last = x.reshape(B, T0, C)[:, -1].contiguous()
        hl = torch.empty(B, C, dtype=torch.bfloat16, device=self.device)
        N.layernorm_fwd(last, w["ln_f.weight"], w["ln_f.bias"], hl, mean[:B], rstd[:B], self.eps)
        logits = (hl @ self.head.t())[:, : self.V]
        self.hist.zero_()
        self.hist[:, :T0].copy_(idx)
        self.lens.fill_(T0 - 1)
        self.logits[:, : self.V].copy_(logits)
        N.decode_argmax(self.logits, self.V, self.tok, self.lens, self.hist)  # lens -> T0
        self.prompt_len = T0
        return logits.float()

    # ------------------------------------------------------------ generate --
    @torch.no_grad()
    def generate(self, idx: torch.Tensor, max_new_tokens: int, *, do_sample: bool = False,
                 temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
                 eos_token_id: Optional[int] = None, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """Same contract as :func:`gpt2_harness_b200.inference.sampling.generate`."""
        B, T0 = idx.shape
        n = min(max_new_tokens, self.Tmax - T0)
        if n <= 0:
            return idx.clone()
        logits = self.prefill(idx)
        if do_sample:
            return self._generate_sampled(idx, logits, n, temperature, top_k, top_p, eos_token_id, generator)
        out = [self.tok.clone()]
        done = torch.zeros(B, dtype=torch.bool, device=self.device)
        if eos_token_id is not None:
            done |= out[-1] == eos_token_id
        for _ in range(n - 1):
            if eos_token_id is not None and bool(done.all()):
                break
            self.step()
            out.append(self.tok.clone())
            if eos_token_id is not None:
                done |= out[-1] == eos_token_id
        new = torch.stack(out, dim=1)
        if eos_token_id is not None:
            # rows that finished keep emitting EOS
            hit = (new == eos_token_id).cumsum(dim=1) > 0
            first = hit & ~torch.cat([torch.zeros_like(hit[:, :1]), hit[:, :-1]], dim=1)
            new = torch.where(hit & ~first, torch.full_like(new, eos_token_id), new)
        return torch.cat([idx.to(self.device), new], dim=1)

    def _generate_sampled(self, idx, logits, n, temperature, top_k, top_p, eos_token_id, generator):
        B = idx.shape[0]
        done = torch.zeros(B, dtype=torch.bool, device=self.device)
        toks = []
        for i in range(n):
            nxt = sample_next(logits, do_sample=True, temperature=temperature, top_k=top_k, top_p=top_p,
                              generator=generator).squeeze(1).to(self.device)
            if eos_token_id is not None:
                nxt = nxt.masked_fill(done, eos_token_id)
                done |= nxt == eos_token_id
            toks.append(nxt)
            if i + 1 == n or (eos_token_id is not None and bool(done.all())):
                break
            # feed the sampled token: position lens, then the body yields logits
            self.tok.copy_(nxt)
            self._body()
            self.lens.add_(1)
            logits = self.logits[:, : self.V].float()
        return torch.cat([idx.to(self.device), torch.stack(toks, dim=1)], dim=1)

    @torch.no_grad()
    def forced_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """Teacher-forced check: prefill tokens[:, :1], then feed tokens[:, t]
        one at a time; returns the (B, T, V) logits of every position."""
        B, T = tokens.shape
        outs = [self.prefill(tokens[:, :1])]
        for t in range(1, T):
            self.tok.copy_(tokens[:, t].to(self.device))
            self._body()
            self.lens.add_(1)
            outs.append(self.logits[:, : self.V].float().clone())
        return torch.stack(outs, dim=1)

    def kv_cache_bytes(self) -> int:
        return 2 * self.k_cache.numel() * self.k_cache.element_size()
