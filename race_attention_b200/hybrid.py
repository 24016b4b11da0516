"""Caller harness for the config-4 measurement: hybrid decode with the Llama-3.2-1B
architecture (random-init bf16 weights), odd layers RACE attention, even layers softmax GQA.

The reference has no decode path for RACE (chat/nanochat/gpt.py:143-146 raises); this
harness is where the library's fused decode step (race_decode_step through RaceDecodeState)
meets a real model loop: a batched prefill that leaves each RACE layer's (A, B) state and
each softmax layer's KV cache, then greedy decode steps, each one fused RACE state update +
readout per RACE layer (grouped-query: 32 query heads read 8 kv states) and one
race_gqa_decode_attn launch per softmax layer (appends the token's key/value to the cache
and attends over it; the cache length lives in device memory).  Because no launch of a
decode step depends on host-side position values, DecodeGraph captures one whole step as a
CUDA graph and replays it.  Architecture: 16 layers, hidden 2048, 32 / 8 heads, head_dim 64,
SwiGLU MLP 8192, RMSNorm (eps 1e-5), RoPE theta 500000, vocabulary 128256 with the LM head
tied to the embedding.  Decoding runs in bf16 (the softmax layers' kernel is bf16-only).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .decode import RaceDecodeState, prefill_with_state
from .race_common import build_planes_protos


@dataclass
class HybridConfig:
    vocab_size: int = 128256
    n_layer: int = 16
    hidden: int = 2048
    n_head: int = 32
    n_kv_head: int = 8
    mlp_hidden: int = 8192
    rope_theta: float = 500000.0
    norm_eps: float = 1e-5
    race_L: int = 8
    race_P: int = 4
    race_eps: float = 1e-6


class _RMSNorm(nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        return F.rms_norm(x, (x.size(-1),), self.weight, self.eps)


def _rope(x, cos, sin):
    # x [B, H, T, D]; rotate the two halves of the head dimension
    h = x.shape[-1] // 2
    a, b = x[..., :h], x[..., h:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)


class Layer(nn.Module):
    def __init__(self, cfg: HybridConfig, idx: int):
        super().__init__()
        self.cfg, self.race = cfg, idx % 2 == 1
        hd = cfg.hidden // cfg.n_head
        self.hd = hd
        self.ln1 = _RMSNorm(cfg.hidden, cfg.norm_eps)
        self.ln2 = _RMSNorm(cfg.hidden, cfg.norm_eps)
        # q, k, v projections as one [(Hq + 2 Hkv) * hd, hidden] weight and gate/up as one
        # [2 * mlp, hidden] weight: one GEMM each (the split is a view of the output)
        self.qkv = nn.Linear(cfg.hidden, (cfg.n_head + 2 * cfg.n_kv_head) * hd, bias=False)
        self.o = nn.Linear(cfg.n_head * hd, cfg.hidden, bias=False)
        self.gate_up = nn.Linear(cfg.hidden, 2 * cfg.mlp_hidden, bias=False)
        self.down = nn.Linear(cfg.mlp_hidden, cfg.hidden, bias=False)
        if self.race:
            planes_T, _ = build_planes_protos(hd, cfg.race_P, cfg.race_L, 1, device="cpu", seed=idx)
            self.register_buffer("planes_T", planes_T)
        self.state = None      # RACE layers: RaceDecodeState
        self.cache = None      # softmax layers: (K, V) [B, Hkv, Tmax, D]
        self.attn_ws = None    # softmax layers: race_gqa_decode_attn workspace and its split count
        self.n_splits = 1

    def _qkv(self, x, cos, sin):
        B, T, _ = x.shape
        cfg, hd = self.cfg, self.hd
        q, k, v = self.qkv(x).view(B, T, cfg.n_head + 2 * cfg.n_kv_head, hd).split(
            [cfg.n_head, cfg.n_kv_head, cfg.n_kv_head], dim=2)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        return _rope(q, cos, sin), _rope(k, cos, sin), v

    def _mlp(self, x):
        g, u = self.gate_up(x).chunk(2, dim=-1)
        return self.down(F.silu(g) * u)

    def prefill(self, x, cos, sin, t_max, b0, batch):
        """x [mb, T, hidden]: sequences [b0, b0 + mb) of a batch of `batch`, from position 0;
        fills their slice of the layer's decode state / KV cache (allocated on b0 == 0)."""
        mb, T, _ = x.shape
        cfg = self.cfg
        q, k, v = self._qkv(self.ln1(x), cos, sin)
        if self.race:
            y, st = prefill_with_state(q.contiguous(), k.contiguous(), v.contiguous(), self.planes_T, cfg.race_L,
                                       cfg.race_P, cfg.race_eps)
            if b0 == 0:
                self.state = RaceDecodeState(batch, cfg.n_kv_head, self.hd, cfg.race_L, cfg.race_P, self.planes_T,
                                             cfg.race_eps, device=x.device)
            rows = slice(b0 * cfg.n_kv_head, (b0 + mb) * cfg.n_kv_head)
            self.state.A[rows].copy_(st.A)
            self.state.B[rows].copy_(st.B)
            self.state.tokens = T
        else:
            if b0 == 0:
                self.cache = tuple(torch.empty(batch, cfg.n_kv_head, t_max, self.hd, dtype=k.dtype, device=k.device)
                                   for _ in range(2))
                self.n_splits = ops.gqa_decode_splits(batch, cfg.n_kv_head, t_max, k.device)
                self.attn_ws = ops.gqa_decode_workspace(batch, cfg.n_head, cfg.n_kv_head, self.n_splits, k.device)
            self.cache[0][b0:b0 + mb, :, :T].copy_(k)
            self.cache[1][b0:b0 + mb, :, :T].copy_(v)
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        x = x + self.o(y.transpose(1, 2).reshape(mb, T, -1))
        return x + self._mlp(self.ln2(x))

    def step(self, x, cos, sin, pos):
        """x [B, 1, hidden] at position pos (int32 device tensor [1] = tokens already seen)."""
        B = x.shape[0]
        q, k, v = self._qkv(self.ln1(x), cos, sin)  # [B, H, 1, D]
        q, k, v = q[:, :, 0].contiguous(), k[:, :, 0].contiguous(), v[:, :, 0].contiguous()
        if self.race:
            y = self.state.step(q, k, v)
        else:
            y = ops.gqa_decode_attention(q, k, v, self.cache[0], self.cache[1], pos, self.attn_ws, self.n_splits)
        x = x + self.o(y.reshape(B, 1, -1))
        return x + self._mlp(self.ln2(x))


class HybridLlama(nn.Module):
    def __init__(self, cfg: HybridConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden)
        self.layers = nn.ModuleList(Layer(cfg, i) for i in range(cfg.n_layer))
        self.norm = _RMSNorm(cfg.hidden, cfg.norm_eps)
        self.pos = None        # int32 device tensor [1]: tokens in the decode state / caches
        self.n_tokens = 0      # the same count on the host
        self.t_max = 0

    def init_weights(self, std=0.02):
        for name, p in self.named_parameters():
            if p.dim() > 1:
                nn.init.normal_(p, mean=0.0, std=std)

    def _inv_freq(self, device):
        hd = self.cfg.hidden // self.cfg.n_head
        return self.cfg.rope_theta ** (-torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd)

    def _angles(self, pos0, T, device, dtype):
        ang = torch.outer(torch.arange(pos0, pos0 + T, device=device, dtype=torch.float32), self._inv_freq(device))
        return ang.cos().to(dtype), ang.sin().to(dtype)

    def _logits(self, x):
        return F.linear(self.norm(x), self.embed.weight)

    @torch.no_grad()
    def prefill(self, idx, t_max, micro_batch=4):
        """idx [B, T] token ids -> next-token ids [B] (greedy); sequences go through the
        layers micro_batch at a time (the MLP's [mb, T, 8192] activations bound memory)."""
        B, T = idx.shape
        cos, sin = self._angles(0, T, idx.device, self.embed.weight.dtype)
        nxt = []
        for b0 in range(0, B, micro_batch):
            x = self.embed(idx[b0:b0 + micro_batch])
            for layer in self.layers:
                x = layer.prefill(x, cos, sin, t_max, b0, B)
            nxt.append(self._logits(x[:, -1]).argmax(-1))
        self.pos = torch.full((1,), T, dtype=torch.int32, device=idx.device)
        self.n_tokens, self.t_max = T, t_max
        return torch.cat(nxt)

    @torch.no_grad()
    def logits_full(self, idx):
        """Last-position logits of a plain causal forward over idx [B, T] (no caches kept)."""
        B, T = idx.shape
        kept = [(layer.state, layer.cache, layer.attn_ws, layer.n_splits) for layer in self.layers]
        cos, sin = self._angles(0, T, idx.device, self.embed.weight.dtype)
        x = self.embed(idx)
        for layer in self.layers:
            x = layer.prefill(x, cos, sin, T, 0, B)
        for layer, (st, cache, ws, ns) in zip(self.layers, kept):  # the decode state stays as it was
            layer.state, layer.cache, layer.attn_ws, layer.n_splits = st, cache, ws, ns
        return self._logits(x[:, -1])

    def _step_logits(self, tok):
        """One decode step on the device: every position-dependent value comes from self.pos,
        so the launches are the same at every step (capturable)."""
        ang = self.pos.float()[:, None] * self._inv_freq(tok.device)[None]
        dtype = self.embed.weight.dtype
        cos, sin = ang.cos().to(dtype), ang.sin().to(dtype)
        x = self.embed(tok[:, None])
        for layer in self.layers:
            x = layer.step(x, cos, sin, self.pos)
        self.pos.add_(1)
        return self._logits(x[:, -1])

    def _advance(self, n):
        self.n_tokens += n
        for layer in self.layers:
            if layer.race:
                layer.state.tokens = self.n_tokens

    @torch.no_grad()
    def step_logits(self, tok):
        """tok [B] -> next-token logits [B, vocab]; appends tok to the decode state."""
        if self.pos is None or self.n_tokens >= self.t_max:
            raise RuntimeError(f"decode state full ({self.n_tokens} of {self.t_max} positions) or not prefilled")
        logits = self._step_logits(tok)
        self._advance(1)
        return logits

    @torch.no_grad()
    def step(self, tok):
        """tok [B] -> next-token ids [B] (greedy)."""
        return self.step_logits(tok).argmax(-1)


class DecodeGraph:
    """One greedy decode step of a prefilled HybridLlama captured as a CUDA graph.

    replay() feeds the token held in self.tok, advances the model by one position and leaves
    the next token in self.tok.  Capture runs nothing on the device; call model.step at
    least once before capturing (first-use initialisation of the libraries must happen
    outside capture) and do not mix eager steps with replays afterwards unless self.tok is
    refreshed."""

    def __init__(self, model: HybridLlama, tok):
        self.model = model
        self.tok = tok.clone()
        saved = model.n_tokens
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.tok.copy_(model._step_logits(self.tok).argmax(-1))
        model.n_tokens = saved
        model._advance(0)

    def replay(self):
        m = self.model
        if m.n_tokens >= m.t_max:
            raise RuntimeError(f"decode state full ({m.n_tokens} of {m.t_max} positions)")
        self.graph.replay()
        m._advance(1)
        return self.tok
