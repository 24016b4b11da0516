"""Caller harness for the config-4 measurement: hybrid decode with the Llama-3.2-1B
architecture (random-init bf16 weights), odd layers RACE attention, even layers softmax GQA.

The reference has no decode path for RACE (chat/nanochat/gpt.py:143-146 raises); this
harness is where the library's fused decode step (race_decode_step through RaceDecodeState)
meets a real model loop: a batched prefill that leaves each RACE layer's (A, B) state and
each softmax layer's KV cache, then greedy decode steps, each one fused RACE state update +
readout per RACE layer (grouped-query: 32 query heads read 8 kv states) and one SDPA call
over the cache per softmax layer.  Architecture: 16 layers, hidden 2048, 32 / 8 heads,
head_dim 64, SwiGLU MLP 8192, RMSNorm (eps 1e-5), RoPE theta 500000, vocabulary 128256 with
the LM head tied to the embedding.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

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
        self.q = nn.Linear(cfg.hidden, cfg.n_head * hd, bias=False)
        self.k = nn.Linear(cfg.hidden, cfg.n_kv_head * hd, bias=False)
        self.v = nn.Linear(cfg.hidden, cfg.n_kv_head * hd, bias=False)
        self.o = nn.Linear(cfg.n_head * hd, cfg.hidden, bias=False)
        self.gate = nn.Linear(cfg.hidden, cfg.mlp_hidden, bias=False)
        self.up = nn.Linear(cfg.hidden, cfg.mlp_hidden, bias=False)
        self.down = nn.Linear(cfg.mlp_hidden, cfg.hidden, bias=False)
        if self.race:
            planes_T, _ = build_planes_protos(hd, cfg.race_P, cfg.race_L, 1, device="cpu", seed=idx)
            self.register_buffer("planes_T", planes_T)
        self.state = None      # RACE layers: RaceDecodeState
        self.cache = None      # softmax layers: (K, V) [B, Hkv, Tmax, D]
        self.length = 0

    def _qkv(self, x, cos, sin):
        B, T, _ = x.shape
        cfg, hd = self.cfg, self.hd
        q = self.q(x).view(B, T, cfg.n_head, hd).transpose(1, 2)
        k = self.k(x).view(B, T, cfg.n_kv_head, hd).transpose(1, 2)
        v = self.v(x).view(B, T, cfg.n_kv_head, hd).transpose(1, 2)
        return _rope(q, cos, sin), _rope(k, cos, sin), v

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
            self.cache[0][b0:b0 + mb, :, :T].copy_(k)
            self.cache[1][b0:b0 + mb, :, :T].copy_(v)
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        self.length = T
        x = x + self.o(y.transpose(1, 2).reshape(mb, T, -1))
        h = self.ln2(x)
        return x + self.down(F.silu(self.gate(h)) * self.up(h))

    def step(self, x, cos, sin):
        """x [B, 1, hidden] at position self.length."""
        B = x.shape[0]
        q, k, v = self._qkv(self.ln1(x), cos, sin)  # [B, H, 1, D]
        if self.race:
            y = self.state.step(q[:, :, 0].contiguous(), k[:, :, 0].contiguous(), v[:, :, 0].contiguous())
            y = y.unsqueeze(2)
        else:
            t = self.length
            self.cache[0][:, :, t:t + 1].copy_(k)
            self.cache[1][:, :, t:t + 1].copy_(v)
            y = F.scaled_dot_product_attention(q, self.cache[0][:, :, :t + 1], self.cache[1][:, :, :t + 1],
                                               enable_gqa=True)
        self.length += 1
        x = x + self.o(y.transpose(1, 2).reshape(B, 1, -1))
        h = self.ln2(x)
        return x + self.down(F.silu(self.gate(h)) * self.up(h))


class HybridLlama(nn.Module):
    def __init__(self, cfg: HybridConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden)
        self.layers = nn.ModuleList(Layer(cfg, i) for i in range(cfg.n_layer))
        self.norm = _RMSNorm(cfg.hidden, cfg.norm_eps)

    def init_weights(self, std=0.02):
        for name, p in self.named_parameters():
            if p.dim() > 1:
                nn.init.normal_(p, mean=0.0, std=std)

    def _angles(self, pos0, T, device, dtype):
        hd = self.cfg.hidden // self.cfg.n_head
        inv = self.cfg.rope_theta ** (-torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd)
        ang = torch.outer(torch.arange(pos0, pos0 + T, device=device, dtype=torch.float32), inv)
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
        return torch.cat(nxt)

    @torch.no_grad()
    def logits_full(self, idx):
        """Last-position logits of a plain causal forward over idx [B, T] (no caches kept)."""
        B, T = idx.shape
        kept = [(layer.state, layer.cache, layer.length) for layer in self.layers]
        cos, sin = self._angles(0, T, idx.device, self.embed.weight.dtype)
        x = self.embed(idx)
        for layer in self.layers:
            x = layer.prefill(x, cos, sin, T, 0, B)
        for layer, (st, cache, length) in zip(self.layers, kept):  # the decode state stays as it was
            layer.state, layer.cache, layer.length = st, cache, length
        return self._logits(x[:, -1])

    @torch.no_grad()
    def step(self, tok):
        """tok [B] -> next-token ids [B] (greedy)."""
        pos = self.layers[0].length
        cos, sin = self._angles(pos, 1, tok.device, self.embed.weight.dtype)
        x = self.embed(tok[:, None])
        for layer in self.layers:
            x = layer.step(x, cos, sin)
        return self._logits(x[:, -1]).argmax(-1)
