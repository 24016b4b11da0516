"""Caller harness for the config-5 measurement: a nanochat-shaped GPT whose every attention
layer is causal RACE on the tcgen05 kernels.

Structure follows the reference caller (chat/nanochat/gpt.py:55-176): token embedding,
blocks of pre-norm attention and ReLU^2 MLP with parameter-free RMSNorm, rotary position
embedding and QK norm in the attention, planes of layer i seeded with i
(chat/nanochat/gpt.py:284-286 via build_planes_protos), an untied LM head.  The RACE call
takes q, k, v in the [B, T, H, D] layout the projections produce (nanochat_race_attention:
no transposes).  Value embeddings, sliding windows and the KV cache of the reference model
are not part of this harness.  Linear layers keep fp32 master weights and run in the
activation dtype (bf16).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .race_causal_cuda import nanochat_race_attention
from .race_common import build_planes_protos


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    mlp_hidden: int = 3072
    race_L: int = 16
    race_P: int = 4
    race_eps: float = 1e-6
    rope_base: float = 10000.0


def _rms(x):
    return F.rms_norm(x, (x.size(-1),))


class _Linear(nn.Linear):
    """fp32 master weight, matmul in the input's dtype."""

    def forward(self, x):
        return F.linear(x, self.weight.to(x.dtype))


def _rotary(x, cos, sin):
    # x [B, T, H, D]: rotate the two halves of the head dimension by the position angles
    h = x.shape[-1] // 2
    a, b = x[..., :h], x[..., h:]
    return torch.cat([a * cos + b * sin, b * cos - a * sin], dim=-1)


class RaceAttention(nn.Module):
    def __init__(self, cfg: GPTConfig, layer_idx: int):
        super().__init__()
        self.cfg = cfg
        self.n_head = cfg.n_head
        self.head_dim = cfg.n_embd // cfg.n_head
        self.c_q = _Linear(cfg.n_embd, cfg.n_embd, bias=False)
        self.c_k = _Linear(cfg.n_embd, cfg.n_embd, bias=False)
        self.c_v = _Linear(cfg.n_embd, cfg.n_embd, bias=False)
        self.c_proj = _Linear(cfg.n_embd, cfg.n_embd, bias=False)
        planes_T, _ = build_planes_protos(self.head_dim, cfg.race_P, cfg.race_L, 1, device="cpu", seed=layer_idx)
        self.register_buffer("planes_T", planes_T)

    def forward(self, x, cos, sin):
        B, T, C = x.shape
        q = self.c_q(x).view(B, T, self.n_head, self.head_dim)
        k = self.c_k(x).view(B, T, self.n_head, self.head_dim)
        v = self.c_v(x).view(B, T, self.n_head, self.head_dim)
        q, k = _rms(_rotary(q, cos, sin)) * 1.2, _rms(_rotary(k, cos, sin)) * 1.2  # QK norm, sharpened
        y = nanochat_race_attention(q, k, v, self.planes_T, self.cfg.race_L, self.cfg.race_P, 1, self.cfg.race_eps)
        return self.c_proj(y.reshape(B, T, C))


class MLP(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.c_fc = _Linear(cfg.n_embd, cfg.mlp_hidden, bias=False)
        self.c_proj = _Linear(cfg.mlp_hidden, cfg.n_embd, bias=False)

    def forward(self, x):
        return self.c_proj(F.relu(self.c_fc(x)).square())


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig, layer_idx: int):
        super().__init__()
        self.attn = RaceAttention(cfg, layer_idx)
        self.mlp = MLP(cfg)

    def forward(self, x, cos, sin):
        x = x + self.attn(_rms(x), cos, sin)
        return x + self.mlp(_rms(x))


class RaceGPT(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.cfg = cfg
        self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.blocks = nn.ModuleList(Block(cfg, i) for i in range(cfg.n_layer))
        self.lm_head = _Linear(cfg.n_embd, cfg.vocab_size, bias=False)

    def init_weights(self, std: float = 0.02):
        for name, p in self.named_parameters():
            nn.init.normal_(p, mean=0.0, std=std)

    def _angles(self, T, device, dtype):
        hd = self.cfg.n_embd // self.cfg.n_head
        inv = self.cfg.rope_base ** (-torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd)
        ang = torch.outer(torch.arange(T, device=device, dtype=torch.float32), inv)
        return ang.cos().to(dtype)[None, :, None, :], ang.sin().to(dtype)[None, :, None, :]

    def forward(self, idx, targets=None, dtype=torch.bfloat16):
        B, T = idx.shape
        cos, sin = self._angles(T, idx.device, dtype)
        x = _rms(self.wte(idx).to(dtype))
        for blk in self.blocks:
            x = blk(x, cos, sin)
        logits = self.lm_head(_rms(x))
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.size(-1)), targets.view(-1))
