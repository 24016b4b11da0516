"""Incremental decoding with a persistent RACE state (no reference counterpart:
the reference's KV-cache branch raises, chat/nanochat/gpt.py:143-146).

The state of one layer is race_prefix_ref's (A_final, B_final)
(scaling/race_common.py:88-90) per key/value stream: A [B*Hkv, S] and
B [B*Hkv, S, D], float32.  Grouped-query attention: query head h of batch b
reads kv stream b*Hkv + h // (Hq // Hkv).
"""
from __future__ import annotations

import torch

from . import ops


class RaceDecodeState:
    def __init__(self, batch, n_kv_heads, head_dim, L, P, planes_T, eps=1e-6, logit_scale=None, device="cuda"):
        self.batch, self.n_kv_heads, self.head_dim = batch, n_kv_heads, head_dim
        self.L, self.P = L, P
        self.S = L << P
        self.eps = eps
        self.logit_scale = logit_scale
        self.planes_T = planes_T.to(device=device, dtype=torch.float32).contiguous()
        n = batch * n_kv_heads
        self.A = torch.zeros((n, self.S), dtype=torch.float32, device=device)
        self.B = torch.zeros((n, self.S, head_dim), dtype=torch.float32, device=device)
        self.tokens = 0

    def reset(self):
        self.A.zero_()
        self.B.zero_()
        self.tokens = 0

    def prefill(self, K, V):
        """Fold prefill keys/values [B, Hkv, T, D] into the state (continuing from it)."""
        B_, H, T, D = K.shape
        A, Bs = ops.state_from_prefill(K.reshape(B_ * H, T, D), V.reshape(B_ * H, T, D), self.planes_T, self.L,
                                       self.P, self.logit_scale, self.A, self.B)
        self.A.copy_(A)
        self.B.copy_(Bs)
        self.tokens += T

    def step(self, q, k, v):
        """One token: q [B, Hq, D], k/v [B, Hkv, D] -> out [B, Hq, D]; updates the state in place."""
        B_, Hq, D = q.shape
        out = ops.decode_step(q.reshape(B_ * Hq, D), k.reshape(-1, D), v.reshape(-1, D), self.planes_T, self.A,
                              self.B, self.L, self.P, self.eps, self.logit_scale)
        self.tokens += 1
        return out.view(B_, Hq, D)


def prefill_with_state(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None):
    """Prefill outputs for Q [B,Hq,T,D] over K/V [B,Hkv,T,D] plus the decode state.

    Returns (out [B,Hq,T,D], RaceDecodeState)."""
    B_, Hq, T, D = Q.shape
    Hkv = K.shape[1]
    group = Hq // Hkv
    st = RaceDecodeState(B_, Hkv, D, L, P, planes_T, eps, logit_scale, device=Q.device)
    if group == 1:
        out, A, Bs = ops.fwd_qkv(Q, K, V, planes_T, L, P, eps, logit_scale, return_state=True)
        st.A.copy_(A)
        st.B.copy_(Bs)
        st.tokens = T
        return out.view(B_, Hq, T, D), st
    Ke = K.repeat_interleave(group, dim=1)
    Ve = V.repeat_interleave(group, dim=1)
    out = ops.fwd_qkv(Q, Ke, Ve, planes_T, L, P, eps, logit_scale)
    st.prefill(K, V)
    return out.view(B_, Hq, T, D), st
