"""Drop-in for scaling/race_causal_cuda.py on B200.

* ``RaceCausalFn`` / ``race_cuda_fused`` -- the probability-level autograd op
  with the reference signature (scaling/race_causal_cuda.py:47-73):
  ``(probsK[N,T,S] f32, probsQ[N,T,S] f32, V2[N,T,D] f32, eps) -> out[N,T,D]``
  and gradients ``(gradProbsK, gradProbsQ, gradV2, None)``.
* ``RaceCausalCuda`` -- the ``[B,H,T,D]`` module with the reference
  constructor (scaling/race_causal_cuda.py:76-102).  Its forward runs the
  fused soft-hash + scan kernels without materialising the [N,T,S]
  probabilities; bf16 inputs stay bf16 end to end (fp32 state accumulation).
* ``race_causal`` / ``RaceQKVFn`` -- the fused op itself.
* ``fwd_chunk`` -- the reference's chunk heuristic
  (scaling/race_causal_cuda.py:33-44).  The library picks its own internal
  chunking; the value is accepted for API compatibility and does not change
  results.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
from torch.autograd import Function

from . import ops
from .race_common import build_planes_protos, check_protos, soft_hash_probs  # noqa: F401


def fwd_chunk(T):
    if T <= 4096:
        return int(T)
    e = int(math.ceil(math.log2(max(1.0, T / 48.0))))
    e = max(11, min(16, e))
    return min(1 << e, int(T))


class RaceCausalFn(Function):
    """out = causal RACE(probsK, probsQ, V2). Exact grads w.r.t. probsK/probsQ/V2."""

    @staticmethod
    def forward(ctx, probsK, probsQ, V2, eps):
        probsK = probsK.contiguous().float()
        probsQ = probsQ.contiguous().float()
        V2 = V2.contiguous().float()
        C = fwd_chunk(probsK.shape[1])
        out = ops.race_fused_fwd(probsK, probsQ, V2, float(eps), C)
        ctx.save_for_backward(probsK, probsQ, V2)
        ctx.eps = float(eps)
        ctx.chunk = C
        return out

    @staticmethod
    def backward(ctx, grad_out):
        probsK, probsQ, V2 = ctx.saved_tensors
        grad_out = grad_out.contiguous().float()
        gpk, gpq, gv = ops.race_backward(probsK, probsQ, V2, grad_out, ctx.eps, ctx.chunk)
        return gpk, gpq, gv, None


def race_cuda_fused(probsK, probsQ, V2, eps=1e-6):
    return RaceCausalFn.apply(probsK, probsQ, V2, eps)


class RaceQKVFn(Function):
    """Fused causal RACE layer on Q, K, V [N,T,D] or [B,H,T,D] (one plane set)."""

    @staticmethod
    def forward(ctx, Q, K, V, planes_T, L, P, eps, logit_scale):
        shape = Q.shape
        # the tcgen05 path keeps its chunk-start states for the backward (None elsewhere)
        out, saved = ops.fwd_qkv(Q, K, V, planes_T, L, P, eps, logit_scale, save=True)
        ctx.save_for_backward(Q, K, V, planes_T, saved)
        ctx.cfg = (L, P, eps, logit_scale, shape)
        return out.view(shape)

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, planes_T, saved = ctx.saved_tensors
        L, P, eps, scale, shape = ctx.cfg
        dQ, dK, dV = ops.bwd_qkv(Q, K, V, dO, planes_T, L, P, eps, scale, saved=saved)
        return dQ.view(shape), dK.view(shape), dV.view(shape), None, None, None, None, None


def race_causal(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None):
    """Causal RACE attention of Q, K, V [B,H,T,D] (or [N,T,D]) with planes_T [D, L*P]."""
    return RaceQKVFn.apply(Q, K, V, planes_T, L, P, eps, logit_scale)


class RaceBTHDFn(Function):
    """Fused causal RACE on q, k, v laid out [B,T,H,D] (tcgen05 configurations)."""

    @staticmethod
    def forward(ctx, q, k, v, planes_T, L, P, eps, logit_scale):
        out, saved = ops.fwd_bthd(q, k, v, planes_T, L, P, eps, logit_scale)
        ctx.save_for_backward(q, k, v, planes_T, saved)
        ctx.cfg = (L, P, eps, logit_scale)
        return out

    @staticmethod
    def backward(ctx, dO):
        q, k, v, planes_T, saved = ctx.saved_tensors
        L, P, eps, scale = ctx.cfg
        dq, dk, dv = ops.bwd_bthd(q, k, v, dO, planes_T, L, P, saved, eps, scale)
        return dq, dk, dv, None, None, None, None, None


def race_causal_bthd(q, k, v, planes_T, L, P, eps=1e-6, logit_scale=None):
    """Causal RACE of q, k, v [B,T,H,D] -> [B,T,H,D], the layout attention modules project
    into.  bf16 with D = 64, P = 4, L in {8, 16} reads and writes it in place through the
    kernels' tensor maps; other configurations run race_causal on [B,H,T,D] copies."""
    D = q.shape[-1]
    if q.dim() == 4 and q.dtype == k.dtype == v.dtype and ops.fast_path(q.dtype, D, L, P):
        return RaceBTHDFn.apply(q, k, v, planes_T, L, P, eps, logit_scale)
    t = lambda x: x.transpose(1, 2).contiguous()  # noqa: E731
    return race_causal(t(q), t(k), t(v), planes_T, L, P, eps, logit_scale).transpose(1, 2)


def nanochat_race_attention(q, k, v, planes_T, race_L, race_K, race_M=1, race_eps=1e-6):
    """The RACE branch of nanochat's CausalSelfAttention.forward (chat/nanochat/gpt.py:131-142):
    q, k, v [B,T,H,D] after rotary embedding and QK norm -> y [B,T,H,D] in q's dtype.
    The reference upcasts to fp32 and transposes to [B,H,T,D] around soft_hash_probs +
    RaceCausalFn and averages the M members, which with shared planes are identical copies;
    here bf16 activations stay bf16 (fp32 accumulation and state) and the layout is read in
    place."""
    del race_M  # shared planes: every ensemble member is the same computation
    if q.dtype == torch.bfloat16:
        return race_causal_bthd(q, k, v, planes_T, race_L, race_K, race_eps)
    y = race_causal_bthd(q.float(), k.float(), v.float(), planes_T, race_L, race_K, race_eps)
    return y.to(q.dtype)


class RaceCausalCuda(nn.Module):
    """Causal RACE over Q,K,V: [B,H,T,D] -> [B,H,T,D] on the B200 kernels.

    Same constructor and buffers (planes_T, protos_T) as the reference module,
    so state_dicts interchange.  ``logit_scale`` defaults to 1/sqrt(d_k), the
    reference's fixed soft-hash temperature (scaling/race_common.py:46).
    With ``share_planes=True`` the M ensemble members are identical copies in
    the reference (packM expands the same inputs through the same planes), so
    the ensemble mean equals one member and is computed once.
    """

    def __init__(self, d_k, Kbits, L, M, device="cuda", share_planes=True, eps=1e-6, seed=0, logit_scale=None):
        super().__init__()
        self.d_k, self.Kbits, self.L, self.M = d_k, Kbits, L, M
        self.share_planes = share_planes
        self.eps = eps
        self.logit_scale = logit_scale
        planes_T, protos_T = build_planes_protos(d_k, Kbits, L, M, device=device, share_planes=share_planes,
                                                 seed=seed)
        self.register_buffer("planes_T", planes_T)
        self.register_buffer("protos_T", protos_T)

    def forward(self, Q, K, V):
        check_protos(self.protos_T, self.Kbits)
        if self.share_planes:
            return race_causal(Q, K, V, self.planes_T, self.L, self.Kbits, self.eps, self.logit_scale)
        outs = [race_causal(Q, K, V, self.planes_T[m], self.L, self.Kbits, self.eps, self.logit_scale)
                for m in range(self.M)]
        return torch.stack(outs, 0).mean(0)
