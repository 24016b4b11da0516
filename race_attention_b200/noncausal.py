"""Non-causal RACE: the reference's BatchedACE with shared planes
(scaling/benchmark_time.py:77-166, misc/classification.py:257-308).

Every query reads the whole sequence's bucket summaries:
    b[s] = sum_t pk[t,s] V_t,   A[s] = sum_t pk[t,s],   E[s] = b[s] / (A[s] + eps),
    out_t = sum_s pq[t,s] E[s]
and the exact gradients
    dE = sum_t pq_t^T dO_t ; dpq_t = dO_t E^T ; db = dE / (A + eps) ;
    dA = -sum_d dE b / (A + eps)^2 ; dpk_t = dA + V_t db^T ; dV_t = pk_t db.
For bf16 with D = 64, P = 4, L in {8, 16} (the tcgen05 path) the whole layer is the
library's race_ace_fwd / race_ace_bwd: the bucket sums (b, A; dE) are single reductions over
tokens by the totals kernel, and every per-token product (out, dQ, dK, dV) is one fused
tile kernel that hashes the token, multiplies by the [S, D] summary on the tensor cores and
takes the soft-hash backward in its epilogue; no [N, T, S] tensor is formed.  Other
configurations (fp32, other shapes) compose the library's soft-hash and totals kernels with
batched GEMMs over [N, T, S] probabilities, as the reference module does.
"""
from __future__ import annotations

import torch
import torch.nn as nn
from torch.autograd import Function

from . import ops


def _streams(x):
    return x.reshape(-1, x.shape[-2], x.shape[-1]).contiguous()


class RaceNonCausalFn(Function):
    @staticmethod
    def forward(ctx, Q, K, V, planes_T, L, P, eps, logit_scale):
        shape, dtype = Q.shape, Q.dtype
        Qn, Kn, Vn = _streams(Q), _streams(K), _streams(V)
        scale = ops.default_logit_scale(Qn.shape[-1]) if logit_scale is None else float(logit_scale)
        if ops.fast_path(dtype, Qn.shape[-1], L, P):
            out, A, b = ops.ace_fwd(Qn, Kn, Vn, planes_T, L, P, eps, scale)
            ctx.save_for_backward(Qn, Kn, Vn, planes_T, A, b)
            ctx.cfg = (L, P, eps, scale, shape)
            return out.view(shape)
        A, b = ops.state_from_prefill(Kn, Vn, planes_T, L, P, scale)          # sum_t pk, sum_t pk^T V
        E = b / (A + eps).unsqueeze(-1)                                          # [N, S, D]
        pq = ops.soft_hash(Qn, planes_T, L, P, scale)                            # [N, T, S] fp32
        out = torch.bmm(pq, E).to(dtype)
        ctx.save_for_backward(Qn, Kn, Vn, planes_T, A, b)
        ctx.cfg = (L, P, eps, scale, shape)
        return out.view(shape)

    @staticmethod
    def backward(ctx, dO):
        Qn, Kn, Vn, planes_T, A, b = ctx.saved_tensors
        L, P, eps, scale, shape = ctx.cfg
        dOn = _streams(dO).to(Qn.dtype)
        if ops.fast_path(Qn.dtype, Qn.shape[-1], L, P):
            dQ, dK, dV = ops.ace_bwd(Qn, Kn, Vn, dOn, planes_T, A, b, L, P, eps, scale)
            return dQ.view(shape), dK.view(shape), dV.view(shape), None, None, None, None, None
        den = (A + eps).unsqueeze(-1)
        E = b / den
        _, dE = ops.state_from_prefill(Qn, dOn, planes_T, L, P, scale)        # sum_t pq^T dO
        db = dE / den
        dA = -(dE * b).sum(-1) / den.squeeze(-1) ** 2
        dpq = torch.bmm(dOn.float(), E.transpose(1, 2))                          # [N, T, S]
        dQ = ops.soft_hash_bwd(Qn, planes_T, dpq, L, P, scale)
        del dpq
        dpk = torch.baddbmm(dA.unsqueeze(1), Vn.float(), db.transpose(1, 2))     # dA + V db^T
        dK = ops.soft_hash_bwd(Kn, planes_T, dpk, L, P, scale)
        del dpk
        pk = ops.soft_hash(Kn, planes_T, L, P, scale)
        dV = torch.bmm(pk, db).to(Vn.dtype)
        return dQ.view(shape), dK.view(shape), dV.view(shape), None, None, None, None, None


def race_noncausal(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None):
    """Non-causal RACE of Q, K, V [N,T,D] or [B,H,T,D] with planes_T [D, L*P]."""
    return RaceNonCausalFn.apply(Q, K, V, planes_T, L, P, eps, logit_scale)


class BatchedACE(nn.Module):
    """Drop-in for the reference module with shared planes (scaling/benchmark_time.py:77-102):
    same buffers (planes_T [d_k, L*K] from randn(L, K, d_k), protos_T [K, 2^K]) and
    forward(Khf, Vhf, Qhf) on [M, B, T, H, d_k].  The temperature logit_temp (soft-hash
    logits tanh(proj) / exp(logit_temp)) is a fixed value here: the library's soft hash
    takes its scale as an argument and does not differentiate with respect to it."""

    def __init__(self, d_k, K, L, M, device="cuda", share_planes=True, logit_temp=0.0):
        super().__init__()
        if not share_planes:
            raise NotImplementedError("only shared planes (every ensemble member the same planes)")
        import itertools
        self.d_k, self.K, self.L, self.M = d_k, K, L, M
        planes = torch.randn(L, K, d_k, device=device)
        self.register_buffer("planes_T", planes.view(L * K, d_k).T.contiguous())
        corners = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=K)), device=device)
        self.register_buffer("protos_T", corners.T.contiguous())
        self.register_buffer("logit_temp", torch.tensor(float(logit_temp), device=device))

    def forward(self, Khf, Vhf, Qhf, eps: float = 1e-6):
        M, B, T, H, dk = Khf.shape
        scale = float(self.logit_temp.exp().clamp(1e-2, 10.0))
        t = lambda x: x.permute(0, 1, 3, 2, 4).reshape(M * B * H, T, dk)  # noqa: E731
        out = race_noncausal(t(Qhf), t(Khf), t(Vhf), self.planes_T, self.L, self.K, eps, 1.0 / scale)
        return out.view(M, B, H, T, dk).permute(0, 1, 3, 2, 4)
