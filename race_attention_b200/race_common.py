"""Drop-in for scaling/race_common.py: hash geometry and the soft hash.

* ``build_planes_protos`` must be bit-identical to the reference
  (scaling/race_common.py:14-33): it draws the hyperplanes from the same seeded
  CPU ``torch.Generator`` in the same call order, so models, checkpoints and
  tests see the same buckets.  This is the one piece that is necessarily alike.
* ``soft_hash_probs`` has the reference signature (scaling/race_common.py:36)
  and returns the same ``(probsK, probsQ, V2, N)``, computed by the library's
  CUDA soft-hash kernel with a CUDA backward.  ``protos_T`` must be the
  canonical +-1 corner matrix that ``build_planes_protos`` returns (the kernel
  derives corner signs from the bucket index); anything else raises.
"""
from __future__ import annotations

import itertools

import torch

from . import ops


def build_planes_protos(d_k, Kbits, L, M, device="cuda", share_planes=True, dtype=torch.float32, seed=0):
    """planes_T [d_k, L*Kbits] (or [M, d_k, L*Kbits]) and protos_T [Kbits, 2^Kbits]."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    if share_planes:
        planes = torch.randn(L, Kbits, d_k, generator=g)
        planes_T = planes.view(L * Kbits, d_k).T.contiguous()
    else:
        planes = torch.randn(M, L, Kbits, d_k, generator=g)
        planes_T = planes.view(M, L * Kbits, d_k).transpose(1, 2).contiguous()
    planes_T = planes_T.to(device=device, dtype=dtype)
    corners = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=Kbits)), dtype=dtype, device=device)
    return planes_T, corners.T.contiguous()


_checked_protos = {}


def check_protos(protos_T: torch.Tensor, Kbits: int) -> None:
    """Raise unless protos_T is the canonical corner matrix for Kbits (cached per tensor version)."""
    R = 1 << Kbits
    if tuple(protos_T.shape) != (Kbits, R):
        raise RuntimeError(f"protos_T must be [{Kbits}, {R}]")
    key = (protos_T.data_ptr(), protos_T.device, protos_T._version, Kbits)
    if key in _checked_protos:
        return
    ref = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=Kbits))).T
    if not torch.equal(protos_T.detach().to("cpu", torch.float32), ref):
        raise RuntimeError("protos_T is not the canonical corner matrix of build_planes_protos")
    if len(_checked_protos) > 256:
        _checked_protos.clear()
    _checked_protos[key] = True


class SoftHashFn(torch.autograd.Function):
    """probs = soft_hash(X) on the CUDA kernels, with the CUDA backward for dX."""

    @staticmethod
    def forward(ctx, X, planes_T, L, P, logit_scale):
        ctx.save_for_backward(X, planes_T)
        ctx.cfg = (L, P, logit_scale)
        return ops.soft_hash(X, planes_T, L, P, logit_scale)

    @staticmethod
    def backward(ctx, dprobs):
        X, planes_T = ctx.saved_tensors
        L, P, scale = ctx.cfg
        dX = ops.soft_hash_bwd(X, planes_T, dprobs, L, P, scale).view_as(X)
        return dX, None, None, None, None


def soft_hash_probs(Q, K, V, planes_T, protos_T, L, Kbits, M, share_planes=True, logit_scale=None):
    """(probsK, probsQ, V2, N) exactly as scaling/race_common.py:36-73 returns them.

    Q, K, V: [B,H,T,D] CUDA tensors.  probs are fp32 [N,T,L*2^Kbits] with
    N = M*B*H ordered (M,B,H); V2 is V packed the same way.
    """
    B, H, T, D = Q.shape
    N = M * B * H
    check_protos(protos_T, Kbits)

    def pack(Z):
        return Z.unsqueeze(0).expand(M, -1, -1, -1, -1).reshape(N, T, D)

    Qn, Kn = Q.reshape(B * H, T, D), K.reshape(B * H, T, D)
    if share_planes:
        pq = SoftHashFn.apply(Qn, planes_T, L, Kbits, logit_scale)
        pk = SoftHashFn.apply(Kn, planes_T, L, Kbits, logit_scale)
        if M > 1:
            pq = pq.unsqueeze(0).expand(M, -1, -1, -1).reshape(N, T, -1)
            pk = pk.unsqueeze(0).expand(M, -1, -1, -1).reshape(N, T, -1)
    else:
        pq = torch.cat([SoftHashFn.apply(Qn, planes_T[m], L, Kbits, logit_scale) for m in range(M)], 0)
        pk = torch.cat([SoftHashFn.apply(Kn, planes_T[m], L, Kbits, logit_scale) for m in range(M)], 0)
    return pk, pq, pack(V), N
