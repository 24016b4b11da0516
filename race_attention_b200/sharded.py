"""Sequence-sharded causal RACE across ranks (one process per GPU).

Rank r holds the contiguous token slice [r*T/W, (r+1)*T/W) of every stream.
The normaliser 1/(A_t + eps) is nonlinear in the running bucket mass, so the
readout must start from the exact prefix of all earlier ranks:

forward   A. local totals (A_tot [N,S], B_tot [N,S,D]) of this slice; its
             segment prefixes stay in the workspace
          -> all_gather -> prefix = sum of ranks < r (fixed order, float64)
          B. fused readout of the slice, that prefix added to every segment's
backward  A. the slice's gradients with a zero suffix at its end, and their
             start-state totals (gA_tot, gB_tot), given the prefix
          -> all_gather -> suffix = sum of ranks > r
          B. that suffix's (linear) share added to the gradients

The exchange is one all_gather_into_tensor of N*(S + S*D) float32 per rank and
direction (266 KB at N=8, S=128, D=64) into one [W, ...] buffer, then one
fixed-order float64 reduction over the earlier (or later) ranks.  Every message
carries a checksum of its exact bits (an integer sum and a position-weighted
integer sum of the float32 words, order independent and exact); a receiver that
finds a mismatch raises instead of using the corrupted state.  The compute
backend defaults to the CUDA library; anything with the same four methods can
stand in (the CPU tests use this to run the exchange logic on gloo ranks).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops

try:
    from torch.cuda import nvtx as _nvtx
except ImportError:  # pragma: no cover
    _nvtx = None

# Test hook (CPU tests only): called with the outgoing message after its checksum
# is computed, to stand for a transport that corrupts it.
_tamper_outgoing = None


class CudaShardBackend:
    def fwd_local(self, K, V, planes_T, L, P, scale):
        """(A_tot, B_tot, handle) of this shard."""
        return ops.fwd_local(K, V, planes_T, L, P, scale)

    def fwd_finish(self, handle, Q, eps, A0, B0):
        """(out, saved): saved = chunk states kept for the backward (None when unused)."""
        return ops.fwd_finish(handle, Q, A0, B0, eps, save=True)

    def bwd_local(self, Q, K, V, dO, planes_T, L, P, eps, scale, A0, B0, saved):
        """(gA_tot, gB_tot, handle) of this shard."""
        return ops.bwd_local(Q, K, V, dO, planes_T, L, P, eps, scale, A0, B0, saved)

    def bwd_finish(self, handle, gA, gB):
        return ops.bwd_finish(handle, gA, gB)


_CS_WORDS = 4  # two int64 checksums as float32 words


def _checksums(words):
    """[..., n] float32 -> [..., 2] int64: sum of the bit patterns and a
    position-weighted sum (weights 1..65521), both exact in wrapping int64."""
    bits = words.view(torch.int32).to(torch.int64)
    w = torch.arange(bits.shape[-1], device=bits.device, dtype=torch.int64) % 65521 + 1
    return torch.stack([bits.sum(-1), (bits * w).sum(-1)], -1)


class ExchangeCorrupted(RuntimeError):
    """A rank's exchanged state did not match its checksum."""


def _message(A, B):
    """This rank's message: (A, B) flattened to float32, then its checksum words."""
    body = torch.cat([A.reshape(-1), B.reshape(-1)]).float()
    return torch.cat([body, _checksums(body).view(torch.float32)]).contiguous()


def exchange(A, B, group=None, direction="prefix"):
    """Sum of the (A, B) totals of ranks before ('prefix') or after ('suffix') this one,
    in float64 and a fixed rank order (deterministic); every rank's message is
    checked against its checksum."""
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    N, S = A.shape
    D = B.shape[-1]
    if _nvtx is not None and A.is_cuda:
        _nvtx.range_push(f"race exchange ({direction})")
    try:
        msg = _message(A, B)
        if _tamper_outgoing is not None:
            msg = _tamper_outgoing(msg)
        flat = torch.empty(W * msg.numel(), dtype=msg.dtype, device=msg.device)
        dist.all_gather_into_tensor(flat, msg, group=group)
        allm = flat.view(W, msg.numel())
        body, cs = allm[:, :-_CS_WORDS], allm[:, -_CS_WORDS:].contiguous().view(torch.int64)
        bad = (_checksums(body) != cs).any(-1)
        if bool(bad.any()):
            raise ExchangeCorrupted(
                f"rank {r}: exchanged state of rank(s) {bad.nonzero().flatten().tolist()} fails its checksum")
        part = body[:r] if direction == "prefix" else body[r + 1:]
        acc = part.double().sum(0) if part.shape[0] else torch.zeros(body.shape[1], dtype=torch.float64,
                                                                       device=body.device)
        acc = acc.float()
        return acc[:N * S].reshape(N, S).contiguous(), acc[N * S:].reshape(N, S, D).contiguous()
    finally:
        if _nvtx is not None and A.is_cuda:
            _nvtx.range_pop()


class ShardedRaceFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, planes_T, L, P, eps, logit_scale, group, backend):
        shape = Q.shape
        D = shape[-1]
        Qn, Kn, Vn = (x.reshape(-1, x.shape[-2], D) for x in (Q, K, V))
        scale = ops.default_logit_scale(D) if logit_scale is None else float(logit_scale)
        A_tot, B_tot, handle = backend.fwd_local(Kn, Vn, planes_T, L, P, scale)
        A0, B0 = exchange(A_tot, B_tot, group, "prefix")
        out, saved = backend.fwd_finish(handle, Qn, eps, A0, B0)
        del handle
        ctx.save_for_backward(Qn, Kn, Vn, planes_T, A0, B0, saved)
        ctx.cfg = (L, P, eps, scale, group, backend, shape)
        return out.reshape(shape)

    @staticmethod
    def backward(ctx, dO):
        Qn, Kn, Vn, planes_T, A0, B0, saved = ctx.saved_tensors
        L, P, eps, scale, group, backend, shape = ctx.cfg
        dOn = dO.reshape(Qn.shape).contiguous()
        gA_tot, gB_tot, handle = backend.bwd_local(Qn, Kn, Vn, dOn, planes_T, L, P, eps, scale, A0, B0, saved)
        gA, gB = exchange(gA_tot, gB_tot, group, "suffix")
        dQ, dK, dV = backend.bwd_finish(handle, gA, gB)
        return dQ.reshape(shape), dK.reshape(shape), dV.reshape(shape), None, None, None, None, None, None, None


def race_causal_sharded(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None, group=None, backend=None):
    """Causal RACE of this rank's contiguous sequence slice, exact w.r.t. the full sequence."""
    return ShardedRaceFn.apply(Q, K, V, planes_T, L, P, eps, logit_scale, group, backend or CudaShardBackend())
