"""Torch-level calls into the C ABI (no autograd here; see race_causal_cuda.py).

Each function validates its tensors the way the reference extension does
(CUDA-only, dtype, rank -> RuntimeError, kernels/gpu/forward_kernel.cu:112-114,
kernels/gpu/backward_kernels.cu:176-179), allocates outputs and workspace with
torch on the inputs' device, and launches on torch's current stream under a
device guard.  torch is only plumbing here: memory, streams and devices.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_DT = {torch.float32: _lib.RACE_F32, torch.bfloat16: _lib.RACE_BF16}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _check_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("CUDA only")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("all tensors must be on the same CUDA device")
    return dev


def _dtype_code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {t.dtype} (float32 or bfloat16)") from None


def _dtype_code_of(dtype):
    try:
        return _DT[dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {dtype} (float32 or bfloat16)") from None


def _workspace(op, N, T, S, D, L, P, dtype, dev):
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.race_workspace_bytes(op, N, T, S, D, L, P, dtype, 0, ctypes.byref(nbytes)),
               "race_workspace_bytes")
    n = int(nbytes.value)
    return torch.empty(max(n, 1), dtype=torch.uint8, device=dev), n


def _as_ntd(x, name):
    if x.dim() == 4:
        x = x.reshape(-1, x.shape[2], x.shape[3])
    if x.dim() != 3:
        raise RuntimeError(f"{name} must be [N,T,D] or [B,H,T,D]")
    return x.contiguous()


def _opt_state(A, B, N, S, D, dev):
    if A is None and B is None:
        return None, None
    if A is None or B is None:
        raise RuntimeError("state A and B must be given together")
    A = A.to(device=dev, dtype=torch.float32).reshape(N, S).contiguous()
    B = B.to(device=dev, dtype=torch.float32).reshape(N, S, D).contiguous()
    return A, B


def fast_path(dtype, D, L, P) -> bool:
    """Whether the library runs the tcgen05 kernels for this configuration
    (same rule as csrc/fast_host.cuh: bf16, D=64, P=4, L in {8,16})."""
    return dtype == torch.bfloat16 and D == 64 and P == 4 and L in (8, 16)


def default_logit_scale(D: int) -> float:
    """The reference divides tanh(proj) by sqrt(D) (scaling/race_common.py:46,68)."""
    return 1.0 / math.sqrt(D)


# ---------------------------------------------------------------------------
# probability-level (reference extension surface)
def race_fused_fwd(probsK, probsQ, V2, eps, chunk=0, return_state=False):
    """out[N,T,D] = causal RACE forward (kernels/gpu/forward_kernel.cu:110 semantics)."""
    dev = _check_cuda(probsK, probsQ, V2)
    if probsK.dtype != torch.float32 or probsQ.dtype != torch.float32 or V2.dtype != torch.float32:
        raise RuntimeError("fp32 only")
    if probsK.dim() != 3 or probsQ.dim() != 3 or V2.dim() != 3:
        raise RuntimeError("shapes [N,T,S],[N,T,S],[N,T,D]")
    probsK, probsQ, V2 = probsK.contiguous(), probsQ.contiguous(), V2.contiguous()
    N, T, S = probsK.shape
    D = V2.shape[2]
    if probsQ.shape != probsK.shape or V2.shape[:2] != probsK.shape[:2]:
        raise RuntimeError("shapes [N,T,S],[N,T,S],[N,T,D]")
    out = torch.empty((N, T, D), dtype=torch.float32, device=dev)
    Af = torch.empty((N, S), dtype=torch.float32, device=dev) if return_state else None
    Bf = torch.empty((N, S, D), dtype=torch.float32, device=dev) if return_state else None
    if T == 0:
        if return_state:
            Af.zero_()
            Bf.zero_()
        return (out, Af, Bf) if return_state else out
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_FWD_PROBS, N, T, S, D, 0, 0, 0, dev)
        _lib.check(lib.race_fwd_probs(_ptr(probsK), _ptr(probsQ), _ptr(V2), _ptr(out), _ptr(Af), _ptr(Bf),
                                      N, T, S, D, float(eps), int(chunk), _ptr(ws), nb, _stream(dev)),
                   "race_fwd_probs")
    return (out, Af, Bf) if return_state else out


def race_backward(probsK, probsQ, V2, grad_out, eps, chunk=0):
    """[gradProbsK, gradProbsQ, gradV] (kernels/gpu/backward_kernels.cu:174 semantics)."""
    dev = _check_cuda(probsK, probsQ, V2, grad_out)
    for t in (probsK, probsQ, V2, grad_out):
        if t.dtype != torch.float32:
            raise RuntimeError("fp32 only")
    probsK, probsQ, V2, grad_out = (t.contiguous() for t in (probsK, probsQ, V2, grad_out))
    N, T, S = probsK.shape
    D = V2.shape[2]
    if S > 1024:
        raise RuntimeError("S must be <= 1024")
    gpk = torch.empty_like(probsK)
    gpq = torch.empty_like(probsQ)
    gv = torch.empty_like(V2)
    if T == 0:
        return [gpk, gpq, gv]
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_BWD_PROBS, N, T, S, D, 0, 0, 0, dev)
        _lib.check(lib.race_bwd_probs(_ptr(probsK), _ptr(probsQ), _ptr(V2), _ptr(grad_out), _ptr(gpk), _ptr(gpq),
                                      _ptr(gv), N, T, S, D, float(eps), int(chunk), _ptr(ws), nb, _stream(dev)),
                   "race_bwd_probs")
    return [gpk, gpq, gv]


# ---------------------------------------------------------------------------
# soft hash
def soft_hash(X, planes_T, L, P, logit_scale=None):
    """probs[N,T,L*2^P] fp32 of X [N,T,D] (bf16 or fp32)."""
    dev = _check_cuda(X, planes_T)
    X = _as_ntd(X, "X")
    N, T, D = X.shape
    S = L << P
    planes_T = planes_T.to(torch.float32).contiguous()
    if planes_T.shape != (D, L * P):
        raise RuntimeError(f"planes_T must be [D, L*P] = [{D}, {L * P}]")
    scale = default_logit_scale(D) if logit_scale is None else float(logit_scale)
    probs = torch.empty((N, T, S), dtype=torch.float32, device=dev)
    if N * T == 0:
        return probs
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.race_soft_hash(_ptr(X), _dtype_code(X), _ptr(planes_T), _ptr(probs), N, T, D, L, P, scale,
                                      _stream(dev)), "race_soft_hash")
    return probs


def soft_hash_bwd(X, planes_T, dprobs, L, P, logit_scale=None):
    dev = _check_cuda(X, planes_T, dprobs)
    X = _as_ntd(X, "X")
    N, T, D = X.shape
    planes_T = planes_T.to(torch.float32).contiguous()
    dprobs = dprobs.to(torch.float32).reshape(N, T, L << P).contiguous()
    scale = default_logit_scale(D) if logit_scale is None else float(logit_scale)
    dX = torch.empty_like(X)
    if N * T == 0:
        return dX
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.race_soft_hash_bwd(_ptr(X), _dtype_code(X), _ptr(planes_T), _ptr(dprobs), _ptr(dX), N, T, D,
                                          L, P, scale, _stream(dev)), "race_soft_hash_bwd")
    return dX


# ---------------------------------------------------------------------------
# fused layer
def _qkv_common(Q, K, V, planes_T, L, P, logit_scale):
    dev = _check_cuda(Q, K, V, planes_T)
    Q, K, V = _as_ntd(Q, "Q"), _as_ntd(K, "K"), _as_ntd(V, "V")
    if not (Q.shape == K.shape == V.shape):
        raise RuntimeError("Q, K, V must have the same shape")
    if not (Q.dtype == K.dtype == V.dtype):
        raise RuntimeError("Q, K, V must have the same dtype")
    N, T, D = Q.shape
    planes_T = planes_T.to(torch.float32).contiguous()
    if planes_T.shape != (D, L * P):
        raise RuntimeError(f"planes_T must be [D, L*P] = [{D}, {L * P}]")
    scale = default_logit_scale(D) if logit_scale is None else float(logit_scale)
    return dev, Q, K, V, planes_T, N, T, D, L << P, scale


def saved_bytes(N, T, D, L, P, dtype) -> int:
    """Size of the chunk-state buffer a saving forward keeps for the backward (0: not used)."""
    nb = ctypes.c_size_t(0)
    _lib.check(_lib.load().race_saved_bytes(N, T, D, L, P, _dtype_code_of(dtype), ctypes.byref(nb)),
               "race_saved_bytes")
    return int(nb.value)


def fwd_qkv(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None, A0=None, B0=None, return_state=False,
            save=False):
    """Fused soft hash + causal scan + readout; out has Q's dtype and [N,T,D] shape.
    save=True also returns the chunk-state buffer for bwd_qkv(saved=...) (None when unused)."""
    dev, Q, K, V, planes_T, N, T, D, S, scale = _qkv_common(Q, K, V, planes_T, L, P, logit_scale)
    A0, B0 = _opt_state(A0, B0, N, S, D, dev)
    out = torch.empty_like(Q)
    Af = torch.empty((N, S), dtype=torch.float32, device=dev) if return_state else None
    Bf = torch.empty((N, S, D), dtype=torch.float32, device=dev) if return_state else None
    lib = _lib.load()
    saved = None
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_FWD_QKV, N, T, S, D, L, P, _dtype_code(Q), dev)
        sb = saved_bytes(N, T, D, L, P, Q.dtype) if save else 0
        if sb:
            saved = torch.empty(sb, dtype=torch.uint8, device=dev)
        _lib.check(lib.race_fwd_qkv_save(_ptr(Q), _ptr(K), _ptr(V), _dtype_code(Q), _ptr(planes_T), _ptr(out),
                                         _ptr(A0), _ptr(B0), _ptr(Af), _ptr(Bf), _ptr(saved), sb, N, T, D, L, P,
                                         float(eps), scale, _ptr(ws), nb, _stream(dev)), "race_fwd_qkv")
    res = (out, Af, Bf) if return_state else (out,)
    if save:
        res = res + (saved,)
    return res if len(res) > 1 else res[0]


def bwd_qkv(Q, K, V, dO, planes_T, L, P, eps=1e-6, logit_scale=None, A0=None, B0=None, gA=None, gB=None,
            return_state_grad=False, saved=None):
    """(dQ, dK, dV[, dA0, dB0]) of the fused layer.  saved: the buffer of fwd_qkv(save=True) on the
    same inputs (skips rebuilding the forward's chunk states)."""
    dev, Q, K, V, planes_T, N, T, D, S, scale = _qkv_common(Q, K, V, planes_T, L, P, logit_scale)
    dO = _as_ntd(dO, "dO").to(Q.dtype)
    A0, B0 = _opt_state(A0, B0, N, S, D, dev)
    gA, gB = _opt_state(gA, gB, N, S, D, dev)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    dA0 = torch.empty((N, S), dtype=torch.float32, device=dev) if return_state_grad else None
    dB0 = torch.empty((N, S, D), dtype=torch.float32, device=dev) if return_state_grad else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_BWD_QKV, N, T, S, D, L, P, _dtype_code(Q), dev)
        sb = saved.numel() if saved is not None else 0
        _lib.check(lib.race_bwd_qkv_saved(_ptr(Q), _ptr(K), _ptr(V), _ptr(dO), _dtype_code(Q), _ptr(planes_T),
                                          _ptr(saved), sb, _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(A0), _ptr(B0),
                                          _ptr(gA), _ptr(gB), _ptr(dA0), _ptr(dB0), N, T, D, L, P, float(eps), scale,
                                          _ptr(ws), nb, _stream(dev)), "race_bwd_qkv")
    return (dQ, dK, dV, dA0, dB0) if return_state_grad else (dQ, dK, dV)


def _bthd_common(Q, K, V, planes_T, L, P, logit_scale):
    dev = _check_cuda(Q, K, V, planes_T)
    if Q.dim() != 4 or not (Q.shape == K.shape == V.shape):
        raise RuntimeError("Q, K, V must have the same [B,T,H,D] shape")
    if not (Q.dtype == K.dtype == V.dtype):
        raise RuntimeError("Q, K, V must have the same dtype")
    Bn, T, H, D = Q.shape
    if not fast_path(Q.dtype, D, L, P):
        raise RuntimeError("the [B,T,H,D] layout needs bf16, D=64, P=4, L in {8,16}")
    planes_T = planes_T.to(torch.float32).contiguous()
    if planes_T.shape != (D, L * P):
        raise RuntimeError(f"planes_T must be [D, L*P] = [{D}, {L * P}]")
    scale = default_logit_scale(D) if logit_scale is None else float(logit_scale)
    return dev, Q.contiguous(), K.contiguous(), V.contiguous(), planes_T, Bn, T, H, D, L << P, scale


def fwd_bthd(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None):
    """Fused layer on [B,T,H,D] activations (no transposes): (out [B,T,H,D], saved chunk states)."""
    dev, Q, K, V, planes_T, Bn, T, H, D, S, scale = _bthd_common(Q, K, V, planes_T, L, P, logit_scale)
    N = Bn * H
    out = torch.empty_like(Q)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_FWD_QKV, N, T, S, D, L, P, _dtype_code(Q), dev)
        sb = saved_bytes(N, T, D, L, P, Q.dtype)
        saved = torch.empty(max(sb, 1), dtype=torch.uint8, device=dev)
        _lib.check(lib.race_fwd_bthd(_ptr(Q), _ptr(K), _ptr(V), _dtype_code(Q), _ptr(planes_T), _ptr(out), _ptr(saved),
                                     sb, Bn, T, H, D, L, P, float(eps), scale, _ptr(ws), nb, _stream(dev)),
                   "race_fwd_bthd")
    return out, saved


def bwd_bthd(Q, K, V, dO, planes_T, L, P, saved, eps=1e-6, logit_scale=None):
    """(dQ, dK, dV) [B,T,H,D] of fwd_bthd, reusing its saved chunk states."""
    dev, Q, K, V, planes_T, Bn, T, H, D, S, scale = _bthd_common(Q, K, V, planes_T, L, P, logit_scale)
    N = Bn * H
    dO = dO.to(Q.dtype).contiguous()
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_BWD_QKV, N, T, S, D, L, P, _dtype_code(Q), dev)
        _lib.check(lib.race_bwd_bthd(_ptr(Q), _ptr(K), _ptr(V), _ptr(dO), _dtype_code(Q), _ptr(planes_T), _ptr(saved),
                                     saved.numel(), _ptr(dQ), _ptr(dK), _ptr(dV), Bn, T, H, D, L, P, float(eps), scale,
                                     _ptr(ws), nb, _stream(dev)), "race_bwd_bthd")
    return dQ, dK, dV


def state_from_prefill(K, V, planes_T, L, P, logit_scale=None, A0=None, B0=None):
    """(A[N,S], B[N,S,D]) fp32 state after the prefill tokens K, V [N,T,D]."""
    dev, K, _, V, planes_T, N, T, D, S, scale = _qkv_common(K, K, V, planes_T, L, P, logit_scale)
    A0, B0 = _opt_state(A0, B0, N, S, D, dev)
    A = torch.empty((N, S), dtype=torch.float32, device=dev)
    B = torch.empty((N, S, D), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_STATE, N, T, S, D, L, P, _dtype_code(K), dev)
        _lib.check(lib.race_state_from_prefill(_ptr(K), _ptr(V), _dtype_code(K), _ptr(planes_T), _ptr(A0), _ptr(B0),
                                               _ptr(A), _ptr(B), N, T, D, L, P, scale, _ptr(ws), nb, _stream(dev)),
                   "race_state_from_prefill")
    return A, B


def ace_fwd(Q, K, V, planes_T, L, P, eps=1e-6, logit_scale=None):
    """Non-causal RACE forward on [N,T,D] (tcgen05 path only: bf16, D=64, P=4, L in {8,16}):
    (out [N,T,D], A [N,S], B [N,S,D]); A and B are the bucket summaries the backward takes."""
    dev, Q, K, V, planes_T, N, T, D, S, scale = _qkv_common(Q, K, V, planes_T, L, P, logit_scale)
    if not fast_path(Q.dtype, D, L, P):
        raise RuntimeError("race_ace_fwd: bf16, D=64, P=4, L in {8,16} only")
    out = torch.empty_like(Q)
    A = torch.empty((N, S), dtype=torch.float32, device=dev)
    B = torch.empty((N, S, D), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_ACE_FWD, N, T, S, D, L, P, _dtype_code(Q), dev)
        _lib.check(lib.race_ace_fwd(_ptr(Q), _ptr(K), _ptr(V), _dtype_code(Q), _ptr(planes_T), _ptr(out), _ptr(A),
                                    _ptr(B), N, T, D, L, P, float(eps), scale, _ptr(ws), nb, _stream(dev)),
                   "race_ace_fwd")
    return out, A, B


def ace_bwd(Q, K, V, dO, planes_T, A, B, L, P, eps=1e-6, logit_scale=None):
    """(dQ, dK, dV) [N,T,D] of ace_fwd, from its summaries A, B."""
    dev, Q, K, V, planes_T, N, T, D, S, scale = _qkv_common(Q, K, V, planes_T, L, P, logit_scale)
    if not fast_path(Q.dtype, D, L, P):
        raise RuntimeError("race_ace_bwd: bf16, D=64, P=4, L in {8,16} only")
    dO = _as_ntd(dO, "dO").to(Q.dtype)
    _check_cuda(Q, dO, A, B)
    A = A.float().reshape(N, S).contiguous()
    B = B.float().reshape(N, S, D).contiguous()
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_ACE_BWD, N, T, S, D, L, P, _dtype_code(Q), dev)
        _lib.check(lib.race_ace_bwd(_ptr(Q), _ptr(K), _ptr(V), _ptr(dO), _dtype_code(Q), _ptr(planes_T), _ptr(A),
                                    _ptr(B), _ptr(dQ), _ptr(dK), _ptr(dV), N, T, D, L, P, float(eps), scale,
                                    _ptr(ws), nb, _stream(dev)),
                   "race_ace_bwd")
    return dQ, dK, dV


class FwdSplit:
    """What race_fwd_local leaves for race_fwd_finish: K, V and the workspace."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def fwd_local(K, V, planes_T, L, P, logit_scale=None):
    """First half of a shard's forward: (A_tot[N,S], B_tot[N,S,D], handle) -- this shard's state
    totals; the handle (holding its segment prefixes) goes to fwd_finish."""
    dev, K, _, V, planes_T, N, T, D, S, scale = _qkv_common(K, K, V, planes_T, L, P, logit_scale)
    A = torch.empty((N, S), dtype=torch.float32, device=dev)
    B = torch.empty((N, S, D), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_FWD_SPLIT, N, T, S, D, L, P, _dtype_code(K), dev)
        _lib.check(lib.race_fwd_local(_ptr(K), _ptr(V), _dtype_code(K), _ptr(planes_T), _ptr(A), _ptr(B), N, T, D,
                                      L, P, scale, _ptr(ws), nb, _stream(dev)), "race_fwd_local")
    return A, B, FwdSplit(K=K, V=V, planes_T=planes_T, L=L, P=P, scale=scale, ws=ws, nb=nb, dev=dev)


def fwd_finish(h, Q, A0=None, B0=None, eps=1e-6, save=False):
    """Second half: out (and, with save=True, the chunk-state buffer for bwd_local/bwd_qkv, None when
    unused) given A0/B0 = the sum of the totals of all earlier shards."""
    dev, Q, K, V, planes_T, N, T, D, S, _ = _qkv_common(Q, h.K, h.V, h.planes_T, h.L, h.P, h.scale)
    A0, B0 = _opt_state(A0, B0, N, S, D, dev)
    out = torch.empty_like(Q)
    lib = _lib.load()
    saved = None
    with torch.cuda.device(dev):
        sb = saved_bytes(N, T, D, h.L, h.P, Q.dtype) if save else 0
        if sb:
            saved = torch.empty(sb, dtype=torch.uint8, device=dev)
        _lib.check(lib.race_fwd_finish(_ptr(Q), _ptr(K), _ptr(V), _dtype_code(Q), _ptr(planes_T), _ptr(out),
                                       _ptr(saved), sb, _ptr(A0), _ptr(B0), N, T, D, h.L, h.P, float(eps), h.scale,
                                       _ptr(h.ws), h.nb, _stream(dev)), "race_fwd_finish")
    return (out, saved) if save else out


class BwdSplit:
    """What race_bwd_local leaves for race_bwd_finish: the inputs and the workspace."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def bwd_local(Q, K, V, dO, planes_T, L, P, eps=1e-6, logit_scale=None, A0=None, B0=None, saved=None):
    """First half of a shard's backward: (gA_tot[N,S], gB_tot[N,S,D], handle) -- this shard's
    gradient totals for its start state; the handle goes to bwd_finish."""
    dev, Q, K, V, planes_T, N, T, D, S, scale = _qkv_common(Q, K, V, planes_T, L, P, logit_scale)
    dO = _as_ntd(dO, "dO").to(Q.dtype)
    A0, B0 = _opt_state(A0, B0, N, S, D, dev)
    gA = torch.empty((N, S), dtype=torch.float32, device=dev)
    gB = torch.empty((N, S, D), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws, nb = _workspace(_lib.OP_BWD_SPLIT, N, T, S, D, L, P, _dtype_code(Q), dev)
        sb = saved.numel() if saved is not None else 0
        _lib.check(lib.race_bwd_local(_ptr(Q), _ptr(K), _ptr(V), _ptr(dO), _dtype_code(Q), _ptr(planes_T),
                                      _ptr(saved), sb, _ptr(A0), _ptr(B0), _ptr(gA), _ptr(gB), N, T, D, L, P,
                                      float(eps), scale, _ptr(ws), nb, _stream(dev)), "race_bwd_local")
    h = BwdSplit(Q=Q, K=K, V=V, dO=dO, planes_T=planes_T, L=L, P=P, eps=eps, scale=scale, A0=A0, B0=B0,
                 saved=saved, ws=ws, nb=nb, dev=dev)
    return gA, gB, h


def bwd_finish(h, gA=None, gB=None):
    """Second half: (dQ, dK, dV) given gA/gB = the sum of the totals of all later shards."""
    N, T, D = h.Q.shape
    S = h.L << h.P
    gA, gB = _opt_state(gA, gB, N, S, D, h.dev)
    dQ, dK, dV = torch.empty_like(h.Q), torch.empty_like(h.K), torch.empty_like(h.V)
    lib = _lib.load()
    with torch.cuda.device(h.dev):
        sb = h.saved.numel() if h.saved is not None else 0
        _lib.check(lib.race_bwd_finish(_ptr(h.Q), _ptr(h.K), _ptr(h.V), _ptr(h.dO), _dtype_code(h.Q),
                                       _ptr(h.planes_T), _ptr(h.saved), sb, _ptr(h.A0), _ptr(h.B0), _ptr(gA),
                                       _ptr(gB), _ptr(dQ), _ptr(dK), _ptr(dV), N, T, D, h.L, h.P, float(h.eps),
                                       h.scale, _ptr(h.ws), h.nb, _stream(h.dev)), "race_bwd_finish")
    return dQ, dK, dV


def decode_step(q, k, v, planes_T, A, B, L, P, eps=1e-6, logit_scale=None):
    """One decode token.  q [Nq,D], k/v [Nkv,D] (Nq = group*Nkv); updates A/B in place; returns out [Nq,D]."""
    dev = _check_cuda(q, k, v, planes_T, A, B)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if not (q.dtype == k.dtype == v.dtype):
        raise RuntimeError("q, k, v must have the same dtype")
    Nq, D = q.shape
    Nkv = k.shape[0]
    S = L << P
    if A.dtype != torch.float32 or B.dtype != torch.float32 or not A.is_contiguous() or not B.is_contiguous():
        raise RuntimeError("decode state A/B must be contiguous float32")
    if A.shape != (Nkv, S) or B.shape != (Nkv, S, D):
        raise RuntimeError(f"decode state must be A[{Nkv},{S}], B[{Nkv},{S},{D}]")
    planes_T = planes_T.to(torch.float32).contiguous()
    scale = default_logit_scale(D) if logit_scale is None else float(logit_scale)
    out = torch.empty_like(q)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.race_decode_step(_ptr(q), _ptr(k), _ptr(v), _dtype_code(q), _ptr(planes_T), _ptr(A), _ptr(B),
                                        _ptr(out), Nq, Nkv, D, L, P, float(eps), scale, _stream(dev)),
                   "race_decode_step")
    return out


def gqa_decode_splits(B, Hkv, t_max, device) -> int:
    """Key ranges per (batch row, kv head) for gqa_decode_attention: about 16 waves of
    two CTAs per SM over the whole grid, at least 512 cache slots per range, at most 64."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    want = -(-16 * 2 * sms // max(1, B * Hkv))
    return int(max(1, min(64, want, max(1, t_max // 512))))


def gqa_decode_workspace(B, Hq, Hkv, n_splits, device):
    """Zero-filled workspace for gqa_decode_attention (reused as is across calls)."""
    nbytes = int(_lib.load().race_gqa_decode_workspace_bytes(B, Hq, Hkv, int(n_splits)))
    if nbytes == 0:
        raise RuntimeError("invalid gqa_decode_attention workspace shape")
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def gqa_decode_attention(q, k_new, v_new, k_cache, v_cache, length, workspace, n_splits, softmax_scale=None):
    """Softmax GQA attention of one decode token over a bf16 KV cache (the softmax layers
    of a hybrid decoder).  q [B,Hq,64], k_new/v_new [B,Hkv,64], caches [B,Hkv,Tmax,64],
    length = int32 device tensor [1] holding the tokens already cached.  Stores k_new/v_new
    at position length, returns out [B,Hq,64]; length itself is not advanced."""
    dev = _check_cuda(q, k_new, v_new, k_cache, v_cache, length, workspace)
    for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new), ("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise RuntimeError(f"{name} must be contiguous bfloat16")
    if length.dtype != torch.int32 or length.numel() != 1:
        raise RuntimeError("length must be an int32 tensor with one element")
    B, Hq, D = q.shape
    Hkv, Tmax = k_cache.shape[1], k_cache.shape[2]
    if k_new.shape != (B, Hkv, D) or v_new.shape != (B, Hkv, D) or k_cache.shape != (B, Hkv, Tmax, D) \
            or v_cache.shape != k_cache.shape:
        raise RuntimeError("gqa_decode_attention: inconsistent shapes")
    lib = _lib.load()
    need = int(lib.race_gqa_decode_workspace_bytes(B, Hq, Hkv, int(n_splits)))
    if workspace.numel() * workspace.element_size() < need:
        raise RuntimeError(f"gqa_decode_attention workspace needs {need} bytes")
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    out = torch.empty_like(q)
    with torch.cuda.device(dev):
        _lib.check(lib.race_gqa_decode_attn(_ptr(q), _ptr(k_new), _ptr(v_new), _ptr(k_cache), _ptr(v_cache),
                                            _ptr(length), _ptr(out), _ptr(workspace), B, Hq, Hkv, Tmax, D,
                                            int(n_splits), scale, _stream(dev)), "race_gqa_decode_attn")
    return out
