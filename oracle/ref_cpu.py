"""The reference's own CPU path for one causal RACE layer -- BASELINE/TEST ONLY.

Used by ``bench.py --impl reference`` and the ``cpu_baseline`` leg to time what a
user of the reference runs on CPU: ``soft_hash_probs`` (torch CPU ops) feeding
``RaceCausalCPUFn`` over the reference's compiled OpenMP kernel
``race_prefix_mean_flat[_bw]`` (kernels/cpu/race_pref.cpp:36-220).

The kernel itself is the reference's: ``make -C oracle ref`` compiles
kernels/cpu/race_pref.cpp from the reference tree into ``oracle/_ref/``.  The
few lines of Python glue around it are restated here because the reference
tree does not exist where the benchmark runs:

* ``soft_hash_probs_ref`` -- scaling/race_common.py:36-73 (share_planes=True)
* ``RefRaceCausalCPUFn``  -- scaling/race_causal_cpu.py:33-72 (flatten with V
  expanded x S, einsum readout, einsum + prefix-mean backward)

When ``oracle/_ref`` was not built, ``available()`` is False and callers fall
back to the C restatement in ``oracle.py`` (reported as kind "port").
"""
from __future__ import annotations

import glob
import importlib.util
import math
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_EXT = None


def _ext():
    global _EXT
    if _EXT is None:
        cands = sorted(glob.glob(os.path.join(_HERE, "_ref", "race_pref_ref*.so")))
        if not cands:
            raise FileNotFoundError("oracle/_ref/race_pref_ref*.so not built (make -C oracle ref)")
        spec = importlib.util.spec_from_file_location("race_pref_ref", cands[0])
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _EXT = mod
    return _EXT


def available() -> bool:
    try:
        _ext()
        return True
    except Exception:
        return False


def soft_hash_probs_ref(Q, K, V, planes_T, protos_T, L, P):
    """scaling/race_common.py:44-73 with M=1, share_planes=True, on CPU tensors."""
    B, H, T, D = Q.shape
    N = B * H
    scale = math.sqrt(D)
    Km, Qm, Vm = K.reshape(N, T, D), Q.reshape(N, T, D), V.reshape(N, T, D)
    pT = planes_T.to(Qm.dtype)
    projK = (Km @ pT).view(N, T, L, P)
    projQ = (Qm @ pT).view(N, T, L, P)
    prT = protos_T.to(projK.dtype)
    logitsK = (projK.tanh() / scale) @ prT
    logitsQ = (projQ.tanh() / scale) @ prT
    R = prT.shape[1]
    probsK = torch.softmax(logitsK.float(), dim=-1).reshape(N, T, L * R)
    probsQ = torch.softmax(logitsQ.float(), dim=-1).reshape(N, T, L * R)
    return probsK, probsQ, Vm, N


class RefRaceCausalCPUFn(torch.autograd.Function):
    """scaling/race_causal_cpu.py:41-72 over the reference's compiled kernel."""

    @staticmethod
    def forward(ctx, probsK, probsQ, V2, eps):
        ext = _ext()
        probsK = probsK.contiguous().float()
        probsQ = probsQ.contiguous().float()
        V2 = V2.contiguous().float()
        N, T, S = probsK.shape
        D = V2.shape[2]
        pk_flat = probsK.permute(0, 2, 1).reshape(N * S, T).contiguous()
        v_flat = V2.unsqueeze(1).expand(N, S, T, D).reshape(N * S, T, D).contiguous()
        E = ext.race_prefix_mean_flat(pk_flat, v_flat, float(eps)).view(N, S, T, D)
        out = torch.einsum("nts,nstd->ntd", probsQ, E)
        ctx.save_for_backward(pk_flat, v_flat, probsQ, E)
        ctx.eps = float(eps)
        ctx.shape = (N, T, S, D)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        ext = _ext()
        pk_flat, v_flat, probsQ, E = ctx.saved_tensors
        N, T, S, D = ctx.shape
        grad_out = grad_out.contiguous().float()
        g_pq = torch.einsum("ntd,nstd->nts", grad_out, E).contiguous()
        gE = torch.einsum("nts,ntd->nstd", probsQ, grad_out).reshape(N * S, T, D).contiguous()
        gW, gV = ext.race_prefix_mean_flat_bw(pk_flat, v_flat, gE, ctx.eps)
        g_pk = gW.view(N, S, T).permute(0, 2, 1).reshape(N, T, S).contiguous()
        g_v = gV.view(N, S, T, D).sum(dim=1).contiguous()
        return g_pk, g_pq, g_v, None


def layer_fwd_bwd(Q, K, V, dO, planes_T, protos_T, L, P, eps=1e-6):
    """One forward+backward of the reference CPU layer (RaceCausalCuda.forward
    structure, scaling/race_causal_cuda.py:94-102, with the CPU scan swapped in
    the way scaling/bench_race_vs_softmax_cpu.py:44 does).  Returns
    (out, dQ, dK, dV) as fp32 CPU tensors."""
    q = Q.detach().float().requires_grad_(True)
    k = K.detach().float().requires_grad_(True)
    v = V.detach().float().requires_grad_(True)
    B, H, T, D = q.shape
    pk, pq, V2, N = soft_hash_probs_ref(q, k, v, planes_T, protos_T, L, P)
    out = RefRaceCausalCPUFn.apply(pk, pq, V2, eps).view(B, H, T, D)
    out.backward(dO.float())
    return out.detach(), q.grad, k.grad, v.grad
