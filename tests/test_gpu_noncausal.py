"""Non-causal RACE (the reference's BatchedACE, shared planes) on the library's kernels
against the float64 oracle and the reference module's own outputs."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from conftest import relerr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,tol,L", [(torch.float32, 1e-4, 8), (torch.bfloat16, 2e-2, 16), (torch.bfloat16, 2e-2, 8)])
def test_noncausal_layer_vs_oracle(dtype, tol, L):
    import race_attention_b200 as rb
    N, T, D, P = 6, 333, 64, 4
    g = torch.Generator().manual_seed(L)
    Q, K, V, dO = (torch.randn(N, T, D, generator=g) for _ in range(4))
    Q, K, V = (x / 8 for x in (Q, K, V))
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cpu", seed=0)
    args = [x.to(dtype).cuda().requires_grad_(True) for x in (Q, K, V)]
    out = rb.race_noncausal(*args, planes.cuda(), L, P)
    out.backward(dO.to(dtype).cuda())
    ref_in = [x.to(dtype).float() for x in (Q, K, V)]
    ref, _, _ = O.ace_fwd(*ref_in, planes, L, P)
    dQ, dK, dV = O.ace_bwd(*ref_in, dO.to(dtype).float(), planes, L, P)
    assert out.dtype == dtype
    assert relerr(out.float().cpu(), ref) < tol
    for a, r in zip(args, (dQ, dK, dV)):
        assert relerr(a.grad.float().cpu(), r) < tol


def test_batched_ace_module_vs_reference_golden():
    """The drop-in module on the reference module's own inputs and planes (golden_ace.npz):
    output and gradients of the [M, B, T, H, d_k] layout, fp32 against the reference's float64."""
    import race_attention_b200 as rb
    G = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_ace.npz"))
    for i, (B, T, H, dk, K, L, seed) in enumerate(G["cases"]):
        mod = rb.BatchedACE(int(dk), int(K), int(L), 1, device="cuda")
        mod.planes_T.copy_(torch.as_tensor(G[f"c{i}_planes_T"]).float())
        Kh, Vh, Qh = (torch.as_tensor(G[f"c{i}_{n}"]).float().cuda().requires_grad_(True) for n in ("K", "V", "Q"))
        out = mod(Kh, Vh, Qh)
        out.backward(torch.as_tensor(G[f"c{i}_dO"]).float().cuda())
        assert out.shape == Kh.shape
        assert relerr(out.detach().cpu().double(), G[f"c{i}_out"]) < 1e-4
        assert relerr(Qh.grad.cpu().double(), G[f"c{i}_dQ"]) < 1e-4
        assert relerr(Kh.grad.cpu().double(), G[f"c{i}_dK"]) < 1e-4
        assert relerr(Vh.grad.cpu().double(), G[f"c{i}_dV"]) < 1e-4


@pytest.mark.parametrize("B,H,T,L,scale", [(2, 8, 5000, 16, None), (1, 3, 129, 8, None), (1, 4, 700, 16, 1.0)])
def test_noncausal_fused_path(B, H, T, L, scale):
    """bf16, D = 64, P = 4: the layer runs as the library's fused kernels -- forward = totals
    + segment scan + one tile kernel, backward = totals + scan + two tile kernels -- with no
    [N, T, S] tensor (peak extra memory far below one fp32 probability tensor), against the
    float64 oracle at rel 2e-2.  Multi-segment streams, a partial last tile, one and two
    bucket groups, and the SFU sigmoid path (logit scale 1, the reference module's default)."""
    import race_attention_b200 as rb
    D, P = 64, 4
    N, S = B * H, L << P
    g = torch.Generator().manual_seed(T + L)
    Q, K, V, dO = (torch.randn(B, H, T, D, generator=g) for _ in range(4))
    Q, K, V = (x / 8 for x in (Q, K, V))
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cpu", seed=0)
    args = [x.to(torch.bfloat16).cuda().requires_grad_(True) for x in (Q, K, V)]
    dOc = dO.to(torch.bfloat16).cuda()
    pc = planes.cuda()
    lib = rb._lib.load()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    n0 = lib.race_launch_counter()
    out = rb.race_noncausal(*args, pc, L, P, logit_scale=scale)
    torch.cuda.synchronize()
    n1 = lib.race_launch_counter()
    out.backward(dOc)
    torch.cuda.synchronize()
    n2 = lib.race_launch_counter()
    assert (n1 - n0, n2 - n1) == (3, 4)
    peak = torch.cuda.max_memory_allocated() - base
    # what the layer needs: its workspace, four [N,T,D] bf16 results, the fp32 summaries;
    # an [N,T,S] fp32 probability tensor would add N*T*S*4 bytes on top
    import ctypes
    ws = []
    for op in (rb._lib.OP_ACE_FWD, rb._lib.OP_ACE_BWD):
        nb = ctypes.c_size_t(0)
        assert lib.race_workspace_bytes(op, N, T, 0, D, L, P, 1, 0, ctypes.byref(nb)) == 0
        ws.append(nb.value)
    budget = max(ws) + 4 * N * T * D * 2 + 2 * N * S * (D + 1) * 4 + (1 << 21)
    assert peak < budget + N * T * S * 4 // 8, (peak, budget, N * T * S * 4)
    ref_in = [x.to(torch.bfloat16).float() for x in (Q, K, V)]
    ref, _, _ = O.ace_fwd(*ref_in, planes, L, P, logit_scale=scale)
    dQ, dK, dV = O.ace_bwd(*ref_in, dO.to(torch.bfloat16).float(), planes, L, P, logit_scale=scale)
    assert relerr(out.float().cpu(), ref.reshape(out.shape)) < 2e-2
    for a, r in zip(args, (dQ, dK, dV)):
        assert relerr(a.grad.float().cpu(), r.reshape(a.shape)) < 2e-2, relerr(a.grad.float().cpu(), r.reshape(a.shape))
