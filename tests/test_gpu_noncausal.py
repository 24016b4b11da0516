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
