"""Pin the CPU oracle to the reference: every golden vector in tests/golden/golden.npz
was produced by running the reference's own code (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from conftest import relerr


def test_soft_hash_matches_reference(golden):
    for i, (B, H, T, D, kb, L, seed) in enumerate(golden["hash_cases"]):
        pT = golden[f"hash{i}_planes_T"]
        pk = O.soft_hash(golden[f"hash{i}_K"], pT, int(L), int(kb))
        pq = O.soft_hash(golden[f"hash{i}_Q"], pT, int(L), int(kb))
        # reference computes in fp32; the oracle in fp64
        assert np.abs(pk - golden[f"hash{i}_probsK"].reshape(pk.shape)).max() < 2e-7
        assert np.abs(pq - golden[f"hash{i}_probsQ"].reshape(pq.shape)).max() < 2e-7


@pytest.mark.parametrize("i", range(8))
def test_scan_fwd_bwd_matches_reference_fp64(golden, i):
    g = lambda k: golden[f"scan{i}_{k}"]  # noqa: E731
    out, Af, Bf = O.race_fwd(g("pk"), g("pq"), g("V"))
    assert relerr(out, g("out")) < 1e-12
    assert relerr(Af, g("A_final")) < 1e-12
    assert relerr(Bf, g("B_final")) < 1e-12
    dpk, dpq, dV, _, _ = O.race_bwd(g("pk"), g("pq"), g("V"), g("dO"))
    # T=1 gradProbsK is an exact cancellation (gA + V.gB): compare on an absolute floor
    assert relerr(dpk, g("dpk")) < 1e-10 or np.abs(dpk - g("dpk")).max() < 1e-12
    assert relerr(dpq, g("dpq")) < 1e-12
    assert relerr(dV, g("dV")) < 1e-12


def test_reference_cpu_kernel_matches_oracle(golden):
    """The reference's compiled OpenMP kernel (fp32) agrees with the oracle at its own tolerances."""
    g = lambda k: golden[f"scan0_{k}"]  # noqa: E731
    out, _, _ = O.race_fwd(g("pk"), g("pq"), g("V"))
    dpk, dpq, dV, _, _ = O.race_bwd(g("pk"), g("pq"), g("V"), g("dO"))
    assert relerr(golden["refcpu_out"], out) < 1e-4
    assert relerr(golden["refcpu_dpk"], dpk) < 1e-3
    assert relerr(golden["refcpu_dpq"], dpq) < 1e-3
    assert relerr(golden["refcpu_dV"], dV) < 1e-3


@pytest.mark.parametrize("i", range(5))
def test_full_layer_matches_reference_module(golden, i):
    """Soft hash + scan + ensemble mean vs the reference's RaceCumsumCausal (fp32)."""
    B, H, T, D, kb, L, M, share, seed = (int(x) for x in golden["e2e_cases"][i])
    g = lambda k: golden[f"e2e{i}_{k}"]  # noqa: E731
    pl = g("planes_T")
    planes = [pl] * M if share else [pl[m] for m in range(M)]
    outs, grads = [], []
    for pm in planes:
        outs.append(O.race_qkv_fwd(g("Q"), g("K"), g("V"), pm, L, kb)[0])
        grads.append(O.race_qkv_bwd(g("Q"), g("K"), g("V"), g("dO") / M, pm, L, kb)[:3])
    out = sum(outs) / M
    dQ, dK, dV = (sum(x[j] for x in grads) for j in range(3))
    assert relerr(out, g("out")) < 2e-5
    assert relerr(dQ, g("dQ")) < 2e-3
    assert relerr(dK, g("dK")) < 2e-3
    assert relerr(dV, g("dV")) < 2e-3


def test_state_carry_equals_full_sequence(golden):
    """Splitting the sequence with a carried state reproduces the full scan (decode / shard oracle)."""
    g = lambda k: golden[f"scan4_{k}"]  # noqa: E731
    pk, pq, V, dO = g("pk"), g("pq"), g("V"), g("dO")
    full, Af, Bf = O.race_fwd(pk, pq, V)
    c = 37
    o1, A1, B1 = O.race_fwd(pk[:, :c], pq[:, :c], V[:, :c])
    o2, A2, B2 = O.race_fwd(pk[:, c:], pq[:, c:], V[:, c:], A0=A1, B0=B1)
    assert relerr(np.concatenate([o1, o2], 1), full) < 1e-13
    assert relerr(A2, Af) < 1e-13 and relerr(B2, Bf) < 1e-13
    # backward across the split: later half's dA0/dB0 is the earlier half's incoming gradient
    dpk_f, dpq_f, dV_f, _, _ = O.race_bwd(pk, pq, V, dO)
    dpk2, dpq2, dV2, gA, gB = O.race_bwd(pk[:, c:], pq[:, c:], V[:, c:], dO[:, c:], A0=A1, B0=B1)
    dpk1, dpq1, dV1, _, _ = O.race_bwd(pk[:, :c], pq[:, :c], V[:, :c], dO[:, :c], gA=gA, gB=gB)
    assert relerr(np.concatenate([dpk1, dpk2], 1), dpk_f) < 1e-12
    assert relerr(np.concatenate([dpq1, dpq2], 1), dpq_f) < 1e-12
    assert relerr(np.concatenate([dV1, dV2], 1), dV_f) < 1e-12


def test_oracle_soft_hash_grad_matches_autograd():
    """oracle_soft_hash_bwd vs torch autograd of the reference's soft-hash formula (fp64)."""
    import itertools
    g = torch.Generator().manual_seed(3)
    X = torch.randn(2, 9, 16, generator=g, dtype=torch.float64, requires_grad=True)
    L, P = 3, 3
    planes = torch.randn(16, L * P, generator=g, dtype=torch.float64)
    protos = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=P)), dtype=torch.float64).T
    proj = (X @ planes).view(2, 9, L, P)
    probs = torch.softmax((proj.tanh() / 4.0) @ protos, -1).reshape(2, 9, -1)
    gp = torch.randn(probs.shape, generator=g, dtype=torch.float64)
    (probs * gp).sum().backward()
    dX = O.soft_hash_bwd(X.detach(), planes, L, P, gp, 0.25)
    assert relerr(dX, X.grad) < 1e-12
    assert relerr(O.soft_hash(X.detach(), planes, L, P, 0.25), probs.detach()) < 1e-13


def _ace_streams(x):
    """[1, B, T, H, d] (BatchedACE layout) -> [B*H, T, d] streams."""
    x = np.asarray(x)[0]
    B, T, H, d = x.shape
    return np.ascontiguousarray(x.transpose(0, 2, 1, 3).reshape(B * H, T, d))


def test_oracle_noncausal_matches_reference_module():
    """ace_fwd / ace_bwd against the reference's own BatchedACE (shared planes, float64,
    tests/golden/make_golden_ace.py): output and all three input gradients."""
    import os
    G = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_ace.npz"))
    for i, (B, T, H, dk, K, L, seed) in enumerate(G["cases"]):
        planes = G[f"c{i}_planes_T"]
        Q, Kx, V, dO = (_ace_streams(G[f"c{i}_{n}"]) for n in ("Q", "K", "V", "dO"))
        out, _, _ = O.ace_fwd(Q, Kx, V, planes, int(L), int(K), 1e-6, 1.0)
        assert O.relerr(out, _ace_streams(G[f"c{i}_out"])) < 1e-10
        dQ, dK, dV = O.ace_bwd(Q, Kx, V, dO, planes, int(L), int(K), 1e-6, 1.0)
        assert O.relerr(dQ, _ace_streams(G[f"c{i}_dQ"])) < 1e-9
        assert O.relerr(dK, _ace_streams(G[f"c{i}_dK"])) < 1e-9
        assert O.relerr(dV, _ace_streams(G[f"c{i}_dV"])) < 1e-10


def test_build_planes_protos_bit_identical_to_reference(golden):
    """race_attention_b200.build_planes_protos makes the reference's seeded CPU-generator
    calls (scaling/race_common.py:14-33): planes_T and protos_T are bit-identical to the
    reference's for every golden geometry, including the config-2 geometry (64, 4, 16),
    per-member planes (share_planes=False) and non-zero seeds."""
    import race_attention_b200 as rb
    cases = golden["planes_cases"]
    assert len(cases) == 7
    for i, (d, kb, L, M, share, seed) in enumerate(cases):
        pT, prT = rb.build_planes_protos(int(d), int(kb), int(L), int(M), device="cpu",
                                         share_planes=bool(share), seed=int(seed))
        want_p, want_c = golden[f"planes{i}_planes_T"], golden[f"planes{i}_protos_T"]
        assert pT.dtype == torch.float32 and tuple(pT.shape) == want_p.shape, i
        assert np.array_equal(pT.numpy(), want_p), i
        assert np.array_equal(prT.numpy(), want_c), i


def test_long_sequence_oracle_matches_the_serial_oracle():
    """oracle.layer_long (multithreaded, one stream at a time, float storage of its
    [T,S] intermediates) agrees with the serial fp64 oracle it restates."""
    import race_attention_b200 as rb
    g = torch.Generator().manual_seed(0)
    for N, T, L, D in ((2, 300, 8, 64), (1, 129, 16, 64), (3, 50, 4, 32)):
        Q, K, V, dO = (torch.randn(N, T, D, generator=g) * 0.3 for _ in range(4))
        planes, _ = rb.build_planes_protos(D, 4, L, 1, device="cpu", seed=1)
        want = list(O.race_qkv_fwd(Q, K, V, planes, L, 4)) + list(O.race_qkv_bwd(Q, K, V, dO, planes, L, 4)[:3])
        got = O.layer_long(Q, K, V, planes, L, 4, dO=dO)
        for a, b in zip(got, want):
            assert relerr(a, b) < 1e-6
