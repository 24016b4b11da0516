"""Probability-level operator (RaceCausalFn / race_fused_fwd / race_backward) vs
the fp64 oracle -- the reference's own sweep (scaling/test_kernels.py:132-158):
(L,K) in {(2,2),(3,3),(4,4)}, N in {1,2,4}, D in {16,64,128}; T in
{1,2,7,64,256,4096,16384,65536}; odd D {96,130,256}; the unnormalised "raw"
distribution; chunk sizes 1024/4096/8192; determinism (bitwise here)."""
import pytest
import torch

from oracle import oracle as O
from conftest import close

pytestmark = pytest.mark.gpu
PARAM_SETS = [(2, 2), (3, 3), (4, 4)]


def make_inputs(N, T, L, R, D, seed, dist="softmax"):
    # scaling/test_kernels.py:54-66
    g = torch.Generator().manual_seed(seed)
    if dist == "softmax":
        lk = torch.randn(N, T, L, R, generator=g, dtype=torch.float64)
        lq = torch.randn(N, T, L, R, generator=g, dtype=torch.float64)
        pk = torch.softmax(lk, dim=-1).reshape(N, T, L * R)
        pq = torch.softmax(lq, dim=-1).reshape(N, T, L * R)
    else:
        pk = torch.rand(N, T, L * R, generator=g, dtype=torch.float64)
        pq = torch.rand(N, T, L * R, generator=g, dtype=torch.float64)
    V = torch.randn(N, T, D, generator=g, dtype=torch.float64)
    go = torch.randn(N, T, D, generator=g, dtype=torch.float64)
    return pk, pq, V, go


def run_case(N, T, L, Kb, D, seed, eps=1e-6, dist="softmax", fwd_tol=2e-5, grad_tol=3e-3):
    import race_attention_b200 as rb
    ext = rb.load_ext()
    pk, pq, V, go = make_inputs(N, T, L, 1 << Kb, D, seed, dist)
    out_t, _, _ = O.race_fwd(pk, pq, V, eps)
    dpk_t, dpq_t, dV_t, _, _ = O.race_bwd(pk, pq, V, go, eps)
    pkc, pqc, vc = (x.float().cuda().contiguous() for x in (pk, pq, V))
    fails = []
    for C in (1024, 4096, 8192):
        ok, re = close(ext.race_fused_fwd(pkc, pqc, vc, eps, C), torch.from_numpy(out_t), fwd_tol)
        if not ok:
            fails.append(f"fwd C={C} relerr={re:.2e}")
    a = ext.race_fused_fwd(pkc, pqc, vc, eps, 4096)
    b = ext.race_fused_fwd(pkc, pqc, vc, eps, 4096)
    if not torch.equal(a, b):
        fails.append("fwd not bitwise deterministic")
    x = [t.clone().requires_grad_(True) for t in (pkc, pqc, vc)]
    out = rb.RaceCausalFn.apply(*x, eps)
    (out * go.float().cuda()).sum().backward()
    for name, got, ref in (("gradProbsK", x[0].grad, dpk_t), ("gradProbsQ", x[1].grad, dpq_t),
                           ("gradV", x[2].grad, dV_t)):
        ok, re = close(got, torch.from_numpy(ref), grad_tol)
        if not ok:
            fails.append(f"{name} relerr={re:.2e}")
    assert not fails, f"N={N} T={T} L={L} K={Kb} D={D} {dist}: " + "; ".join(fails)


@pytest.mark.parametrize("L,Kb", PARAM_SETS)
@pytest.mark.parametrize("N", [1, 2, 4])
@pytest.mark.parametrize("D", [16, 64, 128])
def test_shape_sweep(L, Kb, N, D):
    run_case(N, 1024, L, Kb, D, seed=N + D)


@pytest.mark.parametrize("L,Kb", PARAM_SETS)
@pytest.mark.parametrize("T", [1, 2, 7, 64, 256, 4096, 16384, 65536])
def test_T_sweep(L, Kb, T):
    run_case(2, T, L, Kb, 64, seed=T, grad_tol=5e-3)


@pytest.mark.parametrize("L,Kb", PARAM_SETS)
@pytest.mark.parametrize("D", [96, 130, 256])
def test_odd_D(L, Kb, D):
    run_case(2, 512, L, Kb, D, seed=D)


@pytest.mark.parametrize("L,Kb", PARAM_SETS)
def test_raw_distribution(L, Kb):
    run_case(2, 1024, L, Kb, 64, seed=7, dist="raw")


def test_golden_scan_cases(golden):
    """The committed reference fp64 vectors, through the probability-level op."""
    import race_attention_b200 as rb
    for i in range(len(golden["scan_cases"])):
        g = lambda k: torch.from_numpy(golden[f"scan{i}_{k}"])  # noqa: E731
        x = [g(k).float().cuda().requires_grad_(True) for k in ("pk", "pq", "V")]
        out = rb.RaceCausalFn.apply(*x, 1e-6)
        (out * g("dO").float().cuda()).sum().backward()
        assert close(out, g("out"), 2e-5)[0], i
        for j, k in enumerate(("dpk", "dpq", "dV")):
            assert close(x[j].grad, g(k), 3e-3)[0], (i, k)


def test_final_state_matches_reference(golden):
    import race_attention_b200 as rb
    for i in range(len(golden["scan_cases"])):
        g = lambda k: torch.from_numpy(golden[f"scan{i}_{k}"]).float().cuda()  # noqa: E731
        out, Af, Bf = rb.ops.race_fused_fwd(g("pk"), g("pq"), g("V"), 1e-6, 0, return_state=True)
        assert close(Af, g("A_final"), 1e-6)[0]
        assert close(Bf, g("B_final"), 1e-5)[0]


def test_errors_are_runtime_errors():
    import race_attention_b200 as rb
    ext = rb.load_ext()
    with pytest.raises(RuntimeError, match="CUDA only"):
        ext.race_fused_fwd(torch.rand(1, 4, 8), torch.rand(1, 4, 8), torch.rand(1, 4, 8), 1e-6, 0)
    with pytest.raises(RuntimeError, match="fp32 only"):
        z = torch.rand(1, 4, 8, device="cuda", dtype=torch.float64)
        ext.race_fused_fwd(z, z, z, 1e-6, 0)
    with pytest.raises(RuntimeError, match="S must be <= 1024"):
        z = torch.rand(1, 4, 1032, device="cuda")
        ext.race_backward(z, z, torch.rand(1, 4, 8, device="cuda"), torch.rand(1, 4, 8, device="cuda"), 1e-6, 0)
