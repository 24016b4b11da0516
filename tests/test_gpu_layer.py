"""Fused layer (soft hash + scan + readout, forward and backward) vs the oracle
and vs the reference's own outputs (golden), fp32 and bf16."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from conftest import close, relerr

pytestmark = pytest.mark.gpu


def qkv(B, H, T, D, seed, scale=1.0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    Q, K, V, dO = (torch.randn(B, H, T, D, generator=g) for _ in range(4))
    Q, K, V = Q * scale, K * scale, V * scale
    return [x.to(dtype) for x in (Q, K, V, dO)]


def test_golden_module_cases(golden):
    """RaceCausalCuda vs the reference's RaceCumsumCausal outputs and grads
    (scaling/test_kernels.py:107-129 tolerances: out 2e-5, grads 2e-3)."""
    import race_attention_b200 as rb
    for i, c in enumerate(golden["e2e_cases"]):
        B, H, T, D, kb, L, M, share, seed = (int(x) for x in c)
        g = lambda k: torch.from_numpy(golden[f"e2e{i}_{k}"]).cuda()  # noqa: E731
        mod = rb.RaceCausalCuda(D, kb, L, M, device="cuda", share_planes=bool(share), seed=seed)
        assert torch.equal(mod.planes_T, g("planes_T"))
        q, k, v = (g(n).clone().requires_grad_(True) for n in ("Q", "K", "V"))
        out = mod(q, k, v)
        (out * g("dO")).sum().backward()
        assert close(out, g("out"), 2e-5)[0], (i, relerr(out, g("out")))
        for n, t in (("dQ", q), ("dK", k), ("dV", v)):
            assert close(t.grad, g(n), 2e-3)[0], (i, n, relerr(t.grad, g(n)))


def test_soft_hash_matches_reference(golden):
    import race_attention_b200 as rb
    for i, (B, H, T, D, kb, L, seed) in enumerate(golden["hash_cases"]):
        pT = torch.from_numpy(golden[f"hash{i}_planes_T"]).cuda()
        for X, ref in (("Q", "probsQ"), ("K", "probsK")):
            x = torch.from_numpy(golden[f"hash{i}_{X}"]).cuda()
            p = rb.ops.soft_hash(x, pT, int(L), int(kb))
            assert (p.cpu() - torch.from_numpy(golden[f"hash{i}_{ref}"])).abs().max() < 1e-6


def test_soft_hash_grad():
    import race_attention_b200 as rb
    g = torch.Generator().manual_seed(5)
    X = torch.randn(3, 40, 64, generator=g)
    planes = torch.randn(64, 32, generator=g)
    dp = torch.randn(3, 40, 128, generator=g)
    dX = rb.ops.soft_hash_bwd(X.cuda(), planes.cuda(), dp.cuda(), 8, 4)
    ref = O.soft_hash_bwd(X, planes, 8, 4, dp)
    assert relerr(dX, ref) < 1e-5


@pytest.mark.parametrize("T", [1, 2, 7, 33, 512, 4096])
def test_fp32_config1_shape(T):
    """BASELINE config 1 geometry (H=8, D=64, L=8, P=4, seed-0 planes), fp32:
    north-star tolerance rel 1e-4 on the output and all gradients."""
    import race_attention_b200 as rb
    Q, K, V, dO = qkv(1, 8, T, 64, seed=T)
    planes, _ = rb.build_planes_protos(64, 4, 8, 1, device="cpu", seed=0)
    out_r, _, _ = O.race_qkv_fwd(Q, K, V, planes, 8, 4)
    dQ_r, dK_r, dV_r, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, 8, 4)
    q, k, v = (x.cuda().requires_grad_(True) for x in (Q, K, V))
    out = rb.race_causal(q, k, v, planes.cuda(), 8, 4)
    out.backward(dO.cuda())
    assert relerr(out, out_r) < 1e-4
    # at T=1 the exact dQ is a cancellation (dprobs is constant over each table's
    # corners, which the softmax Jacobian annihilates): the reference's
    # absolute floor applies there (scaling/test_kernels.py:38-51)
    assert close(q.grad, dQ_r, 1e-4)[0], relerr(q.grad, dQ_r)
    assert close(k.grad, dK_r, 1e-4)[0], relerr(k.grad, dK_r)
    assert relerr(v.grad, dV_r) < 1e-4


@pytest.mark.parametrize("T,L,H", [(1, 16, 2), (7, 16, 2), (300, 16, 4), (2048, 16, 4), (1500, 8, 3)])
def test_bf16_vs_fp32_oracle(T, L, H):
    """BASELINE config 2 geometry (L=16 or 8, P=4, D=64, inputs N(0,1)/8) in bf16:
    north-star tolerance rel 2e-2 against the oracle on the same (bf16-rounded) inputs."""
    import race_attention_b200 as rb
    Q, K, V, dO = qkv(1, H, T, 64, seed=11 * T + L, scale=1.0 / 8.0, dtype=torch.bfloat16)
    planes, _ = rb.build_planes_protos(64, 4, L, 1, device="cpu", seed=0)
    out_r, _, _ = O.race_qkv_fwd(Q, K, V, planes, L, 4)
    dQ_r, dK_r, dV_r, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, L, 4)
    q, k, v = (x.cuda().requires_grad_(True) for x in (Q, K, V))
    out = rb.race_causal(q, k, v, planes.cuda(), L, 4)
    out.backward(dO.cuda())
    assert out.dtype == torch.bfloat16 and q.grad.dtype == torch.bfloat16
    assert relerr(out, out_r) < 2e-2
    floor = 1e-2 if T == 1 else 0.0  # T=1 dQ/dK are exact cancellations (see test_fast_backward_segments)
    assert close(q.grad, dQ_r, 2e-2, floor)[0], relerr(q.grad, dQ_r)
    assert close(k.grad, dK_r, 2e-2, floor)[0], relerr(k.grad, dK_r)
    assert relerr(v.grad, dV_r) < 2e-2


def test_fused_equals_probs_composition():
    """race_causal == soft_hash_probs + RaceCausalFn (the reference module's composition)."""
    import race_attention_b200 as rb
    Q, K, V, dO = qkv(2, 3, 200, 32, seed=2)
    planes, protos = rb.build_planes_protos(32, 3, 4, 1, device="cuda", seed=4)
    Q, K, V, dO = (x.cuda() for x in (Q, K, V, dO))
    pk, pq, V2, N = rb.soft_hash_probs(Q, K, V, planes, protos, 4, 3, 1)
    a = rb.RaceCausalFn.apply(pk, pq, V2, 1e-6).view(2, 3, 200, 32)
    b = rb.race_causal(Q, K, V, planes, 4, 3)
    assert relerr(b, a) < 1e-5


def test_carried_state_and_final_state():
    """fwd_qkv with a carried-in state == the tail of a full run; finals match the oracle."""
    import race_attention_b200 as rb
    Q, K, V, dO = qkv(1, 2, 300, 64, seed=9)
    planes, _ = rb.build_planes_protos(64, 4, 8, 1, device="cpu", seed=0)
    Qc, Kc, Vc, pc = Q.cuda(), K.cuda(), V.cuda(), planes.cuda()
    full, Af, Bf = rb.ops.fwd_qkv(Qc, Kc, Vc, pc, 8, 4, return_state=True)
    _, A1, B1 = rb.ops.fwd_qkv(Qc[:, :, :120], Kc[:, :, :120], Vc[:, :, :120], pc, 8, 4, return_state=True)
    tail = rb.ops.fwd_qkv(Qc[:, :, 120:], Kc[:, :, 120:], Vc[:, :, 120:], pc, 8, 4, A0=A1, B0=B1)
    assert relerr(tail, full.view(1, 2, 300, 64)[:, :, 120:].reshape(tail.shape)) < 1e-5
    _, Ar, Br = O.race_qkv_fwd(Q, K, V, planes, 8, 4)
    assert relerr(Af, Ar) < 1e-5 and relerr(Bf, Br) < 1e-5
    # total soft-bucket mass: every table's probabilities sum to 1 per token
    assert abs(float(Af.sum(1)[0]) - 300 * 8) < 1e-2


def test_logit_scale_argument():
    import race_attention_b200 as rb
    Q, K, V, _ = qkv(1, 2, 50, 64, seed=1)
    planes, _ = rb.build_planes_protos(64, 4, 8, 1, device="cpu", seed=0)
    out = rb.race_causal(Q.cuda(), K.cuda(), V.cuda(), planes.cuda(), 8, 4, logit_scale=1.0)
    ref, _, _ = O.race_qkv_fwd(Q, K, V, planes, 8, 4, logit_scale=1.0)
    assert relerr(out, ref) < 1e-4


@pytest.mark.parametrize("B,H,T,L", [(2, 16, 4000, 16), (4, 8, 3000, 8), (1, 2, 129, 16), (1, 3, 128, 8)])
def test_fast_forward_segments(B, H, T, L):
    """tcgen05 forward (bf16, D=64, P=4, L in {8,16}): multi-chunk segments, a
    partial last chunk, one and two bucket groups; output and final state vs the
    oracle, and the launch count proves the fused path ran (totals, segment
    scan, readout)."""
    import race_attention_b200 as rb
    Q, K, V, _ = qkv(B, H, T, 64, seed=T + L, scale=1.0 / 8.0, dtype=torch.bfloat16)
    planes, _ = rb.build_planes_protos(64, 4, L, 1, device="cpu", seed=0)
    lib = rb._lib.load()
    n0 = lib.race_launch_counter()
    out, Af, Bf = rb.ops.fwd_qkv(Q.cuda(), K.cuda(), V.cuda(), planes.cuda(), L, 4, return_state=True)
    torch.cuda.synchronize()
    assert lib.race_launch_counter() - n0 == 3
    ref, Ar, Br = O.race_qkv_fwd(Q, K, V, planes, L, 4)
    assert relerr(out, ref) < 2e-2
    # A: sums of fp32 accumulations of the (bf16) probabilities
    assert relerr(Af, Ar) < 1e-3
    assert relerr(Bf, Br) < 2e-2


@pytest.mark.parametrize("B,H,T,L", [(2, 16, 4000, 16), (4, 8, 3000, 8), (1, 2, 129, 16), (1, 3, 128, 8),
                                     (1, 2, 1, 16)])
def test_fast_backward_segments(B, H, T, L):
    """tcgen05 backward: multi-chunk segments, partial last chunk, two and four
    bucket groups; grads vs the oracle, and the launch count proves the fused
    path ran (forward totals + prefix scan, chunk states, segment-local reverse
    walk, suffix scan, suffix fix-up)."""
    import race_attention_b200 as rb
    Q, K, V, dO = qkv(B, H, T, 64, seed=3 * T + L, scale=1.0 / 8.0, dtype=torch.bfloat16)
    planes, _ = rb.build_planes_protos(64, 4, L, 1, device="cpu", seed=0)
    lib = rb._lib.load()
    n0 = lib.race_launch_counter()
    dQ, dK, dV = rb.ops.bwd_qkv(Q.cuda(), K.cuda(), V.cuda(), dO.cuda(), planes.cuda(), L, 4)
    torch.cuda.synchronize()
    assert lib.race_launch_counter() - n0 == 6
    dQ_r, dK_r, dV_r, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, L, 4)
    # T=1: the exact dK is a cancellation (dpk = -pq/pk (dO.V) + pq/pk (V.dO) = 0);
    # only an absolute floor at the bf16 resolution of the O(10) cancelling terms
    # (2^-8 relative) is meaningful there
    floor = 1e-2 if T == 1 else 0.0
    assert close(dQ, dQ_r, 2e-2, floor)[0], relerr(dQ, dQ_r)
    assert close(dK, dK_r, 2e-2, floor)[0], relerr(dK, dK_r)
    assert close(dV, dV_r, 2e-2, floor)[0], relerr(dV, dV_r)


@pytest.mark.parametrize("logit_scale,eps", [(1.0, 1e-6), (0.125, 1e-9), (2.0, 1e-10)])
def test_fast_path_general_scale_and_eps(logit_scale, eps):
    """The tcgen05 kernels take the plane sigmoids from a series only when
    2|logit_scale| <= 1/2 and batch the reciprocals of A + eps four at a time
    only when eps >= 1e-8; these cases take the SFU exponential and/or one
    reciprocal per bucket instead, forward and backward, against the oracle."""
    import race_attention_b200 as rb
    B, H, T, L = 1, 4, 700, 16
    Q, K, V, dO = qkv(B, H, T, 64, seed=17, scale=1.0 / 8.0, dtype=torch.bfloat16)
    planes, _ = rb.build_planes_protos(64, 4, L, 1, device="cpu", seed=0)
    assert rb.ops.fast_path(torch.bfloat16, 64, L, 4)
    args = (Q.cuda(), K.cuda(), V.cuda())
    out = rb.ops.fwd_qkv(*args, planes.cuda(), L, 4, eps=eps, logit_scale=logit_scale)
    dQ, dK, dV = rb.ops.bwd_qkv(*args, dO.cuda(), planes.cuda(), L, 4, eps=eps, logit_scale=logit_scale)
    ref, _, _ = O.race_qkv_fwd(Q, K, V, planes, L, 4, eps=eps, logit_scale=logit_scale)
    dQ_r, dK_r, dV_r, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, L, 4, eps=eps, logit_scale=logit_scale)
    assert relerr(out, ref) < 2e-2
    assert relerr(dQ, dQ_r) < 2e-2 and relerr(dK, dK_r) < 2e-2 and relerr(dV, dV_r) < 2e-2


@pytest.mark.parametrize("B,H,T,L", [(2, 16, 4000, 16), (1, 3, 129, 8)])
def test_saved_states_backward(B, H, T, L):
    """fwd_qkv(save=True) keeps the chunk-start states; bwd_qkv(saved=...) skips the
    two passes that rebuild them (3 launches: reverse walk, suffix scan, fix-up) and
    gives the same gradients as the rebuilding backward and the oracle."""
    import race_attention_b200 as rb
    Q, K, V, dO = qkv(B, H, T, 64, seed=5 * T + L, scale=1.0 / 8.0, dtype=torch.bfloat16)
    planes, _ = rb.build_planes_protos(64, 4, L, 1, device="cpu", seed=0)
    args = (Q.cuda(), K.cuda(), V.cuda())
    pc = planes.cuda()
    out, saved = rb.ops.fwd_qkv(*args, pc, L, 4, save=True)
    assert saved is not None and saved.numel() == rb.ops.saved_bytes(B * H, T, 64, L, 4, torch.bfloat16)
    lib = rb._lib.load()
    n0 = lib.race_launch_counter()
    g_saved = rb.ops.bwd_qkv(*args, dO.cuda(), pc, L, 4, saved=saved)
    torch.cuda.synchronize()
    assert lib.race_launch_counter() - n0 == 3
    g_full = rb.ops.bwd_qkv(*args, dO.cuda(), pc, L, 4)
    ref = O.race_qkv_bwd(Q, K, V, dO, planes, L, 4)[:3]
    for gs, gf, r in zip(g_saved, g_full, ref):
        assert relerr(gs, gf) < 2e-3
        assert relerr(gs, r) < 2e-2
    # the autograd path uses the saved states
    q, k, v = (x.clone().requires_grad_(True) for x in args)
    rb.race_causal(q, k, v, pc, L, 4).backward(dO.cuda())
    assert relerr(q.grad, g_saved[0]) < 1e-6 and relerr(k.grad, g_saved[1]) < 1e-6


@pytest.mark.parametrize("B,H,T,L", [(2, 3, 333, 8), (1, 4, 1200, 16)])
def test_bthd_layout_matches_bhtd(B, H, T, L):
    """q, k, v in the attention module's [B,T,H,D] layout (strided tensor maps, no
    transposes) give exactly the [B,H,T,D] results and gradients: same kernels, same
    segment plan, only the addressing differs."""
    import race_attention_b200 as rb
    D, P = 64, 4
    g = torch.Generator().manual_seed(B * 100 + T)
    q, k, v, do = (torch.randn(B, T, H, D, generator=g).mul_(0.125).to(torch.bfloat16).cuda() for _ in range(4))
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cpu", seed=0)
    pc = planes.cuda()
    a = [x.clone().requires_grad_(True) for x in (q, k, v)]
    y = rb.race_causal_bthd(*a, pc, L, P)
    y.backward(do)
    t = lambda x: x.transpose(1, 2).contiguous().requires_grad_(True)  # noqa: E731
    b = [t(x) for x in (q, k, v)]
    y2 = rb.race_causal(*b, pc, L, P)
    y2.backward(do.transpose(1, 2).contiguous())
    torch.cuda.synchronize()
    assert y.shape == (B, T, H, D)
    assert torch.equal(y, y2.transpose(1, 2))
    for ga, gb in zip(a, b):
        assert torch.equal(ga.grad, gb.grad.transpose(1, 2))


def test_nanochat_attention_branch():
    """nanochat's RACE branch (fp32 transposes, soft_hash_probs + RaceCausalFn, mean over
    M) against the drop-in on the same post-rotary q, k, v: fp32 goes through the
    [B,H,T,D] path (rel 1e-4), bf16 through the in-place layout (rel 2e-2)."""
    import race_attention_b200 as rb
    B, T, H, D, L, P, M = 2, 300, 2, 64, 8, 4, 2
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(B, T, H, D, generator=g) for _ in range(3))
    planes, protos = rb.build_planes_protos(D, P, L, M, device="cpu", seed=0)
    tr = lambda x: x.transpose(1, 2).contiguous()  # noqa: E731
    ref, _, _ = O.race_qkv_fwd(tr(q).reshape(B * H, T, D), tr(k).reshape(B * H, T, D), tr(v).reshape(B * H, T, D),
                               planes, L, P)
    ref = torch.as_tensor(np.asarray(ref, dtype=np.float64)).reshape(B, H, T, D).transpose(1, 2)
    y32 = rb.nanochat_race_attention(q.cuda(), k.cuda(), v.cuda(), planes.cuda(), L, P, M, 1e-6)
    assert y32.dtype == torch.float32 and relerr(y32.cpu(), ref) < 1e-4
    yb = rb.nanochat_race_attention(*(x.to(torch.bfloat16).cuda() for x in (q, k, v)), planes.cuda(), L, P, M, 1e-6)
    assert yb.dtype == torch.bfloat16 and relerr(yb.float().cpu(), ref) < 2e-2


def test_gpt_training_steps():
    """The config-5 caller harness at toy size: every layer's attention runs the in-place
    [B,T,H,D] kernels; a few AdamW steps on one fixed batch lower the loss, and all
    gradients are finite."""
    from race_attention_b200.gpt import GPTConfig, RaceGPT
    torch.manual_seed(0)
    cfg = GPTConfig(vocab_size=512, n_layer=2, n_head=2, n_embd=128, mlp_hidden=256, race_L=8)
    model = RaceGPT(cfg).cuda()
    model.init_weights(0.02)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    g = torch.Generator(device="cuda").manual_seed(1)
    idx = torch.randint(0, cfg.vocab_size, (2, 700), device="cuda", generator=g)
    tgt = torch.roll(idx, -1, 1)
    losses = []
    for _ in range(6):
        opt.zero_grad(set_to_none=True)
        loss = model(idx, tgt)
        loss.backward()
        assert all(torch.isfinite(p.grad).all() for p in model.parameters() if p.grad is not None)
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0] - 0.1, losses
