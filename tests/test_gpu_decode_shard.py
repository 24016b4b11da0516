"""Decode step, prefill->state handoff and sequence-shard phases vs the oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from conftest import relerr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 2)])
def test_prefill_then_decode(dtype, tol, Hq, Hkv):
    import race_attention_b200 as rb
    B, T0, steps, D, L, P = 3, 40, 6, 64, 8, 4
    g = torch.Generator().manual_seed(Hq * 10 + Hkv)
    T = T0 + steps
    Q = torch.randn(B, Hq, T, D, generator=g).to(dtype)
    K = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    V = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cpu", seed=1)
    grp = Hq // Hkv
    Ke, Ve = K.repeat_interleave(grp, 1), V.repeat_interleave(grp, 1)
    ref, _, _ = O.race_qkv_fwd(Q, Ke, Ve, planes, L, P)  # [B*Hq, T, D]
    ref = ref.reshape(B, Hq, T, D)
    out0, st = rb.prefill_with_state(Q[:, :, :T0].cuda(), K[:, :, :T0].cuda(), V[:, :, :T0].cuda(),
                                     planes.cuda(), L, P)
    assert relerr(out0, ref[:, :, :T0]) < tol
    _, Ar, Br = O.race_qkv_fwd(K[:, :, :T0], K[:, :, :T0], V[:, :, :T0], planes, L, P)
    # bf16 path: the state accumulates bf16-rounded bucket probabilities (fp32 sums)
    assert relerr(st.A, Ar) < tol and relerr(st.B, Br) < tol
    for t in range(T0, T):
        o = st.step(Q[:, :, t].cuda(), K[:, :, t].cuda(), V[:, :, t].cuda())
        assert relerr(o, ref[:, :, t]) < tol, t
    assert st.tokens == T


@pytest.mark.parametrize("L", [8, 16])
@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (12, 4), (16, 2)])
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_decode_d64_tables_and_groups(L, Hq, Hkv, dtype, tol):
    """The compile-time-shaped decode kernel (head_dim 64, 4 planes) at 8 and 16 tables and
    query groups 1, 2, 3 (a group below the kernel's width) and 8, against the oracle's rows."""
    import race_attention_b200 as rb
    B, T0, steps, D, P = 2, 24, 4, 64, 4
    g = torch.Generator().manual_seed(100 * L + 10 * Hq + Hkv)
    T = T0 + steps
    Q = torch.randn(B, Hq, T, D, generator=g).to(dtype)
    K = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    V = torch.randn(B, Hkv, T, D, generator=g).to(dtype)
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cpu", seed=2)
    grp = Hq // Hkv
    ref, _, _ = O.race_qkv_fwd(Q, K.repeat_interleave(grp, 1), V.repeat_interleave(grp, 1), planes, L, P)
    ref = ref.reshape(B, Hq, T, D)
    _, st = rb.prefill_with_state(Q[:, :, :T0].cuda(), K[:, :, :T0].cuda(), V[:, :, :T0].cuda(), planes.cuda(), L, P)
    for t in range(T0, T):
        o = st.step(Q[:, :, t].cuda(), K[:, :, t].cuda(), V[:, :, t].cuda())
        assert relerr(o, ref[:, :, t]) < tol, (t, relerr(o, ref[:, :, t]))


def test_decode_rejects_misaligned_state():
    """A state buffer that is contiguous but not 16-byte aligned (a view one float into an
    allocation) is refused on the host before anything is launched."""
    import race_attention_b200 as rb
    Nkv, S, D, L, P = 4, 128, 64, 8, 4
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cuda", seed=0)
    A = torch.zeros(Nkv * S + 1, device="cuda")[1:].view(Nkv, S)
    B = torch.zeros(Nkv, S, D, device="cuda")
    q = torch.randn(Nkv, D, device="cuda")
    assert A.is_contiguous() and A.data_ptr() % 16 != 0
    with pytest.raises(RuntimeError, match="aligned"):
        rb.ops.decode_step(q, q, q, planes, A, B, L, P)
    torch.cuda.synchronize()  # the context is still healthy


@pytest.mark.parametrize("D,Hq,Hkv,L,P", [(30, 16, 2, 4, 3), (32, 12, 2, 4, 3), (64, 10, 2, 8, 4)])
def test_decode_generic_shapes(D, Hq, Hkv, L, P):
    """Decode steps for head dims off the float4 path (D % 4 != 0) and query groups above
    4 (the wide-accumulator kernel), fp32, against the oracle's rows."""
    import race_attention_b200 as rb
    B, T0, steps = 2, 20, 5
    g = torch.Generator().manual_seed(D + Hq)
    T = T0 + steps
    Q = torch.randn(B, Hq, T, D, generator=g)
    K = torch.randn(B, Hkv, T, D, generator=g)
    V = torch.randn(B, Hkv, T, D, generator=g)
    planes = torch.randn(D, L * P, generator=g)
    grp = Hq // Hkv
    ref, _, _ = O.race_qkv_fwd(Q, K.repeat_interleave(grp, 1), V.repeat_interleave(grp, 1), planes, L, P)
    ref = ref.reshape(B, Hq, T, D)
    _, st = rb.prefill_with_state(Q[:, :, :T0].cuda(), K[:, :, :T0].cuda(), V[:, :, :T0].cuda(), planes.cuda(), L, P)
    for t in range(T0, T):
        o = st.step(Q[:, :, t].cuda(), K[:, :, t].cuda(), V[:, :, t].cuda())
        assert relerr(o, ref[:, :, t]) < 1e-5, t


def test_state_from_prefill_with_initial_state():
    import race_attention_b200 as rb
    g = torch.Generator().manual_seed(0)
    K, V = torch.randn(4, 100, 32, generator=g), torch.randn(4, 100, 32, generator=g)
    planes = torch.randn(32, 12, generator=g)
    A1, B1 = rb.ops.state_from_prefill(K[:, :60].cuda(), V[:, :60].cuda(), planes.cuda(), 4, 3)
    A2, B2 = rb.ops.state_from_prefill(K[:, 60:].cuda(), V[:, 60:].cuda(), planes.cuda(), 4, 3, None, A1, B1)
    _, Ar, Br = O.race_qkv_fwd(K, K, V, planes, 4, 3)
    assert relerr(A2, Ar) < 1e-5 and relerr(B2, Br) < 1e-5


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_sequence_shard_phases_emulated(world, dtype, tol):
    """W ranks emulated on one GPU: forward local half (totals) -> host prefix sums ->
    finishing half (readout, keeping chunk states) ; backward local half -> host
    suffix sums -> finishing half; the concatenation equals the single-run result
    (oracle)."""
    import race_attention_b200 as rb
    N, T, D, L, P = 4, 333, 64, 8, 4
    g = torch.Generator().manual_seed(world)
    Q, K, V, dO = (torch.randn(N, T, D, generator=g).to(dtype) for _ in range(4))
    planes, _ = rb.build_planes_protos(D, P, L, 1, device="cpu", seed=0)
    pc = planes.cuda()
    bounds = np.linspace(0, T, world + 1).astype(int)
    sl = [slice(bounds[r], bounds[r + 1]) for r in range(world)]
    c = lambda x, r: x[:, sl[r]].cuda().contiguous()  # noqa: E731
    tots = [rb.ops.fwd_local(c(K, r), c(V, r), pc, L, P) for r in range(world)]
    pref = []
    for r in range(world):
        A = sum((tots[i][0].double() for i in range(r)), torch.zeros_like(tots[0][0], dtype=torch.float64))
        B = sum((tots[i][1].double() for i in range(r)), torch.zeros_like(tots[0][1], dtype=torch.float64))
        pref.append((A.float(), B.float()))
    # rank 0 has no earlier shard: no prefix at all
    fw = [rb.ops.fwd_finish(tots[r][2], c(Q, r), *(pref[r] if r else (None, None)), save=True)
          for r in range(world)]
    outs = [f[0] for f in fw]
    gt = [rb.ops.bwd_local(c(Q, r), c(K, r), c(V, r), c(dO, r), pc, L, P, A0=pref[r][0], B0=pref[r][1],
                           saved=fw[r][1]) for r in range(world)]
    grads = []
    for r in range(world):
        gA = sum((gt[i][0].double() for i in range(r + 1, world)), torch.zeros_like(gt[0][0], dtype=torch.float64))
        gB = sum((gt[i][1].double() for i in range(r + 1, world)), torch.zeros_like(gt[0][1], dtype=torch.float64))
        grads.append(rb.ops.bwd_finish(gt[r][2], gA.float(), gB.float()))
    out_r, _, _ = O.race_qkv_fwd(Q, K, V, planes, L, P)
    dQ_r, dK_r, dV_r, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, L, P)
    cat = lambda xs: torch.cat([x.float().cpu() for x in xs], 1)  # noqa: E731
    assert relerr(cat(outs), out_r) < tol
    assert relerr(cat([x[0] for x in grads]), dQ_r) < tol
    assert relerr(cat([x[1] for x in grads]), dK_r) < tol
    assert relerr(cat([x[2] for x in grads]), dV_r) < tol


def test_hybrid_decode_matches_prefill():
    """The config-4 harness at toy size: after a prefill of T tokens, greedy decode steps in
    bf16 (fused RACE decode step in the odd layers, race_gqa_decode_attn over the KV cache in
    the even ones) give the next-token logits of a plain causal forward of an fp32 copy of
    the model over the T + k tokens, within the bf16 tolerance (rel 2e-2)."""
    import copy
    from race_attention_b200.hybrid import HybridConfig, HybridLlama
    torch.manual_seed(0)
    cfg = HybridConfig(vocab_size=1000, n_layer=4, hidden=256, n_head=4, n_kv_head=2, mlp_hidden=512)
    model = HybridLlama(cfg).cuda()
    model.init_weights(0.05)
    model = model.to(torch.bfloat16)
    ref = copy.deepcopy(model).float()  # the same (bf16-representable) weights, fp32 arithmetic
    g = torch.Generator(device="cuda").manual_seed(1)
    idx = torch.randint(0, cfg.vocab_size, (3, 150), device="cuda", generator=g)
    tok = model.prefill(idx, t_max=160, micro_batch=2)
    seq = torch.cat([idx, tok[:, None]], 1)
    for _ in range(4):
        logits_step = model.step_logits(tok).float()
        full = ref.logits_full(seq)
        assert relerr(logits_step, full) < 2e-2
        tok = full.argmax(-1)  # follow the fp32 model's tokens so both see the same sequence
        seq = torch.cat([seq, tok[:, None]], 1)
    assert model.n_tokens == 154 and int(model.pos.item()) == 154


def test_hybrid_graph_replay_matches_eager():
    """A decode step captured as a CUDA graph and replayed gives the eager steps' tokens,
    caches and RACE states (same kernels, same inputs)."""
    from race_attention_b200.hybrid import DecodeGraph, HybridConfig, HybridLlama
    cfg = HybridConfig(vocab_size=1000, n_layer=4, hidden=256, n_head=4, n_kv_head=2, mlp_hidden=512)
    models = []
    for _ in range(2):
        torch.manual_seed(0)
        m = HybridLlama(cfg).cuda()
        m.init_weights(0.05)
        models.append(m.to(torch.bfloat16))
    g = torch.Generator(device="cuda").manual_seed(2)
    idx = torch.randint(0, cfg.vocab_size, (2, 100), device="cuda", generator=g)
    ta = models[0].prefill(idx, t_max=110)
    tb = models[1].prefill(idx, t_max=110)
    assert torch.equal(ta, tb)
    ta, tb = models[0].step(ta), models[1].step(tb)
    dg = DecodeGraph(models[1], tb)
    for _ in range(6):
        ta = models[0].step(ta)
        tb = dg.replay()
        assert torch.equal(ta, tb)
    a, b = models
    assert a.n_tokens == b.n_tokens == 107 and int(b.pos.item()) == 107  # 100 prefill + 1 eager + 6
    for la, lb in zip(a.layers, b.layers):
        if la.race:
            assert lb.state.tokens == 107
            assert torch.allclose(la.state.B, lb.state.B, rtol=1e-6, atol=1e-6)
        else:
            assert torch.equal(la.cache[0][:, :, :107], lb.cache[0][:, :, :107])
