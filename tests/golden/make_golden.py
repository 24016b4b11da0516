"""Generate tests/golden/golden.npz by running the REFERENCE implementation.

Run once where the reference tree exists (it never exists on a GPU box):

    CXX=/usr/bin/g++ python tests/golden/make_golden.py --ref <path of the reference checkout>

It imports the reference's own modules from ``<ref>/scaling``:
  * build_planes_protos / soft_hash_probs / race_prefix_ref (race_common.py)
  * RaceCausalCPUFn (race_causal_cpu.py, JIT-builds kernels/cpu/race_pref.cpp)
  * RaceCumsumCausal (race_torch_cumsum.py) for end-to-end module cases
and stores inputs plus outputs as small arrays.  Scan cases follow the input
generator of scaling/test_kernels.py:54-66 (seeded torch.Generator, "softmax"
and "raw" distributions); the ground truth is race_prefix_ref in float64 with
autograd, exactly as scaling/test_kernels.py:75-81 computes it.  Inputs are
rounded to float32 before the float64 reference runs, so a float32 kernel sees
bit-identical inputs.
"""
import argparse
import os
import sys
import tempfile

import numpy as np
import torch

ap = argparse.ArgumentParser()
ap.add_argument("--ref", default=os.environ.get("RACE_REF_ROOT"),
                help="path of the reference checkout (or set RACE_REF_ROOT)")
ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz"))
args = ap.parse_args()
if not args.ref:
    ap.error("give --ref <path of the reference checkout> or set RACE_REF_ROOT")

os.environ.setdefault("TORCH_EXTENSIONS_DIR", tempfile.mkdtemp(prefix="race_golden_ext_"))
sys.path.insert(0, os.path.join(args.ref, "scaling"))
from race_common import build_planes_protos, soft_hash_probs, race_prefix_ref  # noqa: E402
from race_causal_cpu import RaceCausalCPUFn  # noqa: E402
from race_torch_cumsum import RaceCumsumCausal  # noqa: E402

G = {}

# ---- A. hash geometry (bit-exact: seeded CPU generator) ----------------------
PLANES = [  # (d_k, Kbits, L, M, share_planes, seed)
    (64, 4, 8, 1, True, 0),
    (64, 4, 16, 1, True, 0),
    (16, 2, 2, 1, True, 0),
    (24, 3, 3, 1, True, 3),
    (64, 4, 4, 1, True, 7),
    (64, 4, 8, 1, True, 1),
    (32, 3, 2, 2, False, 1),
]
G["planes_cases"] = np.array(PLANES, dtype=np.int64)
for i, (d, kb, L, M, sh, seed) in enumerate(PLANES):
    pT, prT = build_planes_protos(d, kb, L, M, device="cpu", share_planes=sh, seed=seed)
    G[f"planes{i}_planes_T"] = pT.numpy()
    G[f"planes{i}_protos_T"] = prT.numpy()

# ---- B. soft hash (fp32, the reference's own arithmetic) ---------------------
HASH = [  # (B, H, T, D, Kbits, L, seed)
    (1, 2, 24, 64, 4, 8, 0),
    (1, 2, 24, 16, 2, 2, 0),
    (2, 1, 17, 24, 3, 3, 3),
    (1, 2, 20, 64, 4, 16, 0),
]
G["hash_cases"] = np.array(HASH, dtype=np.int64)
for i, (B, H, T, D, kb, L, seed) in enumerate(HASH):
    g = torch.Generator().manual_seed(100 + i)
    Q = torch.randn(B, H, T, D, generator=g)
    K = torch.randn(B, H, T, D, generator=g)
    V = torch.randn(B, H, T, D, generator=g)
    pT, prT = build_planes_protos(D, kb, L, 1, device="cpu", seed=seed)
    pk, pq, V2, N = soft_hash_probs(Q, K, V, pT, prT, L, kb, 1, True)
    G[f"hash{i}_Q"] = Q.numpy()
    G[f"hash{i}_K"] = K.numpy()
    G[f"hash{i}_planes_T"] = pT.numpy()
    G[f"hash{i}_probsK"] = pk.numpy()
    G[f"hash{i}_probsQ"] = pq.numpy()


# ---- C. causal scan fwd/bwd, float64 ground truth ----------------------------
def make_inputs(N, T, L, R, D, seed, dist):
    # same generator as scaling/test_kernels.py:54-66
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
    r32 = lambda x: x.float().double()  # noqa: E731  float32-representable
    return r32(pk), r32(pq), r32(V), r32(go)


SCAN = [  # (N, T, L, Kbits, D, dist_id(0=softmax,1=raw), seed)
    (2, 64, 2, 2, 16, 0, 1),
    (1, 1, 3, 3, 8, 0, 2),
    (2, 2, 2, 2, 8, 0, 3),
    (2, 7, 4, 4, 16, 1, 4),
    (1, 96, 4, 4, 64, 0, 5),
    (2, 33, 3, 3, 130, 0, 6),
    (1, 48, 8, 4, 64, 0, 7),
    (1, 40, 2, 2, 24, 1, 8),
]
G["scan_cases"] = np.array(SCAN, dtype=np.int64)
eps = 1e-6
for i, (N, T, L, kb, D, dist, seed) in enumerate(SCAN):
    R = 1 << kb
    pk, pq, V, go = make_inputs(N, T, L, R, D, seed, "softmax" if dist == 0 else "raw")
    a, b, c = (x.clone().requires_grad_(True) for x in (pk, pq, V))
    out, Af, Bf = race_prefix_ref(a, b, c, eps)
    (out * go).sum().backward()
    for k, v in dict(pk=pk, pq=pq, V=V, dO=go, out=out, A_final=Af, B_final=Bf,
                     dpk=a.grad, dpq=b.grad, dV=c.grad).items():
        G[f"scan{i}_{k}"] = v.detach().numpy()

# ---- D. the reference's compiled CPU kernel (fp32) on scan case 0 ------------
pk, pq, V, go = (torch.from_numpy(G[f"scan0_{k}"]).float() for k in ("pk", "pq", "V", "dO"))
a, b, c = (x.clone().requires_grad_(True) for x in (pk, pq, V))
out = RaceCausalCPUFn.apply(a, b, c, eps)
(out * go).sum().backward()
G["refcpu_out"] = out.detach().numpy()
G["refcpu_dpk"] = a.grad.numpy()
G["refcpu_dpq"] = b.grad.numpy()
G["refcpu_dV"] = c.grad.numpy()

# ---- E. end-to-end module (soft hash + scan + ensemble mean), fp32 -----------
E2E = [  # (B, H, T, D, Kbits, L, M, share, seed)
    (1, 2, 32, 16, 2, 2, 1, 1, 0),
    (1, 2, 48, 64, 4, 4, 1, 1, 1),
    (1, 1, 40, 32, 3, 3, 2, 1, 2),
    (2, 1, 24, 16, 3, 2, 2, 0, 3),
    (1, 2, 64, 64, 4, 8, 1, 1, 0),
]
G["e2e_cases"] = np.array(E2E, dtype=np.int64)
for i, (B, H, T, D, kb, L, M, share, seed) in enumerate(E2E):
    g = torch.Generator().manual_seed(1000 + i)
    Q = torch.randn(B, H, T, D, generator=g)
    K = torch.randn(B, H, T, D, generator=g)
    V = torch.randn(B, H, T, D, generator=g)
    go = torch.randn(B, H, T, D, generator=g)
    mod = RaceCumsumCausal(D, kb, L, M, device="cpu", share_planes=bool(share), eps=eps, seed=seed)
    q, k, v = (x.clone().requires_grad_(True) for x in (Q, K, V))
    o = mod(q, k, v)
    (o * go).sum().backward()
    for kk, vv in dict(Q=Q, K=K, V=V, dO=go, out=o, dQ=q.grad, dK=k.grad, dV=v.grad,
                       planes_T=mod.planes_T).items():
        G[f"e2e{i}_{kk}"] = vv.detach().numpy()

np.savez_compressed(args.out, **G)
print(f"wrote {args.out}: {len(G)} arrays, {os.path.getsize(args.out) / 1024:.1f} KiB")
