"""Generate tests/golden/golden_ace.npz by running the REFERENCE non-causal RACE module.

Run once where the reference tree exists (it never exists on a GPU box):

    python tests/golden/make_golden_ace.py --ref <path of the reference checkout>

It imports ``BatchedACE`` from ``<ref>/scaling/benchmark_time.py`` (shared planes; the
module's plotting import is replaced by an empty stand-in, it is not used), runs it in
float64 on seeded inputs ([M=1, B, T, H, d_k], the module's own layout) with its learnable
temperature at its initial value (scale 1), and stores inputs, the module's planes, the
output and the input gradients for a seeded upstream gradient.
"""
import argparse
import os
import sys
import types

import numpy as np
import torch

ap = argparse.ArgumentParser()
ap.add_argument("--ref", default=os.environ.get("RACE_REF_ROOT"),
                help="path of the reference checkout (or set RACE_REF_ROOT)")
ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_ace.npz"))
args = ap.parse_args()
if not args.ref:
    ap.error("give --ref <path of the reference checkout> or set RACE_REF_ROOT")

mpl = types.ModuleType("matplotlib")
mpl.pyplot = types.ModuleType("matplotlib.pyplot")
sys.modules.setdefault("matplotlib", mpl)
sys.modules.setdefault("matplotlib.pyplot", mpl.pyplot)
sys.path.insert(0, os.path.join(args.ref, "scaling"))
from benchmark_time import BatchedACE  # noqa: E402

G = {}
CASES = [  # (B, T, H, d_k, K, L, seed)
    (1, 37, 2, 64, 4, 8, 0),
    (2, 50, 1, 64, 4, 16, 1),
    (1, 29, 3, 16, 2, 3, 2),
]
G["cases"] = np.array(CASES, dtype=np.int64)
for i, (B, T, H, dk, K, L, seed) in enumerate(CASES):
    torch.manual_seed(seed)
    mod = BatchedACE(dk, K, L, 1, device="cpu", share_planes=True).double()
    g = torch.Generator().manual_seed(100 + seed)
    Kh, Vh, Qh, dO = (torch.randn(1, B, T, H, dk, generator=g, dtype=torch.float64) for _ in range(4))
    Kh.requires_grad_(True)
    Vh.requires_grad_(True)
    Qh.requires_grad_(True)
    out = mod(Kh, Vh, Qh)
    out.backward(dO)
    G[f"c{i}_planes_T"] = mod.planes_T.detach().numpy()
    for name, x in (("K", Kh), ("V", Vh), ("Q", Qh), ("dO", dO)):
        G[f"c{i}_{name}"] = x.detach().numpy()
    G[f"c{i}_out"] = out.detach().numpy()
    G[f"c{i}_dQ"] = Qh.grad.numpy()
    G[f"c{i}_dK"] = Kh.grad.numpy()
    G[f"c{i}_dV"] = Vh.grad.numpy()
np.savez_compressed(args.out, **G)
print("wrote", args.out, {k: v.shape for k, v in G.items() if k.startswith("c0_")})
