"""race_gqa_decode_attn (the softmax layers of the hybrid decoder) vs an fp32 torch
reference of grouped-query softmax attention, plus the cache append and the
out-of-range length status."""
import math

import pytest
import torch

from conftest import relerr

pytestmark = pytest.mark.gpu


def _reference(q, k_cache, v_cache, n, k_new, v_new, scale):
    """fp32 softmax attention of q [B,Hq,D] over cache rows [0, n) plus the new row."""
    K = torch.cat([k_cache[:, :, :n].float(), k_new.float()[:, :, None]], 2)
    V = torch.cat([v_cache[:, :, :n].float(), v_new.float()[:, :, None]], 2)
    G = q.shape[1] // K.shape[1]
    K, V = K.repeat_interleave(G, 1), V.repeat_interleave(G, 1)
    p = (torch.einsum("bhd,bhtd->bht", q.float(), K) * scale).softmax(-1)
    return torch.einsum("bht,bhtd->bhd", p, V)


@pytest.mark.parametrize("B,Hq,Hkv,Tmax,n,splits,sharp", [
    (2, 8, 8, 64, 0, 1, 1.0),        # empty cache: the new token only
    (2, 8, 2, 300, 17, 4, 1.0),      # more splits than needed for the keys
    (3, 32, 8, 1000, 999, 7, 1.0),   # the cache's last slot
    (1, 16, 2, 5000, 4321, 64, 1.0),
    (2, 8, 1, 2048, 1500, 16, 8.0),  # peaked softmax: running-max rescaling
    (4, 32, 8, 4096, 3000, 1, 1.0),  # one split: direct write, no merge
    (2, 12, 4, 777, 500, 5, 1.0),    # group of 3
    (2, 8, 8, 40, 33, 64, 1.0),      # more splits than key blocks: empty splits
])
def test_gqa_decode_matches_fp32(B, Hq, Hkv, Tmax, n, splits, sharp):
    from race_attention_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + n)
    bf = dict(device="cuda", dtype=torch.bfloat16)
    q = (torch.randn(B, Hq, 64, device="cuda", generator=g) * sharp).to(torch.bfloat16)
    k_new = torch.randn(B, Hkv, 64, device="cuda", generator=g).to(torch.bfloat16)
    v_new = torch.randn(B, Hkv, 64, device="cuda", generator=g).to(torch.bfloat16)
    k_cache = torch.randn(B, Hkv, Tmax, 64, device="cuda", generator=g).to(**bf)
    v_cache = torch.randn(B, Hkv, Tmax, 64, device="cuda", generator=g).to(**bf)
    k0, v0 = k_cache.clone(), v_cache.clone()
    length = torch.tensor([n], dtype=torch.int32, device="cuda")
    ws = ops.gqa_decode_workspace(B, Hq, Hkv, splits, "cuda")
    out = ops.gqa_decode_attention(q, k_new, v_new, k_cache, v_cache, length, ws, splits)
    ref = _reference(q, k0, v0, n, k_new, v_new, 1.0 / math.sqrt(64))
    assert relerr(out, ref) < 1e-2
    # the new row went to position n; nothing else changed; the length is not advanced
    assert torch.equal(k_cache[:, :, n], k_new) and torch.equal(v_cache[:, :, n], v_new)
    k0[:, :, n], v0[:, :, n] = k_new, v_new
    assert torch.equal(k_cache, k0) and torch.equal(v_cache, v0)
    assert int(length.item()) == n
    # the workspace is ready for the next call as it was left: same inputs, same bits
    out2 = ops.gqa_decode_attention(q, k_new, v_new, k_cache, v_cache, length, ws, splits)
    assert torch.equal(out, out2)
    assert int(ws[-4:].view(torch.int32).item()) == 0


def test_gqa_decode_full_cache_reports_status():
    """A length with no free cache slot stores nothing and sets the workspace status word."""
    from race_attention_b200 import ops
    B, Hq, Hkv, Tmax = 2, 8, 2, 128
    q = torch.randn(B, Hq, 64, device="cuda").to(torch.bfloat16)
    kv = torch.randn(B, Hkv, 64, device="cuda").to(torch.bfloat16)
    k_cache = torch.zeros(B, Hkv, Tmax, 64, device="cuda", dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    ws = ops.gqa_decode_workspace(B, Hq, Hkv, 2, "cuda")
    length = torch.tensor([Tmax], dtype=torch.int32, device="cuda")
    ops.gqa_decode_attention(q, kv, kv, k_cache, v_cache, length, ws, 2)
    torch.cuda.synchronize()
    assert int(ws[-4:].view(torch.int32).item()) == 1
    assert int(k_cache.abs().sum().item()) == 0
