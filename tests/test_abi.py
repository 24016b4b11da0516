"""The C ABI library loads and exports every entry point include/race_b200.h
declares; host-side validation returns the documented status codes before any
CUDA call (so these run without a GPU)."""
import ctypes
import os
import re

import pytest

from race_attention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "race_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(race_\w+)\s*\(", src, flags=re.M)))


def status_codes():
    src = open(HEADER).read()
    return {k: int(v) for k, v in re.findall(r"#define (RACE_(?:OK|ERR_\w+))\s+(\d+)", src)}


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"{n} declared in race_b200.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert lib.race_abi_version() == 1


def test_status_strings():
    lib = _lib.load()
    for name, code in status_codes().items():
        s = lib.race_status_string(code).decode()
        assert s and s != "unknown status", name


def test_workspace_query_is_host_only():
    lib = _lib.load()
    nb = ctypes.c_size_t(0)
    # config-1 shape, fused forward fp32
    rc = lib.race_workspace_bytes(_lib.OP_FWD_QKV, 8, 4096, 0, 64, 8, 4, _lib.RACE_F32, 0, ctypes.byref(nb))
    assert rc == 0 and nb.value > 0
    rc = lib.race_workspace_bytes(_lib.OP_BWD_PROBS, 2, 1024, 64, 64, 0, 0, 0, 0, ctypes.byref(nb))
    assert rc == 0 and nb.value > 0
    # bad op / bad dtype
    assert lib.race_workspace_bytes(99, 1, 1, 1, 1, 1, 1, 0, 0, ctypes.byref(nb)) == status_codes()["RACE_ERR_ARG"]
    assert lib.race_workspace_bytes(_lib.OP_FWD_QKV, 1, 1, 0, 8, 1, 1, 7, 0, ctypes.byref(nb)) == \
        status_codes()["RACE_ERR_DTYPE"]


@pytest.mark.parametrize("N,T,S,D,code", [
    (0, 8, 8, 8, "RACE_ERR_SHAPE"),
    (1, 0, 8, 8, "RACE_ERR_SHAPE"),
    (1, 8, 1025, 8, "RACE_ERR_SHAPE"),
    (1, 8, 8, 257, "RACE_ERR_SHAPE"),
    (1, 8, 8, 8, "RACE_ERR_WORKSPACE"),
])
def test_fwd_probs_validation(N, T, S, D, code):
    lib = _lib.load()
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    rc = lib.race_fwd_probs(p, p, p, p, None, None, N, T, S, D, 1e-6, 0, None, 0, None)
    assert rc == status_codes()[code]
    assert lib.race_last_error().decode()


def test_null_pointer_rejected():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    rc = lib.race_fwd_probs(None, p, p, p, None, None, 1, 8, 8, 8, 1e-6, 0, None, 0, None)
    assert rc == status_codes()["RACE_ERR_ARG"]
    assert "probsK" in lib.race_last_error().decode()


def test_decode_validation():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    codes = status_codes()
    # Nq not a multiple of Nkv
    assert lib.race_decode_step(p, p, p, 0, p, p, p, p, 5, 2, 64, 8, 4, 1e-6, 0.125, None) == codes["RACE_ERR_SHAPE"]
    # P out of range
    assert lib.race_decode_step(p, p, p, 0, p, p, p, p, 4, 2, 64, 8, 11, 1e-6, 0.125, None) == codes["RACE_ERR_SHAPE"]
    # group too large
    assert lib.race_decode_step(p, p, p, 0, p, p, p, p, 64, 2, 64, 8, 4, 1e-6, 0.125, None) == \
        codes["RACE_ERR_UNSUPPORTED"]


def test_kernel_timing_host_side():
    """The timing diagnostic toggles and reports zero launches with no GPU work,
    and rejects an out-of-range kernel id."""
    import ctypes
    from race_attention_b200 import _lib
    lib = _lib.load()
    assert lib.race_kernel_timing(1) == 0
    ms, n = ctypes.c_double(-1.0), ctypes.c_longlong(-1)
    assert lib.race_kernel_time(3, ctypes.byref(ms), ctypes.byref(n)) == 0
    assert ms.value == 0.0 and n.value == 0
    assert lib.race_kernel_time(len(_lib.KERNEL_NAMES), ctypes.byref(ms), ctypes.byref(n)) != 0
    assert lib.race_kernel_timing(0) == 0


def test_bthd_layout_needs_tcgen05_path():
    """The [B,T,H,D] entry points reject configurations the tcgen05 kernels do not run
    (fp32 here) before any GPU work."""
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    codes = status_codes()
    rc = lib.race_fwd_bthd(p, p, p, _lib.RACE_F32, p, p, None, 0, 2, 128, 3, 64, 8, 4, 1e-6, 0.125, p, 1 << 20, None)
    assert rc == codes["RACE_ERR_UNSUPPORTED"]
    rc = lib.race_bwd_bthd(p, p, p, p, _lib.RACE_F32, p, None, 0, p, p, p, 2, 128, 3, 64, 8, 4, 1e-6, 0.125, p,
                           1 << 20, None)
    assert rc == codes["RACE_ERR_UNSUPPORTED"]
    assert lib.race_fwd_bthd(p, p, p, _lib.RACE_BF16, p, p, None, 0, 0, 128, 3, 64, 8, 4, 1e-6, 0.125, p, 1 << 20,
                             None) == codes["RACE_ERR_SHAPE"]


def test_gqa_decode_validation():
    """race_gqa_decode_attn rejects bad shapes before any CUDA call."""
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    codes = status_codes()
    one = ctypes.c_void_p(256)
    # head dim other than 64
    assert lib.race_gqa_decode_attn(p, p, p, p, p, one, p, p, 2, 8, 2, 100, 128, 4, 0.1, None) == \
        codes["RACE_ERR_UNSUPPORTED"]
    # Hq not a multiple of Hkv
    assert lib.race_gqa_decode_attn(p, p, p, p, p, one, p, p, 2, 6, 4, 100, 64, 4, 0.1, None) == codes["RACE_ERR_SHAPE"]
    # query group 9 (> 8) has no kernel
    assert lib.race_gqa_decode_attn(p, p, p, p, p, one, p, p, 2, 18, 2, 100, 64, 4, 0.1, None) == \
        codes["RACE_ERR_UNSUPPORTED"]
    # split count out of range, null pointer, misaligned cache
    assert lib.race_gqa_decode_attn(p, p, p, p, p, one, p, p, 2, 8, 2, 100, 64, 65, 0.1, None) == codes["RACE_ERR_SHAPE"]
    assert lib.race_gqa_decode_attn(p, p, p, None, p, one, p, p, 2, 8, 2, 100, 64, 4, 0.1, None) == codes["RACE_ERR_ARG"]
    bad = ctypes.c_void_p(264)
    assert lib.race_gqa_decode_attn(p, p, p, bad, p, one, p, p, 2, 8, 2, 100, 64, 4, 0.1, None) == \
        codes["RACE_ERR_ALIGN"]
    # workspace: fp32 partials (64 dims + max + sum) per query head and split, a ticket per kv stream, a status word
    assert lib.race_gqa_decode_workspace_bytes(2, 8, 2, 4) == 4 * 2 * 8 * 4 * 66 + 4 * 4 + 4
    assert lib.race_gqa_decode_workspace_bytes(0, 8, 2, 4) == 0


def test_ops_refuse_host_tensors():
    """The torch-level ops run only on the CUDA library: host tensors raise (no CPU
    fallback), as the reference's extension does for non-CUDA inputs."""
    import torch
    from race_attention_b200 import ops
    q = torch.zeros(2, 8, 64, dtype=torch.bfloat16)
    kv = torch.zeros(2, 2, 64, dtype=torch.bfloat16)
    cache = torch.zeros(2, 2, 16, 64, dtype=torch.bfloat16)
    length = torch.zeros(1, dtype=torch.int32)
    ws = torch.zeros(1024, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.gqa_decode_attention(q, kv, kv, cache, cache, length, ws, 1)
    planes = torch.zeros(64, 32)
    A, B = torch.zeros(2, 128), torch.zeros(2, 128, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.decode_step(q.reshape(-1, 64), kv.reshape(-1, 64), kv.reshape(-1, 64), planes, A, B, 8, 4)


def test_segment_plan_stays_within_the_workspace():
    """The tcgen05 path's segment planner never picks more segments than the workspace
    (sized for 256 SMs) holds -- also for devices with more SMs than that -- covers every
    chunk with no empty segment, and at the config-2 geometry on 148 SMs picks 23
    segments (4.97 waves instead of 3.89)."""
    lib = _lib.load()
    nseg, sc, mx = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    for N in (1, 2, 3, 8, 32, 96, 200, 1024, 5000):
        for T in (1, 127, 128, 129, 4096, 32768, 1 << 20, 12582912):
            for S in (128, 256):
                for sms in (1, 80, 132, 148, 160, 256, 320, 1024):
                    rc = lib.race_plan_segments(N, T, S, sms, ctypes.byref(nseg), ctypes.byref(sc), ctypes.byref(mx))
                    assert rc == 0
                    nch = (T + 127) // 128
                    assert 1 <= nseg.value <= mx.value, (N, T, S, sms)
                    assert sc.value >= 1 and nseg.value * sc.value >= nch > (nseg.value - 1) * sc.value
    assert lib.race_plan_segments(32, 1 << 20, 256, 148, ctypes.byref(nseg), ctypes.byref(sc), ctypes.byref(mx)) == 0
    assert (nseg.value, sc.value) == (23, 357)
    codes = status_codes()
    assert lib.race_plan_segments(32, 1 << 20, 256, 0, ctypes.byref(nseg), ctypes.byref(sc),
                                  ctypes.byref(mx)) == codes["RACE_ERR_ARG"]


def test_wait_controls_validate_on_the_host():
    """The bounded-wait controls are host-only settings; reading a status word needs a
    workspace pointer and somewhere to put the word (checked before any CUDA call)."""
    lib = _lib.load()
    codes = status_codes()
    assert lib.race_set_wait_limit(1 << 20) == 0
    assert lib.race_set_wait_limit(0) == 0
    assert lib.race_test_withhold_first_load(0) == 0
    st = ctypes.c_int(0)
    assert lib.race_read_status(None, None, ctypes.byref(st)) == codes["RACE_ERR_ARG"]
    assert lib.race_read_status(ctypes.c_void_p(256), None, None) == codes["RACE_ERR_ARG"]
