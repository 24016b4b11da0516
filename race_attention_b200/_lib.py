"""ctypes binding of librace_b200.so (the C ABI declared in include/race_b200.h).

There is no fallback: if the library cannot be built or loaded, every operator
raises.  The library is built in-tree on first use when its sources are newer
than the binary (nvcc must then be available).
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

RACE_OK = 0
RACE_F32 = 0
RACE_BF16 = 1
OP_FWD_PROBS, OP_BWD_PROBS, OP_FWD_QKV, OP_BWD_QKV, OP_STATE, OP_BWD_SPLIT, OP_FWD_SPLIT, OP_ACE_FWD, OP_ACE_BWD = \
    range(9)
# kernel ids of race_kernel_time (include/race_b200.h RACE_KT_*)
KERNEL_NAMES = ("fwd_totals_kernel", "fwd_readout_kernel", "bwd_rev_kernel", "chunk_scan", "bwd_fix_kernel",
                "ace_tile_kernel")

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int
_SZ = ctypes.c_size_t

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "race_abi_version": [],
    "race_status_string": [_I],
    "race_last_error": [],
    "race_launch_counter": [],
    "race_kernel_timing": [_I],
    "race_kernel_time": [_I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)],
    "race_set_wait_limit": [ctypes.c_uint],
    "race_set_status_check": [_I],
    "race_read_status": [_P, _P, ctypes.POINTER(_I)],
    "race_test_withhold_first_load": [_I],
    "race_workspace_bytes": [_I, _I64, _I64, _I64, _I64, _I64, _I64, _I, _I64, ctypes.POINTER(_SZ)],
    "race_fwd_probs": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _F, _I64, _P, _SZ, _P],
    "race_bwd_probs": [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _F, _I64, _P, _SZ, _P],
    "race_soft_hash": [_P, _I, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P],
    "race_soft_hash_bwd": [_P, _I, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P],
    "race_fwd_qkv": [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ, _P],
    "race_bwd_qkv": [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                     _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ, _P],
    "race_state_from_prefill": [_P, _P, _I, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P, _SZ, _P],
    "race_decode_step": [_P, _P, _P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F, _P],
    "race_gqa_decode_workspace_bytes": [_I64, _I64, _I64, _I],
    "race_plan_segments": [_I64, _I64, _I64, _I, _P, _P, _P],
    "race_gqa_decode_attn": [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I, _F, _P],
    "race_fwd_bthd": [_P, _P, _P, _I, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ, _P],
    "race_bwd_bthd": [_P, _P, _P, _P, _I, _P, _P, _SZ, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _F, _F, _P,
                      _SZ, _P],
    "race_fwd_local": [_P, _P, _I, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P, _SZ, _P],
    "race_fwd_finish": [_P, _P, _P, _I, _P, _P, _P, _SZ, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ,
                        _P],
    "race_fwd_probs_noalloc": [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _F, _P],
    "race_ace_fwd": [_P, _P, _P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ, _P],
    "race_ace_bwd": [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ,
                     _P],
    "race_bwd_local": [_P, _P, _P, _P, _I, _P, _P, _SZ, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _F,
                       _P, _SZ, _P],
    "race_bwd_finish": [_P, _P, _P, _P, _I, _P, _P, _SZ, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                        _I64, _F, _F, _P, _SZ, _P],
    "race_saved_bytes": [_I64, _I64, _I64, _I64, _I64, _I, ctypes.POINTER(_SZ)],
    "race_fwd_qkv_save": [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _SZ, _I64, _I64, _I64, _I64, _I64, _F, _F, _P,
                          _SZ, _P],
    "race_bwd_qkv_saved": [_P, _P, _P, _P, _I, _P, _P, _SZ, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                           _I64, _I64, _I64, _I64, _I64, _F, _F, _P, _SZ, _P],
}
_RESTYPES = {"race_status_string": ctypes.c_char_p, "race_last_error": ctypes.c_char_p,
             "race_launch_counter": ctypes.c_ulonglong, "race_gqa_decode_workspace_bytes": ctypes.c_size_t}


def library_path() -> str:
    return _build.LIB


def load():
    """Load (building first if stale) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if _build.is_stale():
            try:
                _build.build()
            except Exception as e:  # no silent fallback: surface why
                if not os.path.exists(_build.LIB):
                    raise RuntimeError(f"race_attention_b200: CUDA library unavailable ({e})") from e
        lib = ctypes.CDLL(_build.LIB)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        if os.environ.get("RACE_B200_CHECK") == "1":
            # every tcgen05-path call waits for its stream and fails with
            # RACE_ERR_TIMEOUT if a bounded device-side wait gave up
            lib.race_set_status_check(1)
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != RACE_OK:
        lib = load()
        msg = lib.race_status_string(rc).decode()
        detail = (lib.race_last_error() or b"").decode()
        raise RuntimeError(f"{what}: {msg}" + (f" ({detail})" if detail else ""))
