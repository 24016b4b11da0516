"""Bounded device-side waits of the tcgen05 kernels, made to run out on purpose.

The test hook race_test_withhold_first_load makes the forward kernels issue no
tile load for their first chunk, so the mbarrier those loads would complete is
a flag that nothing sets: the first wait on it gives up after the poll limit
(race_set_wait_limit), with no TMA copy and no MMA in flight.  The call must
report it (RACE_ERR_TIMEOUT through race_set_status_check, or the status word
through race_read_status), and the next ordinary call on the same stream must
be correct, i.e. the context stays usable.  Nothing here faults, traps or hangs
a GPU: every wait is bounded and the expired one guards nothing."""
import ctypes

import pytest
import torch

from oracle import oracle as O
from conftest import relerr

pytestmark = pytest.mark.gpu

SHORT_WAIT = 1 << 14  # polls: well under a millisecond


def _inputs(T=300, H=2, L=8, seed=3):
    import race_attention_b200 as rb
    g = torch.Generator().manual_seed(seed)
    Q, K, V = (torch.randn(1, H, T, 64, generator=g).mul_(0.125).to(torch.bfloat16) for _ in range(3))
    planes, _ = rb.build_planes_protos(64, 4, L, 1, device="cpu", seed=0)
    return Q, K, V, planes


def _withheld(lib, on):
    assert lib.race_test_withhold_first_load(1 if on else 0) == 0
    assert lib.race_set_wait_limit(SHORT_WAIT if on else 0) == 0


def test_expired_wait_raises_timeout_then_next_call_is_correct():
    import race_attention_b200 as rb
    lib = rb._lib.load()
    Q, K, V, planes = _inputs()
    args = (Q.cuda(), K.cuda(), V.cuda(), planes.cuda(), 8, 4)
    assert lib.race_set_status_check(1) == 0
    _withheld(lib, True)
    try:
        with pytest.raises(RuntimeError, match="timed out"):
            rb.ops.fwd_qkv(*args)
    finally:
        _withheld(lib, False)
    out = rb.ops.fwd_qkv(*args)
    torch.cuda.synchronize()
    ref, _, _ = O.race_qkv_fwd(Q, K, V, planes, 8, 4)
    assert relerr(out, ref) < 2e-2


def test_status_word_through_the_c_abi():
    """A C-ABI caller that does not ask for synchronous checking reads the status
    word itself: non-zero after the withheld call, zero after the next one."""
    import race_attention_b200 as rb
    lib = rb._lib.load()
    Q, K, V, planes = _inputs(T=700, H=3, L=16, seed=5)
    Qc, Kc, Vc, pc = (x.cuda().contiguous() for x in (Q, K, V, planes))
    N, T, D, L, P = 3, 700, 64, 16, 4
    nb = ctypes.c_size_t(0)
    assert lib.race_workspace_bytes(2, N, T, 0, D, L, P, 1, 0, ctypes.byref(nb)) == 0
    ws = torch.zeros(nb.value, dtype=torch.uint8, device="cuda")
    out = torch.empty_like(Qc)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def call():
        return lib.race_fwd_qkv(p(Qc), p(Kc), p(Vc), 1, p(pc), p(out), None, None, None, None,
                                N, T, D, L, P, 1e-6, 0.125, p(ws), nb.value, stream)

    st = ctypes.c_int(-1)
    assert lib.race_set_status_check(0) == 0
    try:
        _withheld(lib, True)
        try:
            assert call() == 0  # launched; the failure is on the device
        finally:
            _withheld(lib, False)
        assert lib.race_read_status(p(ws), stream, ctypes.byref(st)) == 0
        assert st.value != 0
        assert call() == 0
        assert lib.race_read_status(p(ws), stream, ctypes.byref(st)) == 0
        assert st.value == 0
    finally:
        lib.race_set_status_check(1)
    ref, _, _ = O.race_qkv_fwd(Q, K, V, planes, L, P)
    assert relerr(out, ref) < 2e-2
