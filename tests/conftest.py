import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")
# surface any expired bounded device-side wait of the tcgen05 kernels as an error
os.environ.setdefault("RACE_B200_CHECK", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def relerr(got, ref):
    """max|got-ref| / max|ref|  (scaling/test_kernels.py:30-31)."""
    import torch
    g = got.detach().double().cpu() if isinstance(got, torch.Tensor) else torch.as_tensor(np.asarray(got, np.float64))
    r = ref.detach().double().cpu() if isinstance(ref, torch.Tensor) else torch.as_tensor(np.asarray(ref, np.float64))
    r = r.reshape(g.shape)
    if r.numel() == 0:
        return 0.0
    return float((g - r).abs().max() / (r.abs().max() + 1e-30))


def maxabs(got, ref):
    import torch
    g = got.detach().double().cpu() if isinstance(got, torch.Tensor) else torch.as_tensor(np.asarray(got, np.float64))
    r = ref.detach().double().cpu() if isinstance(ref, torch.Tensor) else torch.as_tensor(np.asarray(ref, np.float64))
    return float((g - r.reshape(g.shape)).abs().max()) if g.numel() else 0.0


def close(got, ref, tol, abs_floor=2e-5):
    """Pass on relative error or on a tight absolute floor for near-zero refs
    (the reference's criterion, scaling/test_kernels.py:38-51)."""
    re = relerr(got, ref)
    return re <= tol or maxabs(got, ref) <= abs_floor, re
