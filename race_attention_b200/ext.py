"""Mirror of the reference's compiled extension module.

The reference JIT-builds ``race_cuda`` (kernels/gpu/race_cuda_build.py:17-33)
exposing ``race_fused_fwd`` and ``race_backward`` via pybind
(kernels/gpu/race_cuda_binding.cpp:12-23).  ``load_ext()`` here returns a
module with the same two functions, backed by librace_b200.so.
"""
from __future__ import annotations

import sys

from . import _lib
from .ops import race_backward, race_fused_fwd  # noqa: F401


def load_ext(verbose=False):
    _lib.load()
    if verbose:
        print("race_b200 loaded:", _lib.library_path())
    return sys.modules[__name__]
