"""Build librace_b200.so in-tree with nvcc for sm_100a.

    python -m race_attention_b200.build [--force] [--verbose]

The library links the *shared* CUDA runtime so that it sees the caller's
current device and context (torch's runtime when loaded from Python).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "librace_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the RACE CUDA library cannot be built")
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def is_stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not is_stale():
        return LIB
    cuda_home = os.path.dirname(os.path.dirname(_nvcc()))
    cmd = [
        _nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-cudart", "shared",
        "-I", INCLUDE, "-I", CSRC,
        "-Xlinker", f"-rpath,{os.path.join(cuda_home, 'lib64')}",
        "-o", LIB + ".tmp", *sorted(glob.glob(os.path.join(CSRC, "*.cu"))),
    ] + list(extra or [])
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, sep="\n")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
