"""Sequence-sharded orchestration on CPU gloo ranks (world 2 and 3).

Each rank runs race_attention_b200.sharded.race_causal_sharded on its slice,
with the oracle standing in for the CUDA kernels; the concatenated outputs and
gradients must equal the oracle's full-sequence result.  Also: a rank that
drops out makes the survivor's collective fail within the process-group
timeout (failure detection without touching a GPU)."""
import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O
from conftest import relerr
import _shard_workers as W


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_matches_full_sequence(tmp_path, world):
    mp.start_processes(W.sharded_worker, args=(world, _port(), str(tmp_path), "oracle"), nprocs=world,
                       join=True, start_method="spawn")
    Q, K, V, dO, planes = W.make_problem()
    out, _, _ = O.race_qkv_fwd(Q, K, V, planes, 2, 3)
    dQ, dK, dV, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, 2, 3)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    cat = lambda k: np.concatenate([p[k] for p in parts], axis=1)  # noqa: E731
    assert relerr(cat("out"), out) < 1e-5
    assert relerr(cat("dQ"), dQ) < 1e-4
    assert relerr(cat("dK"), dK) < 1e-4
    assert relerr(cat("dV"), dV) < 1e-4


def test_dropped_rank_fails_fast(tmp_path):
    t0 = time.time()
    ctx = mp.start_processes(W.dropped_rank_worker, args=(2, _port(), str(tmp_path), None), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(60)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    status = (tmp_path / "rank0.status").read_text()
    assert status.startswith("error:"), status
    assert time.time() - t0 < 60


def test_delayed_rank_still_exact(tmp_path):
    """A rank that arrives 3 s late (process-group timeout 60 s) delays the step but the
    result is the full-sequence result."""
    world = 3
    mp.start_processes(W.delayed_rank_worker, args=(world, _port(), str(tmp_path), 3.0), nprocs=world,
                       join=True, start_method="spawn")
    Q, K, V, dO, planes = W.make_problem()
    out, _, _ = O.race_qkv_fwd(Q, K, V, planes, 2, 3)
    dQ, dK, dV, _, _ = O.race_qkv_bwd(Q, K, V, dO, planes, 2, 3)
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    cat = lambda k: np.concatenate([p[k] for p in parts], axis=1)  # noqa: E731
    assert relerr(cat("out"), out) < 1e-5
    assert relerr(cat("dK"), dK) < 1e-4 and relerr(cat("dQ"), dQ) < 1e-4 and relerr(cat("dV"), dV) < 1e-4


def test_corrupted_exchange_is_refused(tmp_path):
    """One flipped bit in one rank's exchanged (A, B) totals is caught by the message
    checksum on every rank (ExchangeCorrupted naming rank 1) before any rank uses it."""
    world = 2
    mp.start_processes(W.corrupted_message_worker, args=(world, _port(), str(tmp_path), None), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        status = (tmp_path / f"rank{r}.status").read_text()
        assert status.startswith("corrupted:") and "[1]" in status, (r, status)
