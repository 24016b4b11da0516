"""Worker processes for the multi-rank tests (gloo on CPU, NCCL on GPUs).

The oracle stands in for the CUDA compute on CPU ranks, so the exchange and
autograd orchestration of race_attention_b200.sharded runs for real across
processes without a GPU."""
import datetime
import os
import time
import traceback

import numpy as np
import torch
import torch.distributed as dist

from oracle import oracle as O


class OracleShardBackend:
    """Same methods as sharded.CudaShardBackend, computed by the CPU oracle."""

    @staticmethod
    def _t(x):
        return torch.from_numpy(np.ascontiguousarray(x)).float()

    def fwd_local(self, K, V, planes_T, L, P, scale):
        pk = O.soft_hash(K, planes_T, L, P, scale)
        _, A, B = O.race_fwd(pk, pk, V)
        return self._t(A), self._t(B), (K, V, planes_T, L, P, scale)

    def fwd_finish(self, handle, Q, eps, A0, B0):
        K, V, planes_T, L, P, scale = handle
        out, _, _ = O.race_qkv_fwd(Q, K, V, planes_T, L, P, eps, scale, A0, B0)
        return self._t(out), None

    def bwd_local(self, Q, K, V, dO, planes_T, L, P, eps, scale, A0, B0, saved):
        _, _, _, gA, gB = O.race_qkv_bwd(Q, K, V, dO, planes_T, L, P, eps, scale, A0, B0)
        return self._t(gA), self._t(gB), (Q, K, V, dO, planes_T, L, P, eps, scale, A0, B0)

    def bwd_finish(self, handle, gA, gB):
        dQ, dK, dV, _, _ = O.race_qkv_bwd(*handle, gA, gB)
        return self._t(dQ), self._t(dK), self._t(dV)


def make_problem(N=2, T=48, D=16, L=2, P=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    Q, K, V, dO = (torch.randn(N, T, D, generator=g) for _ in range(4))
    planes = torch.randn(D, L * P, generator=g)
    return Q, K, V, dO, planes


def sharded_worker(rank, world, port, outdir, backend_name):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from race_attention_b200.sharded import race_causal_sharded
        Q, K, V, dO, planes = make_problem()
        T = Q.shape[1]
        bounds = np.linspace(0, T, world + 1).astype(int)
        sl = slice(bounds[rank], bounds[rank + 1])
        q, k, v = (x[:, sl].clone().requires_grad_(True) for x in (Q, K, V))
        out = race_causal_sharded(q, k, v, planes, 2, 3, 1e-6, None, None, OracleShardBackend())
        out.backward(dO[:, sl])
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), out=out.detach().numpy(), dQ=q.grad.numpy(),
                 dK=k.grad.numpy(), dV=v.grad.numpy(), lo=bounds[rank], hi=bounds[rank + 1])
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise


def dropped_rank_worker(rank, world, port, outdir, _):
    """Rank 1 leaves before the exchange; rank 0 must get an error from its
    collective within the short process-group timeout instead of hanging."""
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    if rank == 1:
        os._exit(0)  # leaves between steps: nothing of ours is in flight
    from race_attention_b200.sharded import race_causal_sharded
    Q, K, V, dO, planes = make_problem()
    t0 = time.time()
    status = "no-error"
    try:
        race_causal_sharded(Q[:, :24], K[:, :24], V[:, :24], planes, 2, 3, 1e-6, None, None, OracleShardBackend())
    except Exception as e:  # gloo raises on peer loss / timeout
        status = f"error:{type(e).__name__}"
    with open(os.path.join(outdir, "rank0.status"), "w") as f:
        f.write(f"{status} {time.time() - t0:.1f}")
    os._exit(0)


def delayed_rank_worker(rank, world, port, outdir, delay_s):
    """The last rank starts its step `delay_s` late (well inside the process-group
    timeout); every rank must still finish with the exact result."""
    if rank == world - 1:
        time.sleep(delay_s)
    sharded_worker(rank, world, port, outdir, "oracle")


def corrupted_message_worker(rank, world, port, outdir, _):
    """Rank 1's outgoing forward message has one bit flipped after its checksum was
    taken (a corrupting transport); every rank must refuse the exchanged state."""
    import race_attention_b200.sharded as sh
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    if rank == 1:
        def flip(msg):
            bad = msg.clone()
            bad.view(torch.int32)[3] ^= 1 << 20
            return bad
        sh._tamper_outgoing = flip
    Q, K, V, dO, planes = make_problem()
    status = "no-error"
    try:
        sh.race_causal_sharded(Q[:, :24], K[:, :24], V[:, :24], planes, 2, 3, 1e-6, None, None,
                               OracleShardBackend())
    except sh.ExchangeCorrupted as e:
        status = f"corrupted:{e}"
    except Exception as e:  # any other failure is a test failure
        status = f"other:{type(e).__name__}:{e}"
    with open(os.path.join(outdir, f"rank{rank}.status"), "w") as f:
        f.write(status)
    dist.destroy_process_group()
