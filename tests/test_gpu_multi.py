"""Sequence-sharded layer over NCCL on >= 2 GPUs (one process per GPU):
each rank runs race_causal_sharded on its contiguous slice; outputs and
gradients gathered from all ranks must equal the single-GPU fused layer on the
whole sequence.  Runs with every visible GPU (NVLS off, plain NCCL transport);
skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, dtype_name, L):
    import datetime
    import torch.distributed as dist
    import race_attention_b200 as rb
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    dtype = getattr(torch, dtype_name)
    g = torch.Generator().manual_seed(11)
    N, T, D = 6, 1000 * world + 37, 64
    Q, K, V, dO = (torch.randn(N, T, D, generator=g).mul_(0.125).to(dtype) for _ in range(4))
    planes, _ = rb.build_planes_protos(D, 4, L, 1, device="cpu", seed=0)
    bounds = np.linspace(0, T, world + 1).astype(int)
    sl = slice(bounds[rank], bounds[rank + 1])
    q, k, v = (x[:, sl].cuda().contiguous().requires_grad_(True) for x in (Q, K, V))
    out = rb.race_causal_sharded(q, k, v, planes.cuda(), L, 4)
    out.backward(dO[:, sl].cuda().contiguous())
    torch.cuda.synchronize()
    np.savez(os.path.join(outdir, f"r{rank}.npz"), out=out.detach().float().cpu().numpy(),
             dQ=q.grad.float().cpu().numpy(), dK=k.grad.float().cpu().numpy(), dV=v.grad.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("dtype_name,L,tol", [("bfloat16", 16, 2e-2), ("bfloat16", 8, 2e-2), ("float32", 8, 1e-4)])
def test_sequence_sharded_nccl(tmp_path, dtype_name, L, tol):
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs >= 2 GPUs")
    # every visible GPU (up to the 8 of one box): the exchange's rank order and the
    # fixed-order prefix/suffix are only exercised at the widest world
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path), dtype_name, L), nprocs=world, join=True,
                       start_method="spawn")
    import race_attention_b200 as rb
    from conftest import relerr
    dtype = getattr(torch, dtype_name)
    g = torch.Generator().manual_seed(11)
    N, T, D = 6, 1000 * world + 37, 64
    Q, K, V, dO = (torch.randn(N, T, D, generator=g).mul_(0.125).to(dtype) for _ in range(4))
    planes, _ = rb.build_planes_protos(D, 4, L, 1, device="cpu", seed=0)
    q, k, v = (x.cuda().requires_grad_(True) for x in (Q, K, V))
    ref = rb.race_causal(q, k, v, planes.cuda(), L, 4)
    ref.backward(dO.cuda())
    parts = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    cat = lambda key: np.concatenate([p[key] for p in parts], axis=1)  # noqa: E731
    assert relerr(cat("out"), ref.float()) < tol
    assert relerr(cat("dQ"), q.grad.float()) < tol
    assert relerr(cat("dK"), k.grad.float()) < tol
    assert relerr(cat("dV"), v.grad.float()) < tol
