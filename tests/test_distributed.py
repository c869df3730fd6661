"""Multi-process CPU tests (gloo, world size 2) of the tile sharding and
reassembly in quant_2bit_b200.distributed.  The per-shard compute is the CPU
oracle (the checker), injected through ``compute``; the product default is
the sm_100a kernels."""
import os
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_compute():
    from oracle import oracle

    def fwd(seq, cb, T, L, k, V):
        soft, _, _ = oracle.fb(seq.numpy(), cb.numpy(), float(T), L, k, V)
        return torch.tensor(soft, dtype=torch.float32)

    def bwd(seq, cb, T, soft, grad, L, k, V):
        _, _, d = oracle.fb(seq.numpy(), cb.numpy(), float(T), L, k, V, grad_soft=grad.numpy())
        return torch.tensor(d, dtype=torch.float32)

    return fwd, bwd


def _worker(rank, world, port, B, outdir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from quant_2bit_b200.distributed import sharded_bcjr, shard_range
    L, k, V, N, T = 6, 2, 1, 12, 0.7
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g)
    w = torch.randn(B, N, V, generator=g)
    gr = torch.randn(B, N, V, generator=g)
    x = w.clone().requires_grad_(True)
    soft = sharded_bcjr(x, cb, T, L, k, V, compute=_oracle_compute())
    (soft * gr).sum().backward()
    lo, hi = shard_range(B, world, rank)
    np.savez(os.path.join(outdir, f"r{rank}.npz"), soft=soft.detach().numpy(),
             grad=x.grad.numpy(), lo=lo, hi=hi)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("B", [7, 8, 1])
def test_sharded_forward_backward_matches_single_process(B):
    from oracle import oracle
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), B, d), nprocs=2, join=True,
                           start_method="spawn")
        r0 = dict(np.load(os.path.join(d, "r0.npz")))
        r1 = dict(np.load(os.path.join(d, "r1.npz")))
    L, k, V, N, T = 6, 2, 1, 12, 0.7
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g)
    w = torch.randn(B, N, V, generator=g)
    gr = torch.randn(B, N, V, generator=g)
    s, _, dd = oracle.fb(w.numpy(), cb.numpy(), T, L, k, V, grad_soft=gr.numpy())
    for r in (r0, r1):
        np.testing.assert_allclose(r["soft"], s, rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(r["grad"], dd, rtol=1e-6, atol=1e-7)
    # contiguous, balanced, covering partition
    assert int(r0["lo"]) == 0 and int(r0["hi"]) == int(r1["lo"]) and int(r1["hi"]) == B
    assert abs((int(r0["hi"]) - int(r0["lo"])) - (int(r1["hi"]) - int(r1["lo"]))) <= 1


def test_shard_range_partition():
    from quant_2bit_b200.distributed import shard_range
    for B in (0, 1, 5, 4096, 237568, 1572864):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                lo, hi = shard_range(B, world, r)
                assert 0 <= lo <= hi <= B
                covered.extend(range(lo, hi)) if B < 5000 else None
            if B < 5000:
                assert covered == list(range(B))
            sizes = [shard_range(B, world, r)[1] - shard_range(B, world, r)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def _dying_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)      # leaves between steps, before the collective
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from quant_2bit_b200.distributed import gather_rows
    try:
        gather_rows(torch.zeros(3, 4, 1), 6)
        outcome = "completed"
    except Exception as e:  # the collective must fail, not hang
        outcome = "error: " + type(e).__name__
    with open(os.path.join(outdir, "outcome.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_peer_loss_surfaces_as_error_not_hang():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_dying_worker, args=(2, _free_port(), d), nprocs=2, join=False,
                                 start_method="spawn")
        import time
        deadline = time.time() + 120
        while not ctx.join(timeout=5) and time.time() < deadline:
            pass
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
        outcome = open(os.path.join(d, "outcome.txt")).read()
    assert outcome.startswith("error"), outcome
