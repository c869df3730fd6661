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


L_, K_, V_, N_, T_ = 6, 2, 1, 12, 0.7


def _inputs(B, seed=0):
    g = torch.Generator().manual_seed(seed)
    cb = torch.randn(1 << L_, V_, generator=g)
    w = torch.randn(B, N_, V_, generator=g)
    return cb, w


def _upstream(B, rank):
    # a different upstream gradient on every rank (data parallelism)
    return torch.randn(B, N_, V_, generator=torch.Generator().manual_seed(100 + rank))


def _worker(rank, world, port, B, outdir, grad_reduce):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from quant_2bit_b200.distributed import sharded_bcjr, shard_range
    cb, w = _inputs(B)
    gr = _upstream(B, rank if grad_reduce else 0)
    x = w.clone().requires_grad_(True)
    soft = sharded_bcjr(x, cb, T_, L_, K_, V_, compute=_oracle_compute(), grad_reduce=grad_reduce)
    (soft * gr).sum().backward()
    lo, hi = shard_range(B, world, rank)
    np.savez(os.path.join(outdir, f"r{rank}.npz"), soft=soft.detach().numpy(),
             grad=x.grad.numpy(), lo=lo, hi=hi)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("B,grad_reduce", [(7, True), (8, True), (1, True), (7, False)])
def test_sharded_forward_backward_matches_single_process(B, grad_reduce):
    """Replicated latent weights, rank-dependent upstream gradients: every
    rank gets the full soft tensor and the gradient of the SUMMED loss, i.e.
    the single-process gradient for the sum of the ranks' upstream
    gradients (with grad_reduce=False every rank passes the same one)."""
    from oracle import oracle
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), B, d, grad_reduce), nprocs=world,
                           join=True, start_method="spawn")
        rs = [dict(np.load(os.path.join(d, f"r{r}.npz"))) for r in range(world)]
    cb, w = _inputs(B)
    gsum = sum(_upstream(B, r) for r in range(world)) if grad_reduce else _upstream(B, 0)
    s, _, dd = oracle.fb(w.numpy(), cb.numpy(), T_, L_, K_, V_, grad_soft=gsum.numpy())
    for r in rs:
        np.testing.assert_allclose(r["soft"], s, rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(r["grad"], dd, rtol=1e-6, atol=1e-6)
    # contiguous, balanced, covering partition
    assert int(rs[0]["lo"]) == 0 and int(rs[0]["hi"]) == int(rs[1]["lo"]) and int(rs[1]["hi"]) == B
    assert abs((int(rs[0]["hi"]) - int(rs[0]["lo"])) - (int(rs[1]["hi"]) - int(rs[1]["lo"]))) <= 1


COUNTS = [5, 8, 3, 1]


def _layer_worker(rank, world, port, outdir, owners, grad_reduce):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from quant_2bit_b200.distributed import LayerShards, sharded_bcjr_layer
    shards = LayerShards(COUNTS, world, rank, owners=owners)
    cb, w_all = _inputs(sum(COUNTS), seed=3)
    starts = np.cumsum([0] + COUNTS)
    local = torch.cat([w_all[starts[i] + lo: starts[i] + hi] for i, (lo, hi) in enumerate(shards.ranges)])
    x = local.clone().requires_grad_(True)
    outs = sharded_bcjr_layer(x, cb, T_, shards, L_, K_, V_, grad_reduce=grad_reduce,
                              compute=_oracle_compute())
    loss = 0
    for i, o in enumerate(outs):
        if o.shape[0]:
            gi = _upstream(sum(COUNTS), rank if grad_reduce else 0)[starts[i]: starts[i + 1]]
            if not shards.split:
                gi = gi[shards.ranges[i][0]: shards.ranges[i][1]]
            loss = loss + (o * gi).sum()
    loss.backward()
    np.savez(os.path.join(outdir, f"r{rank}.npz"), grad=x.grad.numpy(),
             ranges=np.array(shards.ranges), **{f"o{i}": o.detach().numpy() for i, o in enumerate(outs)})
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,owners,grad_reduce", [(2, None, True), (3, None, True),
                                                      (2, None, False), (2, [1, 0, 0, 1], True)])
def test_sharded_layer_matches_single_process(world, owners, grad_reduce):
    """The layer op (LayerShards): tiles of every weight split over the ranks
    (ragged counts, a weight with fewer tiles than ranks) or whole weights
    per rank.  Each split weight is all-gathered to its full soft tensor on
    every rank; each rank's gradient is the single-process gradient of its
    own tiles for the summed upstream gradient (reduce-scatter), or for the
    common one when grad_reduce is off."""
    from oracle import oracle
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_layer_worker, args=(world, _free_port(), d, owners, grad_reduce),
                           nprocs=world, join=True, start_method="spawn")
        rs = [dict(np.load(os.path.join(d, f"r{r}.npz"))) for r in range(world)]
    B = sum(COUNTS)
    cb, w = _inputs(B, seed=3)
    # with whole weights per rank every weight's loss lives on its owner only,
    # so the summed upstream gradient of a weight is its owner's
    if owners is not None:
        gsum = torch.cat([_upstream(B, owners[i])[s: e] for i, (s, e) in
                          enumerate(zip(np.cumsum([0] + COUNTS)[:-1], np.cumsum(COUNTS)))])
    elif grad_reduce:
        gsum = sum(_upstream(B, r) for r in range(world))
    else:
        gsum = _upstream(B, 0)
    s, _, dd = oracle.fb(w.numpy(), cb.numpy(), T_, L_, K_, V_, grad_soft=gsum.numpy())
    starts = np.cumsum([0] + COUNTS)
    covered = np.zeros(B, int)
    for r, rr in enumerate(rs):
        off = 0
        for i, (lo, hi) in enumerate(rr["ranges"]):
            o = rr[f"o{i}"]
            if owners is None:
                np.testing.assert_allclose(o, s[starts[i]: starts[i + 1]], rtol=1e-6, atol=1e-7)
            elif owners[i] == r:
                np.testing.assert_allclose(o, s[starts[i]: starts[i + 1]], rtol=1e-6, atol=1e-7)
            else:
                assert o.shape[0] == 0
            np.testing.assert_allclose(rr["grad"][off: off + hi - lo],
                                       dd[starts[i] + lo: starts[i] + hi], rtol=1e-6, atol=1e-6)
            covered[starts[i] + lo: starts[i] + hi] += 1
            off += hi - lo
        assert off == rr["grad"].shape[0]
    assert (covered == 1).all()


def test_layer_shards_partition():
    from quant_2bit_b200.distributed import LayerShards
    counts = [16384, 4096, 4096, 16384, 65536, 65536, 65536]
    for world in (1, 2, 4, 8):
        tot = 0
        for r in range(world):
            sh = LayerShards(counts, world, r)
            assert sh.local == sum(hi - lo for lo, hi in sh.ranges)
            assert sh.offsets[0] == 0 and sh.split == (world > 1)
            tot += sh.local
        assert tot == sum(counts)
    owners = [(i // 3) * 8 // 64 for i in range(192)]
    sizes = [LayerShards([1] * 192, 8, r, owners=owners).local for r in range(8)]
    assert sizes == [24] * 8


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
