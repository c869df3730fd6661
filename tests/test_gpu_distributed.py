"""GPU test of the sharding API's CUDA path (quant_2bit_b200.distributed) in
a one-rank NCCL process group: the layer op that bench.py times (one launch
for all of a rank's sequences, the autograd Function around it) against the
plain autograd op on each weight.  Every sequence's result is independent of
the batch it is computed in, so the comparison is bitwise.  The multi-rank
logic (splits, all-gathers, reduce-scatters) is covered on CPU ranks by
tests/test_distributed.py."""
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def nccl_group(cuda_ok):
    from quant_2bit_b200 import distributed as qd
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_port()}", rank=0,
                            world_size=1, timeout=timedelta(seconds=60),
                            pg_options=qd.nccl_options())
    yield
    dist.destroy_process_group()


def test_sharded_layer_matches_per_weight_op(nccl_group):
    import quant_2bit_b200 as q
    from quant_2bit_b200 import distributed as qd
    dev = torch.device("cuda")
    rng = np.random.default_rng(12)
    counts = [37, 160, 5]                  # three weights, sequences (tiles) each
    N, T = 64, 0.5
    cb = torch.tensor(rng.standard_normal((65536, 1)), dtype=torch.float32, device=dev)
    ws = [torch.tensor(rng.standard_normal((c, N, 1)), dtype=torch.float32, device=dev)
          for c in counts]
    gs = [torch.tensor(rng.standard_normal((c, N, 1)), dtype=torch.float32, device=dev)
          for c in counts]
    shards = qd.LayerShards(counts, 1, 0)
    x = torch.cat(ws).requires_grad_(True)
    outs = qd.sharded_bcjr_layer(x, cb, T, shards, 16, 2, 1)
    torch.autograd.backward(list(outs), gs)
    for i, (w, g) in enumerate(zip(ws, gs)):
        xi = w.clone().requires_grad_(True)
        soft, _ = q.bcjr_forward_backward(xi, cb, T, L=16, k=2, V=1)
        (soft * g).sum().backward()
        assert torch.equal(outs[i].detach(), soft.detach()), i
        assert torch.equal(x.grad[shards.local_slice(i)], xi.grad), i
    # the non-autograd pair that bench.py times gives the same numbers
    soft_local, handle = qd.layer_forward(x.detach(), shards, cb, torch.tensor(T, device=dev),
                                          16, 2, 1)
    handle.wait()
    d = qd.layer_backward(x.detach(), soft_local, torch.cat(gs), cb, torch.tensor(T, device=dev),
                          16, 2, 1)
    torch.cuda.synchronize()
    assert torch.equal(soft_local, torch.cat([o.detach() for o in outs]))
    assert torch.equal(d, x.grad)
