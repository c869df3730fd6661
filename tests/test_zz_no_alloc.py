"""GPU test of bcjr_fb_forward_noalloc, the entry point for callers that
cannot allocate device memory (a host binding the C ABI without a device
allocator, or a loop that must not call cudaMalloc between steps).

It runs on a fixed scratch array inside the library instead of a caller
workspace; this checks, through the C ABI, that two calls in a row give the
same soft codewords and log Z as bcjr_fb_forward within the parity tolerance
(1e-4 relative, 1e-5 absolute) -- including batches with more sequences than
the scratch has slots, where a block takes its next sequence on the slot
its last one left behind, and the longest sequence that fits -- and that a
shape too large for the fixed scratch is refused.  Kept in its own file,
collected last."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("L,k,V,N,B,T", [(8, 2, 1, 256, 64, 1.0), (16, 2, 1, 64, 5, 0.5),
                                         (10, 2, 2, 40, 7, 0.7),
                                         # one 33.8 MB slot fits: 4 sequences on one block
                                         (16, 2, 1, 512, 4, 0.5),
                                         # the longest sequence whose slot fits at L=16, k=2, V=1
                                         (16, 2, 1, 1020, 1, 0.5)])
def test_noalloc_forward_matches_forward(cuda_ok, L, k, V, N, B, T):
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(L * 31 + N)
    cb = torch.tensor(rng.standard_normal((1 << L, V)), dtype=torch.float32, device=dev)
    w = torch.tensor(rng.standard_normal((B, N, V)), dtype=torch.float32, device=dev)
    Tt = torch.tensor(T, dtype=torch.float32, device=dev)
    P, sp = _lib.ptr, _lib.stream_ptr(dev)

    ref_soft = torch.empty_like(w)
    ref_logZ = torch.empty(B, device=dev)
    ws = _lib.workspace(B, N, L, k, V, _lib.WS_FORWARD, dev)
    _lib.check(lib.bcjr_fb_forward(P(w), P(cb), P(Tt), B, N, L, k, V, P(ref_soft), P(ref_logZ),
                                   P(ws), ws.numel(), sp), "bcjr_fb_forward")
    for _ in range(2):
        soft = torch.full_like(w, float("nan"))
        logZ = torch.full((B,), float("nan"), device=dev)
        _lib.check(lib.bcjr_fb_forward_noalloc(P(w), P(cb), P(Tt), B, N, L, k, V,
                                               P(soft), P(logZ), sp), "bcjr_fb_forward_noalloc")
        torch.cuda.synchronize()
        np.testing.assert_allclose(soft.cpu().numpy(), ref_soft.cpu().numpy(), rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(logZ.cpu().numpy(), ref_logZ.cpu().numpy(), rtol=2e-6, atol=1e-4)


@pytest.mark.parametrize("N", [1021, 4096])
def test_noalloc_rejects_shapes_beyond_the_scratch(cuda_ok, N):
    """One slot of (N + 3) 2^14 + 2N floats must fit the 64 MiB scratch:
    N = 1021 and longer are refused before any launch."""
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    w = torch.zeros((1, N, 1), device=dev)
    cb = torch.zeros((65536, 1), device=dev)
    Tt = torch.tensor(1.0, device=dev)
    soft = torch.empty_like(w)
    rc = lib.bcjr_fb_forward_noalloc(_lib.ptr(w), _lib.ptr(cb), _lib.ptr(Tt), 1, N, 16, 2, 1,
                                     _lib.ptr(soft), None, _lib.stream_ptr(dev))
    BCJR_ERR_WORKSPACE = 5
    assert rc == BCJR_ERR_WORKSPACE
