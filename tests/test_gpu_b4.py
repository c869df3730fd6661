"""GPU tests of the L=16, k=2, V=2 (b = 4) cluster kernel (bcjr_b4.cu): against
the fp64 oracle and against the generic kernel on the same inputs, over ragged
shapes (odd B leaves one cluster slot idle, B below the cluster count, the
shortest and longest N it serves, and N beyond it, which falls back), low
temperature, a HYB codebook built the way the reference's callers build it,
a misaligned codebook view (served by the generic kernels), and the bounded
waits."""
import numpy as np
import pytest
import torch

from conftest import hyb_codebook
from oracle import oracle

pytestmark = pytest.mark.gpu


def _run(w, cb, T, grad, generic=False, V=2, cb_offset=0):
    import quant_2bit_b200 as q
    from quant_2bit_b200 import _lib
    with _lib.test_option(_lib.OPT_FORCE_GENERIC, 1 if generic else 0):
        dev = torch.device("cuda")
        wd = torch.tensor(w, device=dev)
        if cb_offset:
            # a view whose data pointer is only 4-byte aligned
            flat = torch.zeros(cb.size + cb_offset, dtype=torch.float32, device=dev)
            flat[cb_offset:] = torch.tensor(cb.reshape(-1), device=dev)
            cbd = flat[cb_offset:].view(cb.shape)
            assert cbd.data_ptr() % 16 != 0
        else:
            cbd = torch.tensor(cb, device=dev)
        soft, logZ = q.bcjr_soft_forward(wd, cbd, T, 16, 2, V)
        d = q.bcjr_soft_backward(wd, cbd, T, soft, torch.tensor(grad, device=dev), 16, 2, V)
        torch.cuda.synchronize()
        return soft.cpu().numpy(), logZ.cpu().numpy(), d.cpu().numpy()


def _inputs(seed, B, N, scale=1.0):
    rng = np.random.default_rng(seed)
    cb = rng.standard_normal((65536, 2)).astype(np.float32)
    w = (scale * rng.standard_normal((B, N, 2))).astype(np.float32)
    g = rng.standard_normal((B, N, 2)).astype(np.float32)
    return cb, w, g


@pytest.mark.parametrize("B,N,T", [(1, 2, 0.5), (3, 3, 1.0), (5, 17, 0.3), (2, 128, 0.1),
                                   (77, 64, 0.5), (2, 512, 0.5), (1, 513, 0.5)])
def test_b4_kernel_vs_generic_and_oracle(cuda_ok, B, N, T):
    cb, w, g = _inputs(B * 1000 + N, B, N)
    s1, z1, d1 = _run(w, cb, T, g)
    s2, z2, d2 = _run(w, cb, T, g, generic=True)
    rows = sorted({0, B - 1})
    s64, z64, d64 = oracle.fb(w[rows], cb, T, 16, 2, 2, grad_soft=g[rows])
    for s, z, d in ((s1, z1, d1), (s2, z2, d2)):
        np.testing.assert_allclose(s[rows], s64, rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(d[rows], d64, rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(z[rows], z64, rtol=2e-6, atol=1e-4)
    np.testing.assert_allclose(s1, s2, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(d1, d2, rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(z1, z2, rtol=1e-6, atol=1e-4)


def test_b4_many_pairs_per_cluster_bitwise(cuda_ok):
    """More sequences than clusters x slots: every cluster loops over several
    pairs; results independent of batch composition (bitwise)."""
    cb, w, g = _inputs(9, 301, 24)
    s_all, z_all, d_all = _run(w, cb, 0.5, g)
    s_sub, z_sub, d_sub = _run(w[150:153], cb, 0.5, g[150:153])
    np.testing.assert_array_equal(s_all[150:153], s_sub)
    np.testing.assert_array_equal(d_all[150:153], d_sub)
    np.testing.assert_array_equal(z_all[150:153], z_sub)


@pytest.mark.parametrize("T", [0.05, 4.0])
def test_b4_temperature_extremes(cuda_ok, T):
    """T = 0.05 on random inputs: soft elementwise, gradient normwise at 1e-4
    (the reference's own parity metric); T = 4 elementwise."""
    cb, w, g = _inputs(2128, 2, 128)
    s64, z64, d64 = oracle.fb(w, cb, T, 16, 2, 2, grad_soft=g)
    s, z, d = _run(w, cb, T, g)
    np.testing.assert_allclose(s, s64, rtol=1e-4, atol=1e-5)
    if T < 0.1:
        assert np.abs(d - d64).max() / np.abs(d64).max() < 1e-4
    else:
        np.testing.assert_allclose(d, d64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(z, z64, rtol=2e-6, atol=1e-4)


def test_b4_hyb_codebook(cuda_ok):
    """The codebook the reference's QAT layers pass (HYB, from a 512 x 2 LUT):
    many repeated codewords and exact ties between states."""
    rng = np.random.default_rng(31)
    lut = rng.standard_normal((512, 2)).astype(np.float32)
    cb = hyb_codebook(lut)
    w = rng.standard_normal((3, 128, 2)).astype(np.float32)
    g = rng.standard_normal((3, 128, 2)).astype(np.float32)
    s, z, d = _run(w, cb, 0.3, g)
    s64, z64, d64 = oracle.fb(w, cb, 0.3, 16, 2, 2, grad_soft=g)
    np.testing.assert_allclose(s, s64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(d, d64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(z, z64, rtol=2e-6, atol=1e-4)


@pytest.mark.parametrize("V", [1, 2])
def test_misaligned_codebook_view_takes_generic_path(cuda_ok, V):
    """The cluster kernels load the codebook with 16-byte vectors; a codebook
    view that is only 4-byte aligned must be served (correctly) by the generic
    kernels, through the same workspace."""
    rng = np.random.default_rng(40 + V)
    cb = rng.standard_normal((65536, V)).astype(np.float32)
    w = rng.standard_normal((3, 16, V)).astype(np.float32)
    g = rng.standard_normal((3, 16, V)).astype(np.float32)
    s1, z1, d1 = _run(w, cb, 0.5, g, V=V, cb_offset=1)
    s2, z2, d2 = _run(w, cb, 0.5, g, V=V, generic=True)
    np.testing.assert_array_equal(s1, s2)
    np.testing.assert_array_equal(d1, d2)
    np.testing.assert_array_equal(z1, z2)


def test_b4_bounded_wait_timeout_is_reported_and_context_survives(cuda_ok):
    """Failure detection without a GPU fault: with the test option
    BCJR_OPT_TEST_DROP_SENDS one CTA of each cluster withholds its outputs,
    every consumer's bounded wait (~1 s) expires, the kernel records
    BCJR_ERR_TIMEOUT in the workspace status word, writes NaN outputs and
    finishes; the next normal call on the same context is correct."""
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda")
    cb_np, w_np, _ = _inputs(4, 2, 8)
    cb = torch.tensor(cb_np, device=dev)
    w = torch.tensor(w_np, device=dev)
    T = torch.tensor(0.5, device=dev)
    soft = torch.zeros_like(w)
    logZ = torch.zeros(2, device=dev)
    ws = _lib.workspace(2, 8, 16, 2, 2, _lib.WS_FORWARD, dev)
    P, sp = _lib.ptr, _lib.stream_ptr(dev)
    with _lib.test_option(_lib.OPT_TEST_DROP_SENDS, 1):
        rc = lib.bcjr_fb_forward(P(w), P(cb), P(T), 2, 8, 16, 2, 2, P(soft), P(logZ),
                                 P(ws), ws.numel(), sp)
    assert rc == 0
    assert lib.bcjr_ws_status(P(ws), sp) == _lib.BCJR_ERR_TIMEOUT
    assert torch.isnan(soft).all() and torch.isnan(logZ).all()
    s1, _, _ = _run(w_np, cb_np, 0.5, np.ones((2, 8, 2), np.float32))
    s64, _, _ = oracle.fb(w_np, cb_np, 0.5, 16, 2, 2)
    np.testing.assert_allclose(s1, s64, rtol=1e-4, atol=1e-5)
