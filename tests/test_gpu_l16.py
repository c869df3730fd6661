"""GPU tests of the L=16, k=2, V=1 cluster kernel (bcjr_l16.cu): against the
fp64 oracle and against the generic kernel on the same inputs, over ragged
shapes (odd B leaves one cluster slot idle, B below the cluster count, the
shortest and longest N it serves, and N beyond it, which falls back)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


def _run(w, cb, T, grad, generic=False):
    import quant_2bit_b200 as q
    from quant_2bit_b200 import _lib
    with _lib.test_option(_lib.OPT_FORCE_GENERIC, 1 if generic else 0):
        dev = torch.device("cuda")
        wd = torch.tensor(w, device=dev)
        cbd = torch.tensor(cb, device=dev)
        soft, logZ = q.bcjr_soft_forward(wd, cbd, T, 16, 2, 1)
        d = q.bcjr_soft_backward(wd, cbd, T, soft, torch.tensor(grad, device=dev), 16, 2, 1)
        torch.cuda.synchronize()
        return soft.cpu().numpy(), logZ.cpu().numpy(), d.cpu().numpy()


@pytest.mark.parametrize("B,N,T", [(1, 2, 0.5), (3, 3, 1.0), (5, 17, 0.3), (2, 256, 0.1),
                                   (77, 64, 0.5), (2, 512, 0.5), (90, 512, 0.5), (1, 513, 0.5)])
def test_cluster_kernel_vs_generic_and_oracle(cuda_ok, B, N, T):
    rng = np.random.default_rng(B * 1000 + N)
    cb = rng.standard_normal((65536, 1)).astype(np.float32)
    w = rng.standard_normal((B, N, 1)).astype(np.float32)
    g = rng.standard_normal((B, N, 1)).astype(np.float32)
    s1, z1, d1 = _run(w, cb, T, g)
    s2, z2, d2 = _run(w, cb, T, g, generic=True)
    rows = sorted({0, B - 1})
    s64, z64, d64 = oracle.fb(w[rows], cb, T, 16, 2, 1, grad_soft=g[rows])
    for s, z, d in ((s1, z1, d1), (s2, z2, d2)):
        np.testing.assert_allclose(s[rows], s64, rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(d[rows], d64, rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(z[rows], z64, rtol=2e-6, atol=1e-4)
    # the two kernels round differently; both sit within the tolerance of fp64
    np.testing.assert_allclose(s1, s2, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(d1, d2, rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(z1, z2, rtol=1e-6, atol=1e-4)


def test_cluster_kernel_many_pairs_per_cluster(cuda_ok):
    """More sequences than clusters x slots: every cluster loops over several
    pairs; results independent of batch composition (bitwise)."""
    rng = np.random.default_rng(9)
    cb = rng.standard_normal((65536, 1)).astype(np.float32)
    B = 301
    w = rng.standard_normal((B, 24, 1)).astype(np.float32)
    g = rng.standard_normal((B, 24, 1)).astype(np.float32)
    s_all, z_all, d_all = _run(w, cb, 0.5, g)
    s_sub, z_sub, d_sub = _run(w[150:153], cb, 0.5, g[150:153])
    np.testing.assert_array_equal(s_all[150:153], s_sub)
    np.testing.assert_array_equal(d_all[150:153], d_sub)
    np.testing.assert_array_equal(z_all[150:153], z_sub)


def _run_clusters(size, w, cb, T, g):
    """Forward and backward with the cluster size of both calls forced to
    `size` (2 or 4; 0 = the automatic choice)."""
    from quant_2bit_b200 import _lib
    with _lib.test_option(_lib.OPT_L16_FORWARD_CLUSTER, size), \
            _lib.test_option(_lib.OPT_L16_BACKWARD_CLUSTER, size):
        return _run(w, cb, T, g)


@pytest.mark.parametrize("B,N", [(301, 24), (160, 256), (75, 2), (80, 512)])
def test_cluster_instances_agree_bitwise(cuda_ok, B, N):
    """The 2-CTA and 4-CTA instances reduce per (1024-butterfly block, warp) in
    one fixed order, so a sequence's soft codewords, log Z and gradient are
    bitwise the same whichever instance runs it: forward on either instance,
    backward on either alone and on both side by side (the default above one
    round of the 2-CTA grid), where sequences go to whichever grid claims
    them first."""
    rng = np.random.default_rng(B * 1000 + N)
    cb = rng.standard_normal((65536, 1)).astype(np.float32)
    w = rng.standard_normal((B, N, 1)).astype(np.float32)
    g = rng.standard_normal((B, N, 1)).astype(np.float32)
    s2, z2, d2 = _run_clusters(2, w, cb, 0.5, g)
    s4, z4, d4 = _run_clusters(4, w, cb, 0.5, g)
    sd, zd, dd = _run_clusters(0, w, cb, 0.5, g)
    np.testing.assert_array_equal(s2, s4)
    np.testing.assert_array_equal(z2, z4)
    np.testing.assert_array_equal(d2, d4)
    np.testing.assert_array_equal(s2, sd)
    np.testing.assert_array_equal(d2, dd)
    s64, z64, d64 = oracle.fb(w[:4], cb, 0.5, 16, 2, 1, grad_soft=g[:4])
    np.testing.assert_allclose(s2[:4], s64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(d2[:4], d64, rtol=1e-4, atol=1e-5)


def test_low_temperature_normwise(cuda_ok):
    """T = 0.05 on random inputs.  Here the fp32 floor of the algorithm is at
    the elementwise tolerance (an fp32 emulation of these recursions reaches
    0.93x of 1e-4/1e-5 on its worst element, dominated by the fp32 storage of
    the log-domain group messages), while the reference's own fp32 result is
    ~1e-2 from fp64.  Checked: soft elementwise, gradient normwise at 1e-4
    (the reference's own parity metric, max|err| / max|ref|)."""
    rng = np.random.default_rng(2256)
    cb = rng.standard_normal((65536, 1)).astype(np.float32)
    w = rng.standard_normal((2, 256, 1)).astype(np.float32)
    g = rng.standard_normal((2, 256, 1)).astype(np.float32)
    s64, z64, d64 = oracle.fb(w, cb, 0.05, 16, 2, 1, grad_soft=g)
    for generic in (False, True):
        s, z, d = _run(w, cb, 0.05, g, generic=generic)
        np.testing.assert_allclose(s, s64, rtol=1e-4, atol=1e-5)
        assert np.abs(d - d64).max() / np.abs(d64).max() < 1e-4
        np.testing.assert_allclose(z, z64, rtol=2e-6)


def test_bounded_wait_timeout_is_reported_and_context_survives(cuda_ok):
    """Failure detection without a GPU fault: with the test option
    BCJR_OPT_TEST_DROP_SENDS one CTA of each cluster withholds its outputs,
    every consumer's bounded wait (~1 s) expires, the kernel records
    BCJR_ERR_TIMEOUT in the workspace status word, writes NaN outputs and
    finishes; the host reads the status, and the next normal call on the
    same context is correct."""
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda")
    rng = np.random.default_rng(4)
    cb = torch.tensor(rng.standard_normal((65536, 1)), dtype=torch.float32, device=dev)
    w = torch.tensor(rng.standard_normal((2, 8, 1)), dtype=torch.float32, device=dev)
    T = torch.tensor(0.5, device=dev)
    soft = torch.zeros_like(w)
    logZ = torch.zeros(2, device=dev)
    ws = _lib.workspace(2, 8, 16, 2, 1, _lib.WS_FORWARD, dev)
    P, sp = _lib.ptr, _lib.stream_ptr(dev)
    with _lib.test_option(_lib.OPT_TEST_DROP_SENDS, 1):
        rc = lib.bcjr_fb_forward(P(w), P(cb), P(T), 2, 8, 16, 2, 1, P(soft), P(logZ),
                                 P(ws), ws.numel(), sp)
    assert rc == 0
    assert lib.bcjr_ws_status(P(ws), sp) == _lib.BCJR_ERR_TIMEOUT
    # the failure reaches the numbers: every output of the failed call is NaN
    assert torch.isnan(soft).all() and torch.isnan(logZ).all()
    s1, _, _ = _run(w.cpu().numpy(), cb.cpu().numpy(), 0.5, np.ones((2, 8, 1), np.float32))
    s64, _, _ = oracle.fb(w.cpu().numpy(), cb.cpu().numpy(), 0.5, 16, 2, 1)
    np.testing.assert_allclose(s1, s64, rtol=1e-4, atol=1e-5)


def test_bounded_wait_timeout_with_two_grids(cuda_ok):
    """The same in the backward when the 4-CTA and 2-CTA grids run side by
    side (B above one round of the 2-CTA grid): both grids stop at the
    timeout, the status is reported, the context stays usable."""
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda")
    rng = np.random.default_rng(5)
    B, N = 160, 8
    cb = torch.tensor(rng.standard_normal((65536, 1)), dtype=torch.float32, device=dev)
    w = torch.tensor(rng.standard_normal((B, N, 1)), dtype=torch.float32, device=dev)
    T = torch.tensor(0.5, device=dev)
    soft = torch.rand_like(w)
    g = torch.ones_like(w)
    d = torch.zeros_like(w)
    ws = _lib.workspace(B, N, 16, 2, 1, _lib.WS_BACKWARD, dev)
    P, sp = _lib.ptr, _lib.stream_ptr(dev)
    with _lib.test_option(_lib.OPT_TEST_DROP_SENDS, 1):
        rc = lib.bcjr_fb_backward(P(w), P(cb), P(T), P(soft), P(g), B, N, 16, 2, 1, P(d),
                                  P(ws), ws.numel(), sp)
    assert rc == 0
    assert lib.bcjr_ws_status(P(ws), sp) == _lib.BCJR_ERR_TIMEOUT
    # every sequence, also those claimed after the failure, has NaN gradients
    assert torch.isnan(d).all()
    wn = w[:3].cpu().numpy()
    s1, _, d1 = _run(wn, cb.cpu().numpy(), 0.5, np.ones((3, N, 1), np.float32))
    s64, _, d64 = oracle.fb(wn, cb.cpu().numpy(), 0.5, 16, 2, 1, grad_soft=np.ones((3, N, 1)))
    np.testing.assert_allclose(d1, d64, rtol=1e-4, atol=1e-5)


def test_kernel_launch_count(cuda_ok):
    """bcjr_kernel_launches reports the grids a call launches: two for the
    L=16, V=1 backward above one round of the 2-CTA grid (74 clusters of one
    sequence on a B200), one otherwise."""
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    n = lambda B, V, flag: lib.bcjr_kernel_launches(B, 256 // V, 16, 2, V, flag)
    assert n(4096, 1, _lib.WS_BACKWARD) == 2
    assert n(74, 1, _lib.WS_BACKWARD) == 1
    assert n(4096, 1, _lib.WS_FORWARD) == 1
    assert n(4096, 2, _lib.WS_BACKWARD) == 1
    assert n(0, 1, _lib.WS_BACKWARD) == 0
    assert n(4096, 1, _lib.WS_FORWARD | _lib.WS_BACKWARD) == 0


def test_graph_capture_replays_forward_and_backward(cuda_ok):
    """Forward + backward captured in one CUDA graph through the C ABI (the
    backward with its two grids, B above one round of the 2-CTA grid) replay
    bitwise like eager calls, also after the inputs change in place."""
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda")
    rng = np.random.default_rng(31)
    B, N = 160, 32
    cb = torch.tensor(rng.standard_normal((65536, 1)), dtype=torch.float32, device=dev)
    w = torch.tensor(rng.standard_normal((B, N, 1)), dtype=torch.float32, device=dev)
    g = torch.tensor(rng.standard_normal((B, N, 1)), dtype=torch.float32, device=dev)
    T = torch.tensor(0.5, device=dev)
    soft, logZ, d = torch.empty_like(w), torch.empty(B, device=dev), torch.empty_like(w)
    ws_f = _lib.workspace(B, N, 16, 2, 1, _lib.WS_FORWARD, dev)
    ws_b = _lib.workspace(B, N, 16, 2, 1, _lib.WS_BACKWARD, dev)
    assert lib.bcjr_kernel_launches(B, N, 16, 2, 1, _lib.WS_BACKWARD) == 2
    P = _lib.ptr

    def calls(stream):
        sp = ctypes.c_void_p(stream.cuda_stream)
        assert lib.bcjr_fb_forward(P(w), P(cb), P(T), B, N, 16, 2, 1, P(soft), P(logZ),
                                   P(ws_f), ws_f.numel(), sp) == 0
        assert lib.bcjr_fb_backward(P(w), P(cb), P(T), P(soft), P(g), B, N, 16, 2, 1, P(d),
                                    P(ws_b), ws_b.numel(), sp) == 0

    def eager():
        calls(torch.cuda.current_stream())
        torch.cuda.synchronize()
        return soft.clone(), logZ.clone(), d.clone()

    ref = eager()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=side):
        calls(side)
    for x in (soft, logZ, d):
        x.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip((soft, logZ, d), ref):
        assert torch.equal(a, b)
    w.copy_(torch.tensor(rng.standard_normal((B, N, 1)), dtype=torch.float32, device=dev))
    graph.replay()
    torch.cuda.synchronize()
    got = (soft.clone(), logZ.clone(), d.clone())
    want = eager()
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    del graph


@pytest.mark.parametrize("V,N,B", [(1, 64, 300), (2, 32, 200)])
def test_reserved_sms_leave_results_unchanged(cuda_ok, V, N, B):
    """Leaving SMs free for collectives (bcjr_set_reserved_sms) shrinks the
    cluster grids and the workspace, and changes nothing in the results:
    bitwise the same soft codewords, log Z and gradient (each sequence is
    computed by one cluster, in a fixed order of operations).  The 4-CTA
    grids use 132 of 148 SMs, so a reserve of up to 16 leaves them as they
    are; 24 shrinks every grid (and drops the L=16 backward's 2-CTA grid)."""
    import quant_2bit_b200 as q
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(31 + V)
    dev = torch.device("cuda")
    cb = torch.tensor(rng.standard_normal((65536, V)), dtype=torch.float32, device=dev)
    w = torch.tensor(rng.standard_normal((B, N, V)), dtype=torch.float32, device=dev)
    g = torch.tensor(rng.standard_normal((B, N, V)), dtype=torch.float32, device=dev)
    outs = []
    sizes = []
    for r in (0, 8, 24):
        with _lib.reserved_sms(r):
            sizes.append(lib.bcjr_workspace_bytes(B, N, 16, 2, V, _lib.WS_FORWARD | _lib.WS_BACKWARD))
            soft, logZ = q.bcjr_soft_forward(w, cb, 0.5, 16, 2, V)
            d = q.bcjr_soft_backward(w, cb, 0.5, soft, g, 16, 2, V)
        torch.cuda.synchronize()
        outs.append((soft.cpu(), logZ.cpu(), d.cpu()))
    assert sizes[0] >= sizes[1] >= sizes[2] and sizes[0] > sizes[2]
    for o in outs[1:]:
        for a, b in zip(o, outs[0]):
            assert torch.equal(a, b)


def test_mufu_probe_measures_the_pipe(cuda_ok):
    """bcjr_probe_mufu, the measured roofline denominator: its ex2 rate lies
    between 60 % and 105 % of 148 SMs x 16 ops per clock at the B200's
    1965 MHz maximum (4653 Gop/s), and its op count is what was launched."""
    import ctypes
    from quant_2bit_b200 import _lib
    dev = torch.device("cuda")
    gops = _lib.measure_mufu_gops(dev, iters=4096, repeats=2)
    spec = torch.cuda.get_device_properties(dev).multi_processor_count * 16 * 1.965
    assert 0.6 * spec < gops < 1.05 * spec, (gops, spec)
    lib = _lib.load()
    ops = ctypes.c_double(0.0)
    out = torch.zeros(1, device=dev)
    assert lib.bcjr_probe_mufu(_lib.ptr(out), 10, ctypes.byref(ops), _lib.stream_ptr(dev)) == 0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    assert ops.value == sms * 4 * 256 * 10 * 8
    assert lib.bcjr_probe_mufu(_lib.ptr(out), 0, ctypes.byref(ops), _lib.stream_ptr(dev)) == 1
