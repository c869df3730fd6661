"""GPU parity tests: the sm_100a kernels (through the C ABI) against the
reference's golden outputs and the CPU oracle.

Tolerance (north star): 1e-4 relative, 1e-5 absolute, elementwise, against
the fp64 run of the reference (``vs64``) and against the reference's fp32
output up to that output's own rounding error (``vs32``); see
conftest.parity_report.
"""
import math

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden, parity_report
from oracle import oracle, torch_port

pytestmark = pytest.mark.gpu

ALL_GOLDEN = (golden_names("small_*.npz") + golden_names("c1_*.npz")
              + golden_names("l16_*.npz") + golden_names("l16v2_*.npz")
              + golden_names("c3_*.npz") + golden_names("c5_*.npz"))


def run_ours(w, cb, T, L, k, V, grad, T_as="cuda"):
    import quant_2bit_b200 as q
    dev = torch.device("cuda")
    x = torch.as_tensor(w, dtype=torch.float32, device=dev).clone().requires_grad_(True)
    c = torch.as_tensor(cb, dtype=torch.float32, device=dev)
    Tt = {"cuda": torch.tensor(T, dtype=torch.float32, device=dev),
          "float": float(T), "cpu": torch.tensor(T)}[T_as]
    soft, logZ = q.bcjr_forward_backward(x, c, Tt, L=L, k=k, V=V)
    (soft * torch.as_tensor(grad, dtype=torch.float32, device=dev)).sum().backward()
    torch.cuda.synchronize()
    return soft.detach().cpu().numpy(), logZ.detach().cpu().numpy(), x.grad.cpu().numpy()


@pytest.mark.parametrize("name", ALL_GOLDEN)
def test_parity_with_reference_goldens(cuda_ok, name):
    d = load_golden(name)
    soft, logZ, dseq = run_ours(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"], d["grad"])
    for ours, key in ((soft, "soft"), (dseq, "dseq")):
        rep = parity_report(ours, d[key + "32"], d[key + "64"])
        assert rep["vs64"], (name, key, rep)
        assert rep["vs32"], (name, key, rep)
    # log Z: absolute error scales with |log Z| ~ N; relative 1e-6 of the fp64 value
    np.testing.assert_allclose(logZ, d["logZ64"], rtol=2e-6, atol=1e-4)


@pytest.mark.parametrize("T_as", ["float", "cpu"])
def test_temperature_argument_forms(cuda_ok, T_as):
    d = load_golden("small_L6_k2_V1.npz")
    a = run_ours(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"], d["grad"], T_as="cuda")
    b = run_ours(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"], d["grad"], T_as=T_as)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_deterministic(cuda_ok):
    d = load_golden("small_L10_k2_V1.npz")
    a = run_ours(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"], d["grad"])
    b = run_ours(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"], d["grad"])
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("case", [(6, 2, 1, 1, 3), (6, 2, 1, 2, 1), (8, 2, 2, 1, 5),
                                  (4, 2, 1, 7, 2), (5, 1, 1, 3, 9), (16, 2, 1, 1, 2),
                                  (16, 2, 1, 3, 1), (16, 2, 2, 2, 1)])
def test_edge_shapes_against_oracle(cuda_ok, case):
    """N = 1, B = 1, odd B, L = kV (a single group), L=16 with tiny N."""
    L, k, V, N, B = case
    rng = np.random.default_rng(L + 17 * N + 101 * B)
    cb = rng.standard_normal((1 << L, V)).astype(np.float32)
    w = rng.standard_normal((B, N, V)).astype(np.float32)
    g = rng.standard_normal((B, N, V)).astype(np.float32)
    T = 0.7
    s64, z64, d64 = oracle.fb(w, cb, T, L, k, V, grad_soft=g)
    soft, logZ, dseq = run_ours(w, cb, T, L, k, V, g)
    np.testing.assert_allclose(soft, s64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dseq, d64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(logZ, z64, rtol=2e-6, atol=1e-4)


def test_empty_batch(cuda_ok):
    import quant_2bit_b200 as q
    x = torch.zeros((0, 16, 1), device="cuda", requires_grad=True)
    cb = torch.randn(256, 1, device="cuda")
    soft, logZ = q.bcjr_forward_backward(x, cb, 1.0, L=8, k=2, V=1)
    assert soft.shape == (0, 16, 1) and logZ.shape == (0,)
    soft.sum().backward()
    assert x.grad.shape == (0, 16, 1)


def test_non_contiguous_input(cuda_ok):
    import quant_2bit_b200 as q
    rng = np.random.default_rng(5)
    base = torch.tensor(rng.standard_normal((20, 3, 1)), dtype=torch.float32, device="cuda")
    x = base.transpose(0, 1)                      # (3, 20, 1), non-contiguous
    cb = torch.tensor(rng.standard_normal((256, 1)), dtype=torch.float32, device="cuda")
    s1, z1 = q.bcjr_forward_backward(x, cb, 0.8, L=8, k=2, V=1)
    s2, z2 = q.bcjr_forward_backward(x.contiguous(), cb, 0.8, L=8, k=2, V=1)
    assert torch.equal(s1, s2) and torch.equal(z1, z2)


def test_shape_errors_mirror_reference(cuda_ok):
    import quant_2bit_b200 as q
    x = torch.randn(2, 8, 1, device="cuda")
    with pytest.raises(AssertionError):
        q.bcjr_forward_backward(x, torch.randn(200, 1, device="cuda"), 1.0, L=8, k=2, V=1)
    with pytest.raises(AssertionError):
        q.bcjr_forward_backward(x, torch.randn(256, 1, device="cuda"), 1.0, L=8, k=2, V=2)
    with pytest.raises(ValueError):
        q.bcjr_forward_backward(torch.randn(2, 8, 2, device="cuda"),
                                torch.randn(256, 2, device="cuda"), 1.0, L=8, k=3, V=2)
    with pytest.raises(AssertionError):
        q.BcjrForwardBackwardMonolithic.apply(x.double(), torch.randn(256, 1, device="cuda"),
                                              torch.tensor(1.0, device="cuda"), None, None)


def test_monolithic_api_with_reference_tables(cuda_ok):
    """BcjrForwardBackwardMonolithic.apply(seq, cb, T, preds, succs) with the
    V=2 (16-predecessor) tables the reference's callers pass."""
    import quant_2bit_b200 as q
    d = load_golden("small_L8_k2_V2.npz")
    preds, succs = q.build_pred_succ_tables(L=8, k=2, V=2, device="cuda")
    x = torch.tensor(d["w"], device="cuda", requires_grad=True)
    cb = torch.tensor(d["cb"], device="cuda")
    T = torch.tensor(d["T"], dtype=torch.float32, device="cuda")
    soft = q.BcjrForwardBackwardMonolithic.apply(x, cb, T, preds, succs)
    soft.backward(torch.tensor(d["grad"], device="cuda"))
    assert parity_report(soft.detach().cpu().numpy(), d["soft32"], d["soft64"])["vs64"]
    assert parity_report(x.grad.cpu().numpy(), d["dseq32"], d["dseq64"])["vs64"]
    s2, none = q.bcjr_forward_backward_monolithic(x.detach(), cb, T, preds=preds, succs=succs)
    assert none is None and torch.equal(s2, soft.detach())


def test_tables_match_reference_definition(cuda_ok):
    import quant_2bit_b200 as q
    for (L, k, V) in [(8, 2, 1), (16, 2, 2), (6, 1, 1)]:
        p1, s1 = q.build_pred_succ_tables(L, k, V, device="cuda")
        p2, s2 = torch_port.build_pred_succ_tables(L, k, V)
        assert torch.equal(p1.cpu(), p2) and torch.equal(s1.cpu(), s2)


def test_logZ_gradient(cuda_ok):
    """Gradient through log_Z alone and through soft + log_Z together, vs
    the reference's autograd (torch port, fp64)."""
    import quant_2bit_b200 as q
    rng = np.random.default_rng(11)
    L, k, V, N, B, T = 6, 2, 1, 12, 3, 0.6
    cb = rng.standard_normal((1 << L, V))
    w = rng.standard_normal((B, N, V))
    gz = rng.standard_normal(B)
    gs = rng.standard_normal((B, N, V))
    xr = torch.tensor(w).requires_grad_(True)
    sr, zr = torch_port.bcjr_forward_backward(xr, torch.tensor(cb), T, L, k, V)
    ((sr * torch.tensor(gs)).sum() + (zr * torch.tensor(gz)).sum()).backward()
    x = torch.tensor(w, dtype=torch.float32, device="cuda", requires_grad=True)
    s, z = q.bcjr_forward_backward(x, torch.tensor(cb, dtype=torch.float32, device="cuda"),
                                   T, L=L, k=k, V=V)
    ((s * torch.tensor(gs, dtype=torch.float32, device="cuda")).sum()
     + (z * torch.tensor(gz, dtype=torch.float32, device="cuda")).sum()).backward()
    np.testing.assert_allclose(x.grad.cpu().numpy(), xr.grad.numpy(), rtol=1e-4, atol=1e-5)
    x2 = torch.tensor(w, dtype=torch.float32, device="cuda", requires_grad=True)
    _, z2 = q.bcjr_forward_backward(x2, torch.tensor(cb, dtype=torch.float32, device="cuda"),
                                    T, L=L, k=k, V=V)
    (z2 * torch.tensor(gz, dtype=torch.float32, device="cuda")).sum().backward()
    xr2 = torch.tensor(w).requires_grad_(True)
    _, zr2 = torch_port.bcjr_forward_backward(xr2, torch.tensor(cb), T, L, k, V)
    (zr2 * torch.tensor(gz)).sum().backward()
    np.testing.assert_allclose(x2.grad.cpu().numpy(), xr2.grad.numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("case", [(6, 2, 1, 10, 2, 0.7), (8, 2, 2, 6, 2, 1.1), (5, 1, 1, 9, 3, 0.4)])
def test_return_internals(cuda_ok, case):
    import quant_2bit_b200 as q
    L, k, V, N, B, T = case
    rng = np.random.default_rng(L * 7 + N)
    cb = rng.standard_normal((1 << L, V))
    w = rng.standard_normal((B, N, V))
    Pr, lar, lbr = torch_port.internals(torch.tensor(w), torch.tensor(cb), T, L, k, V)
    out = q.bcjr_forward_backward(torch.tensor(w, dtype=torch.float32, device="cuda"),
                                  torch.tensor(cb, dtype=torch.float32, device="cuda"),
                                  T, L=L, k=k, V=V, return_internals=True)
    soft, logZ, P, la, lb = [o.detach().cpu().numpy() for o in out]
    np.testing.assert_allclose(P, Pr.numpy(), rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(la, lar.numpy(), rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(lb, lbr.numpy(), rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(P.sum(-1), 1.0, rtol=1e-5)


def _config2_inputs(nseq=4096, seed=0):
    g = torch.Generator().manual_seed(seed)
    cb = torch.randn(65536, 1, generator=g)
    w = torch.randn(nseq, 256, 1, generator=g)
    return cb, w


def test_full_size_config2_properties(cuda_ok):
    """Config 2 at full size (4,096 sequences, L=16, T=0.5): sampled
    sequences against the fp64 oracle, sharding invariance (a sub-batch gives
    bitwise the same rows), soft inside the codebook's range, and linearity
    of the backward in the upstream gradient."""
    import quant_2bit_b200 as q
    cb, w = _config2_inputs()
    T = 0.5
    dev = torch.device("cuda")
    cbd, wd = cb.to(dev), w.to(dev)
    soft, logZ = q.bcjr_soft_forward(wd, cbd, T, 16, 2, 1)
    g1 = torch.ones_like(soft)
    g2 = torch.randn(soft.shape, generator=torch.Generator().manual_seed(2)).to(dev)
    d1 = q.bcjr_soft_backward(wd, cbd, T, soft, g1, 16, 2, 1)
    d2 = q.bcjr_soft_backward(wd, cbd, T, soft, g2, 16, 2, 1)
    d12 = q.bcjr_soft_backward(wd, cbd, T, soft, g1 + g2, 16, 2, 1)
    torch.cuda.synchronize()
    assert torch.isfinite(soft).all() and torch.isfinite(d1).all()
    assert soft.min() >= cb.min() - 1e-5 and soft.max() <= cb.max() + 1e-5
    lin = (d12 - d1 - d2).abs().max().item()
    assert lin <= 1e-4 * d12.abs().max().item() + 1e-5, lin
    # sharding invariance: rows 1000..1003 computed alone
    s_sub, z_sub = q.bcjr_soft_forward(wd[1000:1004], cbd, T, 16, 2, 1)
    d_sub = q.bcjr_soft_backward(wd[1000:1004], cbd, T, s_sub, g1[1000:1004], 16, 2, 1)
    assert torch.equal(s_sub, soft[1000:1004]) and torch.equal(d_sub, d1[1000:1004])
    # sampled rows against the fp64 oracle
    idx = [0, 4095]
    s64, z64, dd64 = oracle.fb(w[idx].numpy(), cb.numpy(), T, 16, 2, 1,
                               grad_soft=np.ones((2, 256, 1)))
    np.testing.assert_allclose(soft[idx].cpu().numpy(), s64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(d1[idx].cpu().numpy(), dd64, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(logZ[idx].cpu().numpy(), z64, rtol=2e-6)


@pytest.mark.parametrize("name", ["c3_scaled_T0.5.npz", "c5_scaled_T0.5.npz"])
def test_scaled_layer_tiles_inside_a_full_batch(cuda_ok, name):
    """Configs 3 and 5 scale the weights by U[0.5, 2] per row or per expert,
    so |w| reaches ~6.4 at T = 0.5, a cost range the N(0,1) and Student-t
    goldens do not reach.  The reference's outputs for the largest-scale
    tiles of each layer, placed among 192 sequences (scale-2 fillers), so
    that the forward runs two rounds of clusters and the L=16 backward its
    4-CTA and 2-CTA grids side by side; elementwise against the reference's
    fp64 and fp32 outputs at 1e-4 relative / 1e-5 absolute."""
    d = load_golden(name)
    rng = np.random.default_rng(77)
    B, N = 192, d["w"].shape[1]
    w = (2.0 * rng.standard_normal((B, N, 1))).astype(np.float32)
    g = rng.standard_normal((B, N, 1)).astype(np.float32)
    pos = [5, 100, 191][:d["w"].shape[0]]
    w[pos] = d["w"]
    g[pos] = d["grad"]
    soft, logZ, dseq = run_ours(w, d["cb"], d["T"], 16, 2, 1, g)
    for ours, key in ((soft[pos], "soft"), (dseq[pos], "dseq")):
        rep = parity_report(ours, d[key + "32"], d[key + "64"])
        assert rep["vs64"], (name, key, rep)
        assert rep["vs32"], (name, key, rep)
    np.testing.assert_allclose(logZ[pos], d["logZ64"], rtol=2e-6, atol=1e-4)
    assert np.isfinite(soft).all() and np.isfinite(dseq).all()


@pytest.mark.parametrize("L,k,V,N", [(16, 2, 1, 64), (16, 2, 2, 32), (8, 2, 1, 32)])
@pytest.mark.parametrize("bad", [float("nan"), float("inf")])
def test_nan_and_inf_inputs_propagate(cuda_ok, L, k, V, N, bad):
    """NaN policy "propagate", as in the reference: one NaN (or infinite)
    weight makes every local energy of its step NaN there, hence log Z,
    every marginal, soft codeword and gradient entry of that sequence NaN
    (forward_backward.py:98-103, :219-232 under IEEE arithmetic).  The other
    sequences of the batch are unaffected, bitwise."""
    rng = np.random.default_rng(L * 7 + V)
    B = 4
    cb = rng.standard_normal((1 << L, V)).astype(np.float32)
    w = rng.standard_normal((B, N, V)).astype(np.float32)
    g = rng.standard_normal((B, N, V)).astype(np.float32)
    clean = run_ours(w, cb, 0.5, L, k, V, g)
    w_bad = w.copy()
    w_bad[1, N // 2, 0] = bad
    out = run_ours(w_bad, cb, 0.5, L, k, V, g)
    for a, b in zip(out, clean):
        assert np.isnan(a[1]).all()
        keep = [0, 2, 3]
        np.testing.assert_array_equal(a[keep], b[keep])


@pytest.mark.parametrize("L,k,V,N", [(16, 2, 1, 16), (16, 2, 2, 16), (6, 2, 1, 8)])
@pytest.mark.parametrize("T", [0.0, -1.0, float("nan"), float("inf")])
def test_unusable_device_temperature_gives_nan(cuda_ok, L, k, V, N, T):
    """A temperature that is not positive and finite: as a python number it
    is refused on the host (ValueError); on the device it cannot be checked
    without a synchronisation, so every kernel writes NaN into every output
    (soft, log Z, gradient)."""
    import quant_2bit_b200 as q
    rng = np.random.default_rng(3)
    dev = torch.device("cuda")
    cb = torch.tensor(rng.standard_normal((1 << L, V)), dtype=torch.float32, device=dev)
    x = torch.tensor(rng.standard_normal((3, N, V)), dtype=torch.float32, device=dev,
                     requires_grad=True)
    soft, logZ = q.bcjr_forward_backward(x, cb, torch.tensor(T, device=dev), L=L, k=k, V=V)
    soft.sum().backward()
    torch.cuda.synchronize()
    assert torch.isnan(soft).all() and torch.isnan(logZ).all() and torch.isnan(x.grad).all()
    with pytest.raises(ValueError):
        q.bcjr_forward_backward(x, cb, T, L=L, k=k, V=V)
