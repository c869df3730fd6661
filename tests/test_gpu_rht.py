"""GPU tests of the native RHT / tiling kernels (csrc/bcjr_rht.cu) and the
quantizer wrapper built on them: against the reference's outputs
(tests/golden/rht.npz) and the numpy oracle (oracle/rht.py) at the shapes of
the reference's layers and the extremes the kernels accept, the adjoint
identities the autograd Functions use, and the error behaviour."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import rht

pytestmark = pytest.mark.gpu

SHAPES = [(16, 16), (32, 64), (16, 32768), (32768, 16), (1024, 2048), (2048, 8192), (512, 1024)]


def _inputs(m, n, seed):
    rng = np.random.default_rng(seed)
    W = rng.standard_normal((m, n)).astype(np.float32)
    sl = rng.choice([-1.0, 1.0], m).astype(np.float32)
    sr = rng.choice([-1.0, 1.0], n).astype(np.float32)
    return W, sl, sr


def _cuda(*a):
    return [torch.tensor(x, device="cuda") for x in a]


def _close(got, ref, tol=2e-6):
    """Absolute error relative to the largest entry (the transform spreads
    fp32 rounding evenly over the output)."""
    ref = np.asarray(ref, np.float64)
    err = np.abs(np.asarray(got, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err < tol, err


def test_rht_matches_reference_golden(cuda_ok):
    from quant_2bit_b200 import quant
    d = dict(np.load(os.path.join(GOLDEN, "rht.npz")))
    W, sl, sr = _cuda(d["W"], d["sign_l"], d["sign_r"])
    np.testing.assert_allclose(quant.apply_rht_gpu(W, sl, sr).cpu().numpy(), d["W_rht"],
                               rtol=1e-5, atol=1e-6)
    Wt = torch.tensor(d["W_rht"].astype(np.float32), device="cuda")
    np.testing.assert_allclose(quant.apply_inverse_rht_gpu(Wt, sl, sr).cpu().numpy(), d["W_inv"],
                               rtol=1e-5, atol=1e-6)
    seqs, r = quant._RhtTile.apply(W, sl, sr)
    rms = float(r)
    np.testing.assert_allclose(seqs.cpu().numpy() * rms, d["tiles"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("m,n", SHAPES)
def test_rht_and_inverse_vs_oracle(cuda_ok, m, n):
    from quant_2bit_b200 import quant
    W, sl, sr = _inputs(m, n, m + 3 * n)
    Wd, sld, srd = _cuda(W, sl, sr)
    Wt = quant.apply_rht_gpu(Wd, sld, srd)
    _close(Wt.cpu().numpy(), rht.apply_rht(W, sl, sr))
    _close(quant.apply_inverse_rht_gpu(Wt, sld, srd).cpu().numpy(), W)


@pytest.mark.parametrize("m,n", SHAPES)
def test_rht_tile_and_untile_vs_oracle(cuda_ok, m, n):
    from quant_2bit_b200 import quant
    W, sl, sr = _inputs(m, n, 7 * m + n)
    Wd, sld, srd = _cuda(W, sl, sr)
    seqs, r = quant._RhtTile.apply(Wd, sld, srd)
    ref_seqs, ref_rms = rht.rht_tile(W, sl, sr)
    np.testing.assert_allclose(float(r), ref_rms, rtol=1e-6)
    _close(seqs.cpu().numpy(), ref_seqs)
    S = np.random.default_rng(m).standard_normal((m * n // 256, 256)).astype(np.float32)
    out = quant._UntileIrht.apply(torch.tensor(S, device="cuda"), sld, srd, r, m, n)
    _close(out.cpu().numpy(), rht.untile_irht(S, sl, sr, m, n, float(r)))


def test_tile_ops_are_adjoint_on_device(cuda_ok):
    """<A(W), G> = <W, A^T(G)> through autograd: the backward of each op is the
    other op."""
    from quant_2bit_b200 import quant
    m, n = 256, 512
    W, sl, sr = _inputs(m, n, 11)
    Wd = torch.tensor(W, device="cuda", requires_grad=True)
    sld, srd = _cuda(sl, sr)
    G = torch.randn(m * n // 256, 256, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    seqs, r = quant._RhtTile.apply(Wd, sld, srd)
    (seqs * G).sum().backward()
    ref = rht.untile_irht(G.cpu().numpy(), sl, sr, m, n, 1.0 / float(r))
    _close(Wd.grad.cpu().numpy(), ref)
    S = torch.randn(m * n // 256, 256, device="cuda", requires_grad=True)
    Gw = torch.randn(m, n, device="cuda")
    (quant._UntileIrht.apply(S, sld, srd, r, m, n) * Gw).sum().backward()
    ref2, _ = rht.rht_tile(Gw.cpu().numpy(), sl, sr, mu=float(r))
    _close(S.grad.cpu().numpy(), ref2)


def test_rht_errors(cuda_ok):
    from quant_2bit_b200 import quant
    sl = torch.ones(24, device="cuda")
    with pytest.raises(AssertionError):
        quant.apply_rht_gpu(torch.ones(24, 32, device="cuda"), sl, torch.ones(32, device="cuda"))
    with pytest.raises(RuntimeError):
        quant.apply_rht_gpu(torch.ones(16, 16), torch.ones(16), torch.ones(16))
