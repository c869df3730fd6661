"""CPU tests of the caller-side oracle (oracle/rht.py, oracle/torch_port.py)
against the reference's outputs (tests/golden/rht.npz), the algebra the
native kernels rely on (orthogonality, the tile/untile adjoint pair), and the
C ABI's shape checks (no GPU work)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import rht, torch_port


def _golden():
    return dict(np.load(os.path.join(GOLDEN, "rht.npz")))


def test_oracle_rht_matches_reference():
    d = _golden()
    np.testing.assert_allclose(rht.apply_rht(d["W"], d["sign_l"], d["sign_r"]), d["W_rht"],
                               rtol=0, atol=1e-6)
    np.testing.assert_allclose(rht.apply_inverse_rht(d["W_rht"], d["sign_l"], d["sign_r"]),
                               d["W_inv"], rtol=0, atol=1e-6)
    # the reference tiles in float32 (src/qat/ste.py:96-98)
    np.testing.assert_array_equal(rht.tile(d["W_rht"].astype(np.float32)), d["tiles"])


def test_torch_restatement_matches_oracle():
    d = _golden()
    args = [torch.tensor(d[k], dtype=torch.float64) for k in ("W", "sign_l", "sign_r")]
    np.testing.assert_allclose(torch_port.apply_rht(*args).numpy(),
                               rht.apply_rht(d["W"], d["sign_l"], d["sign_r"]), rtol=0, atol=1e-12)


@pytest.mark.parametrize("m,n", [(16, 16), (32, 64), (128, 16)])
def test_rht_is_orthogonal_and_tiles_round_trip(m, n):
    rng = np.random.default_rng(m + n)
    W = rng.standard_normal((m, n))
    sl = rng.choice([-1.0, 1.0], m)
    sr = rng.choice([-1.0, 1.0], n)
    Wt = rht.apply_rht(W, sl, sr)
    np.testing.assert_allclose(np.linalg.norm(Wt), np.linalg.norm(W), rtol=1e-12)
    np.testing.assert_allclose(rht.apply_inverse_rht(Wt, sl, sr), W, rtol=0, atol=1e-12)
    np.testing.assert_array_equal(rht.untile(rht.tile(W), m, n), W)


def test_tile_and_untile_ops_are_adjoint():
    """<A(W, mu), S> = <W, B(S, mu)>: the backward of each native op is the
    other op with the same scale."""
    rng = np.random.default_rng(5)
    m, n = 32, 64
    W = rng.standard_normal((m, n))
    S = rng.standard_normal((m * n // 256, 256))
    sl, sr = rng.choice([-1.0, 1.0], m), rng.choice([-1.0, 1.0], n)
    mu = 0.37
    A, _ = rht.rht_tile(W, sl, sr, mu=mu)
    B = rht.untile_irht(S, sl, sr, m, n, mu)
    np.testing.assert_allclose(np.sum(A * S), np.sum(W * B), rtol=1e-12)


def test_default_scale_is_rms_of_rotated_weight():
    rng = np.random.default_rng(6)
    W = 3.0 * rng.standard_normal((64, 32))
    sl, sr = rng.choice([-1.0, 1.0], 64), rng.choice([-1.0, 1.0], 32)
    seqs, r = rht.rht_tile(W, sl, sr)
    np.testing.assert_allclose(r, np.sqrt(np.mean(W ** 2)), rtol=1e-12)   # RHT keeps the norm
    np.testing.assert_allclose(np.sqrt(np.mean(seqs ** 2)), 1.0, rtol=1e-12)


def test_c_abi_rejects_bad_rht_shapes():
    from quant_2bit_b200 import _lib
    lib = _lib.load()
    assert lib.bcjr_rht_workspace_bytes(15, 16) == 0
    assert lib.bcjr_rht_workspace_bytes(16, 65536) == 0
    assert lib.bcjr_rht_workspace_bytes(16, 32) > 2 * 16 * 32 * 4
    for m, n in ((24, 16), (16, 8), (0, 16)):
        assert lib.bcjr_rht(None, None, None, m, n, 0, None, None, 0, None) == _lib.BCJR_ERR_BAD_SHAPE
        assert lib.bcjr_rht_tile(None, None, None, m, n, None, None, None, None, 0,
                                 None) == _lib.BCJR_ERR_BAD_SHAPE
        assert lib.bcjr_untile_irht(None, None, None, m, n, None, None, None, 0,
                                    None) == _lib.BCJR_ERR_BAD_SHAPE
    assert lib.bcjr_rht(None, None, None, 16, 16, 0, None, None, 0,
                        None) == _lib.BCJR_ERR_NULL_POINTER
