"""CPU tests: the oracle against the reference's golden outputs.

Pins the checker before anything is checked against it: the C restatement
(fp64 and fp32), the brute-force enumerator and the torch port must
reproduce the outputs of the reference itself (tests/golden/*.npz, made by
importing the reference's eager bcjr_forward_backward).
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden_names, load_golden, parity_report
from oracle import oracle, torch_port

SMALL = golden_names("small_*.npz")


@pytest.mark.parametrize("name", SMALL)
def test_c_oracle_f64_matches_reference_f64(name):
    d = load_golden(name)
    soft, logZ, dseq = oracle.fb(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"],
                                 grad_soft=d["grad"], dtype=np.float64)
    np.testing.assert_allclose(soft, d["soft64"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(logZ, d["logZ64"], rtol=1e-12, atol=1e-10)
    np.testing.assert_allclose(dseq, d["dseq64"], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("name", SMALL)
def test_c_oracle_f32_matches_reference_f32(name):
    """The fp32 restatement follows the monolithic adjoint backward, whose
    rounding differs from the eager autograd's; the reference's own parity
    scripts accept 1e-3 normwise between its fp32 variants
    (src/tripwires/test_bcjr_monolithic_parity.py:43,53)."""
    d = load_golden(name)
    soft, logZ, dseq = oracle.fb(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"],
                                 grad_soft=d["grad"], dtype=np.float32)
    for ours, key in ((soft, "soft"), (dseq, "dseq")):
        rep = parity_report(ours, d[key + "32"], d[key + "64"])
        assert rep["norm32"] < 1e-3, (name, key, rep)


@pytest.mark.parametrize("name", ["c1_ones.npz", "c1_randgrad.npz"])
def test_c_oracle_config1(name):
    """Config 1 (L=8, k=2, V=1, N=256, 64 sequences, T=1) in full."""
    d = load_golden(name)
    soft, logZ, dseq = oracle.fb(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"],
                                 grad_soft=d["grad"], dtype=np.float64)
    np.testing.assert_allclose(soft, d["soft64"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(logZ, d["logZ64"], rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose(dseq, d["dseq64"], rtol=1e-8, atol=1e-10)


@pytest.mark.parametrize("name", ["l16_gauss_T0.5.npz", "l16_t3_T0.05.npz", "l16_v2.npz",
                                  "l16v2_gauss_T0.05.npz", "l16v2_hyb_T0.3.npz",
                                  "c3_scaled_T0.5.npz", "c5_scaled_T0.5.npz"])
def test_c_oracle_l16(name):
    """L=16 production trellis (V=1 at T=0.5 and the hardest T; V=2 at T=0.5,
    at the hardest T, and with a HYB codebook; the largest-scale tiles of
    the Llama and OLMoE layer workloads, |w| up to ~6.4)."""
    d = load_golden(name)
    soft, logZ, dseq = oracle.fb(d["w"], d["cb"], d["T"], d["L"], d["k"], d["V"],
                                 grad_soft=d["grad"], dtype=np.float64)
    np.testing.assert_allclose(soft, d["soft64"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(logZ, d["logZ64"], rtol=1e-12, atol=1e-8)
    np.testing.assert_allclose(dseq, d["dseq64"], rtol=1e-7, atol=1e-9)


@pytest.mark.parametrize("case", [(4, 2, 1, 4, 3, 1.0), (6, 2, 1, 4, 2, 0.5),
                                  (4, 1, 1, 6, 2, 0.7), (4, 2, 2, 3, 2, 1.3),
                                  (5, 1, 1, 7, 2, 0.3)])
def test_brute_force_matches_c_oracle(case):
    L, k, V, N, B, T = case
    rng = np.random.default_rng(L * 100 + N)
    cb = rng.standard_normal((1 << L, V))
    w = rng.standard_normal((B, N, V))
    g = rng.standard_normal((B, N, V))
    s1, z1, d1 = oracle.brute_force(w, cb, T, L, k, grad_soft=g)
    s2, z2, d2 = oracle.fb(w, cb, T, L, k, V, grad_soft=g)
    np.testing.assert_allclose(s2, s1, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(z2, z1, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(d2, d1, rtol=1e-9, atol=1e-11)


def test_known_answer_all_zero_energies():
    """cb = 0, w = 0: every path has weight 1, log Z = N ln 2^b + L ln 2 and
    soft = 0 (e.g. L=6, b=2, N=5 gives 11.0904)."""
    for L, k, V, N in [(6, 2, 1, 5), (8, 1, 2, 9), (10, 2, 2, 3)]:
        soft, logZ, _ = oracle.fb(np.zeros((2, N, V)), np.zeros((1 << L, V)), 0.7, L, k, V)
        np.testing.assert_allclose(logZ, oracle.all_zero_logZ(N, L, k, V), rtol=1e-12)
        assert np.abs(soft).max() == 0.0
    assert abs(oracle.all_zero_logZ(5, 6) - 11.0904) < 1e-4


def test_high_temperature_limit_is_codebook_mean():
    """T -> infinity: P_t uniform over states, soft -> mean codebook
    (src/bcjr/forward_backward.py:39-40)."""
    rng = np.random.default_rng(3)
    L = 6
    cb = rng.standard_normal((1 << L, 1))
    w = rng.standard_normal((1, 8, 1))
    soft, _, _ = oracle.fb(w, cb, 1e7, L, 2, 1)
    np.testing.assert_allclose(soft[0, :, 0], np.full(8, cb.mean()), atol=1e-5)


@pytest.mark.parametrize("L,k,V", [(6, 2, 1), (8, 2, 2), (6, 1, 2)])
def test_low_temperature_limit_is_the_viterbi_walk(L, k, V):
    """T -> 0: the posterior concentrates on the minimum-cost walk, so the soft
    codewords approach the hard Viterbi reconstruction and -T log Z approaches
    that walk's cost (src/bcjr/forward_backward.py:37-38); the two oracles are
    independent restatements (sum-product in fp64, exact min-sum)."""
    from oracle import viterbi
    rng = np.random.default_rng(L * 10 + V)
    cb = rng.standard_normal((1 << L, V))
    w = rng.standard_normal((3, 12, V))
    T = 1e-5
    soft, logZ, _ = oracle.fb(w, cb, T, L, k, V)
    _, _, rec, mse = viterbi.viterbi(w.reshape(3, -1).astype(np.float32),
                                     cb.astype(np.float32), L, k, V)
    np.testing.assert_allclose(soft.reshape(3, -1), rec, atol=1e-5)
    cost = mse.astype(np.float64) * 12 * V
    np.testing.assert_allclose(-T * logZ, cost, rtol=1e-5, atol=1e-4)


def test_shift_invariance_of_soft():
    """Shifting the codebook and the weights by the same constant leaves every
    |c - w| unchanged: log Z is unchanged and soft shifts by the constant."""
    rng = np.random.default_rng(4)
    L = 6
    cb = rng.standard_normal((1 << L, 1))
    w = rng.standard_normal((2, 10, 1))
    s1, z1, _ = oracle.fb(w, cb, 0.6, L, 2, 1)
    s2, z2, _ = oracle.fb(w + 0.25, cb + 0.25, 0.6, L, 2, 1)
    np.testing.assert_allclose(s2, s1 + 0.25, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(z2, z1, rtol=1e-12)


@pytest.mark.parametrize("name", ["small_L6_k2_V1.npz", "small_L8_k2_V2.npz"])
def test_torch_port_reproduces_reference(name):
    """The torch restatement used as the timed CPU baseline gives the
    reference's fp32 outputs (same operations, same order)."""
    d = load_golden(name)
    w = torch.from_numpy(d["w"])
    cb = torch.from_numpy(d["cb"])
    g = torch.from_numpy(d["grad"])
    soft, logZ, dseq = torch_port.fwd_bwd(w, cb, d["T"], d["L"], d["k"], d["V"], grad_soft=g,
                                          chunk=w.shape[0])
    np.testing.assert_allclose(soft.numpy(), d["soft32"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(logZ.numpy(), d["logZ32"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(dseq.numpy(), d["dseq32"], rtol=1e-5, atol=1e-6)


def test_reference_own_error_is_recorded():
    """The fixtures carry the reference's fp32-vs-fp64 deviation; at T=0.05
    it exceeds the 1e-4 / 1e-5 tolerance, which is why parity tests compare
    against the fp64 run and allow the reference its own rounding."""
    d = load_golden("l16_gauss_T0.05.npz")
    own = np.abs(d["soft32"] - d["soft64"]).max()
    assert own > 1e-5


def test_hyb_codebook_matches_reference_decoder():
    """The HYB codebook rebuilt from the fixture's LUT equals the reference
    decoder's output (src/codes/ref.py:99-114) on the rows stored with it,
    and has the code's structure: every row is +-a LUT row."""
    from conftest import hyb_codebook
    d = dict(np.load(os.path.join(GOLDEN, "l16v2_hyb_T0.3.npz")))
    cb = hyb_codebook(d["lut"])
    np.testing.assert_array_equal(cb[d["cb_rows"]], d["cb_at_rows"])
    assert cb.shape == (65536, 2)
    assert np.isin(cb[:, 0], d["lut"][:, 0]).all()
    assert np.isin(np.abs(cb[:, 1]), np.abs(d["lut"][:, 1])).all()
