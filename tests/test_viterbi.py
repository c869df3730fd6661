"""Hard Viterbi encoder: the CPU oracle (oracle/viterbi.py) against the
reference's own encodes (tests/golden/viterbi_*.npz, made by running
src/viterbi/encode.py), and (GPU) the sm_100a kernel against both, bit-exact
on walks, bitstreams, start states and reconstructions."""
import numpy as np
import pytest
import torch

from conftest import golden_names, hyb_codebook, load_golden
from oracle import viterbi

NAMES = golden_names("viterbi_*.npz")


def _case(name):
    d = load_golden(name)
    return d, d["cb"].reshape(1 << d["L"], d["V"])


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_encoder(name):
    d, cb = _case(name)
    bits, starts, rec, mse = viterbi.viterbi(d["seqs"], cb, d["L"], d["k"], d["V"])
    np.testing.assert_array_equal(bits, d["bits"])
    np.testing.assert_array_equal(starts, d["starts"])
    np.testing.assert_array_equal(rec, d["recons"])
    np.testing.assert_allclose(mse, d["mses"], rtol=1e-6, atol=1e-7)


def test_large_gpu_case_separates_fused_from_exact_costs():
    """The 520 x 512 batch (V=1) of test_cluster_and_generic_kernels_agree
    holds a one-ulp near-tie between two predecessors, so a kernel whose
    costs a + d*d are one fused multiply-add instead of two roundings fails
    that test: row 101's exact walk (the oracle) differs from the same
    recursion with fma(d, d, a) (emulated in fp64: d*d is exact there)."""
    B, N, V = 520, 512, 1
    rng = np.random.default_rng(B + N + V)          # as the GPU test draws them
    cb = rng.standard_normal((1 << 16, 1)).astype(np.float32)
    seq = rng.standard_normal((B, V * N)).astype(np.float32)[101:102]
    bits, starts, _, _ = viterbi.viterbi(seq, cb, 16, 2, 1)
    c = cb[:, 0]
    top = np.arange(1 << 16) >> 2
    cum = np.zeros(1 << 16, np.float32)
    bps = []
    for t in range(N):
        pc = cum.reshape(4, 1 << 14)
        bps.append(pc.argmin(0))
        d = (c - seq[0, t]).astype(np.float32).astype(np.float64)
        cum = (pc.min(0)[top].astype(np.float64) + d * d).astype(np.float32)
    s = int(np.argmin(cum))
    walk = [s]
    for t in range(N - 1, 0, -1):
        s = (int(bps[t][s >> 2]) << 14) | (s >> 2)
        walk.append(s)
    fused_bits = np.array(walk[::-1]) & 3
    assert not np.array_equal(fused_bits, bits[0])


def test_oracle_walk_replays_to_its_reconstruction():
    """viterbi_decode (src/viterbi/encode.py:313-328): replaying the bitstream
    from the start state gives the reconstruction."""
    rng = np.random.default_rng(3)
    L, k, V = 8, 2, 2
    cb = rng.standard_normal((1 << L, V)).astype(np.float32)
    seqs = rng.standard_normal((3, 40)).astype(np.float32)
    bits, starts, rec, _ = viterbi.viterbi(seqs, cb, L, k, V)
    for i in range(3):
        s = int(starts[i])
        out = []
        for t in range(bits.shape[1]):
            s = ((s << (k * V)) | int(bits[i, t])) & ((1 << L) - 1)
            out.append(cb[s])
        np.testing.assert_array_equal(np.concatenate(out), rec[i])


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_kernel_matches_reference_encoder(cuda_ok, name):
    from quant_2bit_b200.viterbi import viterbi_encode_batched
    d, cb = _case(name)
    out = viterbi_encode_batched(torch.tensor(d["seqs"], device="cuda"),
                                 torch.tensor(cb, device="cuda"), d["L"], d["k"], d["V"])
    bits, starts, rec, mse = [o.cpu().numpy() for o in out]
    np.testing.assert_array_equal(bits, d["bits"])
    np.testing.assert_array_equal(starts, d["starts"])
    np.testing.assert_array_equal(rec, d["recons"])
    np.testing.assert_allclose(mse, d["mses"], rtol=1e-6, atol=1e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("L,k,V,B,N,kind", [(16, 2, 2, 301, 128, "hyb"), (16, 2, 1, 5, 256, "gauss"),
                                            (16, 2, 1, 150, 32, "gauss"), (16, 2, 1, 600, 1, "gauss"),
                                            (16, 2, 2, 600, 1, "gauss"), (16, 2, 1, 3, 512, "tied"),
                                            (16, 2, 2, 2, 1, "gauss"), (12, 1, 2, 7, 33, "gauss"),
                                            (4, 2, 2, 3, 9, "gauss"), (16, 4, 1, 2, 64, "gauss")])
def test_kernel_matches_oracle(cuda_ok, L, k, V, B, N, kind):
    """Ragged and large batches (more sequences than blocks or cluster
    slots), N = 1 with several sequence groups per cluster, the smallest
    trellis, and codebooks with repeated codewords (HYB; "tied": 64 distinct
    values) whose exact ties resolve to the lowest index as in the
    reference."""
    from quant_2bit_b200.viterbi import viterbi_encode_batched
    rng = np.random.default_rng(L * 100 + B)
    if kind == "hyb":
        cb = hyb_codebook(rng.standard_normal((512, 2)).astype(np.float32))
    elif kind == "tied":
        cb = rng.standard_normal(64).astype(np.float32)[rng.integers(0, 64, (1 << L, V))]
    else:
        cb = rng.standard_normal((1 << L, V)).astype(np.float32)
    seqs = rng.standard_normal((B, N * V)).astype(np.float32)
    out = viterbi_encode_batched(torch.tensor(seqs, device="cuda"), torch.tensor(cb, device="cuda"),
                                 L, k, V)
    bits, starts, rec, mse = [o.cpu().numpy() for o in out]
    rb, rs, rr, rm = viterbi.viterbi(seqs, cb, L, k, V)
    np.testing.assert_array_equal(bits, rb)
    np.testing.assert_array_equal(starts, rs)
    np.testing.assert_array_equal(rec, rr)
    np.testing.assert_allclose(mse, rm, rtol=1e-6, atol=1e-7)


@pytest.mark.gpu
def test_v1_entry_point_matches_reference_encodes(cuda_ok):
    """quant_2bit_b200.viterbi.viterbi_encode, the drop-in for the
    reference's V=1 viterbi_encode (numpy in and out, a decode_fn), on the
    reference's own encodes: bit-exact walks (L=16, k=2 on the cluster
    kernel; the smaller trellises on the one-block kernel)."""
    from quant_2bit_b200.viterbi import viterbi_encode
    for name in [n for n in NAMES if "_V1_" in n]:
        d, cb = _case(name)
        for i in range(d["seqs"].shape[0]):
            bits, start, rec, mse = viterbi_encode(d["seqs"][i], int(d["L"]), int(d["k"]),
                                                   lambda s: cb[s, 0])
            np.testing.assert_array_equal(bits, d["bits"][i])
            assert start == int(d["starts"][i])
            np.testing.assert_array_equal(rec, d["recons"][i])
            np.testing.assert_allclose(mse, d["mses"][i], rtol=1e-6, atol=1e-7)
    with pytest.raises(NotImplementedError):
        viterbi_encode(np.zeros(8, np.float32), 16, 2, lambda s: cb[s, 0], return_trace=True)


@pytest.mark.gpu
def test_reference_entry_point_and_errors(cuda_ok):
    from quant_2bit_b200.viterbi import viterbi_encode_v_batched_cuda
    d, cb = _case("viterbi_L16_k2_V2_gauss.npz")
    bits, starts, rec, mse = viterbi_encode_v_batched_cuda(torch.tensor(d["seqs"], device="cuda"),
                                                           torch.tensor(cb, device="cuda"))
    np.testing.assert_array_equal(bits.cpu().numpy(), d["bits"])
    with pytest.raises(RuntimeError):
        viterbi_encode_v_batched_cuda(torch.zeros(2, 8), torch.zeros(16, 2))
    with pytest.raises(AssertionError):
        viterbi_encode_v_batched_cuda(torch.zeros(2, 7, device="cuda"),
                                      torch.zeros(16, 2, device="cuda"))


@pytest.mark.gpu
@pytest.mark.parametrize("V,B,N", [(2, 64, 128), (2, 2049, 8), (2, 3, 512), (2, 1024, 512),
                                   (1, 64, 256), (1, 1000, 8), (1, 520, 512)])
def test_cluster_and_generic_kernels_agree(cuda_ok, V, B, N):
    """L=16, k=2 runs on the 4-CTA cluster kernels (b = 4 at V=2, b = 2 at
    V=1); the test option BCJR_OPT_FORCE_GENERIC sends it to the
    one-block-per-sequence kernel.  Both are exact: identical results,
    across the chunking of the cluster paths (2048 sequences at V=2, whole
    waves of at most 2^18 / N sequences at V=1: 520 x 512 takes two
    chunks) and at the longest N they serve.  The large batches hold
    one-ulp near-ties between predecessors, where a fused multiply-add in
    the costs (d*d rounded into the sum) takes another walk: 520 x 512 at
    V=1 did until the sums were separately rounded."""
    from quant_2bit_b200 import _lib
    from quant_2bit_b200.viterbi import viterbi_encode_batched
    rng = np.random.default_rng(B + N + V)
    cb = (hyb_codebook(rng.standard_normal((512, 2)).astype(np.float32)) if V == 2
          else rng.standard_normal((1 << 16, 1)).astype(np.float32))
    cb = torch.tensor(cb, device="cuda")
    seqs = torch.tensor(rng.standard_normal((B, V * N)).astype(np.float32), device="cuda")
    a = viterbi_encode_batched(seqs, cb, 16, 2, V)
    with _lib.test_option(_lib.OPT_FORCE_GENERIC, 1):
        b = viterbi_encode_batched(seqs, cb, 16, 2, V)
    for x, y in zip(a[:3], b[:3]):
        assert torch.equal(x, y)
    torch.testing.assert_close(a[3], b[3], rtol=1e-6, atol=1e-7)
    # one launch pair (min-sum kernel, walk-back) per chunk on the cluster paths
    chunks = {(2, 2049): 2, (1, 520): 2}.get((V, B), 1)
    assert _lib.load().bcjr_viterbi_launches(B, N, 16, 2, V) == 2 * chunks


@pytest.mark.gpu
@pytest.mark.parametrize("V", [2, 1])
def test_cluster_wait_timeout_is_reported_and_context_survives(cuda_ok, V):
    """Failure detection without a GPU fault: with the test option
    BCJR_OPT_TEST_DROP_SENDS one CTA of each cluster withholds its group
    minima, every bounded wait of the cluster Viterbi expires (~1 s), the
    status word reports BCJR_ERR_TIMEOUT, the walk-back still reads in bounds
    and writes NaN reconstructions and MSEs, and the next normal call on the
    same context is bit-exact."""
    from quant_2bit_b200 import _lib
    from quant_2bit_b200.viterbi import viterbi_encode_batched
    lib = _lib.load()
    dev = torch.device("cuda")
    rng = np.random.default_rng(17)
    B, N = 8, 16
    cb = (hyb_codebook(rng.standard_normal((512, 2)).astype(np.float32)) if V == 2
          else rng.standard_normal((1 << 16, 1)).astype(np.float32))
    cb = torch.tensor(cb, device=dev)
    seqs = torch.tensor(rng.standard_normal((B, V * N)).astype(np.float32), device=dev)
    bits = torch.empty((B, N), dtype=torch.int32, device=dev)
    starts = torch.empty((B,), dtype=torch.int32, device=dev)
    rec = torch.empty((B, V * N), dtype=torch.float32, device=dev)
    mse = torch.empty((B,), dtype=torch.float32, device=dev)
    ws = torch.empty(lib.bcjr_viterbi_workspace_bytes(B, N, 16, 2, V), dtype=torch.uint8, device=dev)
    P, sp = _lib.ptr, _lib.stream_ptr(dev)
    with _lib.test_option(_lib.OPT_TEST_DROP_SENDS, 1):
        rc = lib.bcjr_viterbi(P(seqs), P(cb), B, N, 16, 2, V, P(bits), P(starts), P(rec), P(mse),
                              P(ws), ws.numel(), sp)
    assert rc == 0
    assert lib.bcjr_ws_status(P(ws), sp) == _lib.BCJR_ERR_TIMEOUT
    assert int(starts.max()) < 65536 and int(bits.max()) < (1 << (2 * V))
    assert torch.isnan(rec).all() and torch.isnan(mse).all()
    out = [o.cpu().numpy() for o in viterbi_encode_batched(seqs, cb, 16, 2, V)]
    ref = viterbi.viterbi(seqs.cpu().numpy(), cb.cpu().numpy(), 16, 2, V)
    for a, b in zip(out[:3], ref[:3]):
        np.testing.assert_array_equal(a, b)
