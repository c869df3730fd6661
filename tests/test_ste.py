"""Hard-quantizer side (quant_2bit_b200.ste): the reference's STE quantizers
(src/qat/ste.py) on the native RHT / tiling and Viterbi kernels.  Each stage
is checked against the CPU oracle: the walk the kernel takes for the tiles
the native RHT produced is the reference encoder's walk for the same tiles."""
import numpy as np
import pytest
import torch

from conftest import hyb_codebook, load_golden
from oracle import viterbi as ov

pytestmark = pytest.mark.gpu


def _setup(m, n, seed):
    from quant_2bit_b200 import quant
    rng = np.random.default_rng(seed)
    lut = rng.standard_normal((512, 2)).astype(np.float32)
    cb = torch.tensor(hyb_codebook(lut), device="cuda")
    W = torch.tensor((1.7 * rng.standard_normal((m, n))).astype(np.float32), device="cuda")
    sl = torch.tensor(quant.make_sign_vector(m, seed), device="cuda")
    sr = torch.tensor(quant.make_sign_vector(n, seed + 1), device="cuda")
    return lut, cb, W, sl, sr


@pytest.mark.parametrize("m,n", [(64, 128), (512, 256)])
def test_quantize_forward_gpu_is_rht_viterbi_irht(cuda_ok, m, n):
    from quant_2bit_b200 import quant, ste
    _, cb, W, sl, sr = _setup(m, n, m + n)
    Wq = ste.quantize_forward_gpu(W, sl, sr, cb)
    seqs, rms = quant._tile_call(W, sl, sr, m, n)
    _, _, rec, _ = ov.viterbi(seqs.cpu().numpy(), cb.cpu().numpy(), 16, 2, 2)
    ref = quant._untile_call(torch.tensor(rec, device="cuda"), sl, sr, m, n, rms)
    assert torch.equal(Wq, ref)


def test_quantize_forward_gpu_no_rht_and_ip_ste(cuda_ok):
    from quant_2bit_b200 import quant, ste
    _, cb, W, _, _ = _setup(64, 64, 5)
    Wq = ste.quantize_forward_gpu_no_rht(W, cb)
    scale = W.pow(2).mean().sqrt()
    seqs, info = quant._tile_for_viterbi_gpu(W / scale)
    _, _, rec, _ = ov.viterbi(seqs.cpu().numpy(), cb.cpu().numpy(), 16, 2, 2)
    ref = quant._untile_from_viterbi_gpu(torch.tensor(rec, device="cuda"), info, (64, 64)) * scale
    assert torch.equal(Wq, ref)
    x = W.clone().requires_grad_(True)
    y = ste.TrellisQuantSTE_IP.apply(x, cb)
    assert torch.equal(y, Wq)
    g = torch.randn_like(W)
    y.backward(g)
    assert torch.equal(x.grad, g)


def test_trellis_quant_ste_forward_and_straight_through(cuda_ok):
    from quant_2bit_b200 import ste
    _, cb, W, sl, sr = _setup(128, 64, 9)
    x = W.clone().requires_grad_(True)
    y = ste.TrellisQuantSTE.apply(x, sl.cpu().numpy(), sr, cb)   # numpy signs accepted
    assert torch.equal(y, ste.quantize_forward_gpu(W, sl, sr, cb))
    g = torch.randn_like(W)
    y.backward(g)
    assert torch.equal(x.grad, g)
    with pytest.raises(RuntimeError):
        ste.TrellisQuantSTE.apply(W.cpu(), sl, sr, cb)


def test_make_hyb_codebook_gpu(cuda_ok):
    from quant_2bit_b200 import ste
    lut, cb, _, _, _ = _setup(16, 16, 1)
    assert torch.equal(ste.make_hyb_codebook_gpu(lut), cb)


def test_hyb_codebook_matches_reference_decoder(cuda_ok):
    """The expansion kernel against rows of the codebook the reference's
    decode_hyb_batch (src/codes/ref.py:116-128) built from the same LUT."""
    from quant_2bit_b200 import ste
    d = load_golden("l16v2_hyb_T0.3.npz")
    cb = ste.make_hyb_codebook_gpu(d["lut"]).cpu().numpy()
    np.testing.assert_array_equal(cb[d["cb_rows"]], d["cb_at_rows"])


@pytest.mark.parametrize("Q,L", [(1, 4), (9, 8), (9, 16), (12, 16), (15, 16), (9, 20)])
def test_hyb_codebook_shapes(cuda_ok, Q, L):
    from quant_2bit_b200 import ste
    lut = np.random.default_rng(Q * 100 + L).standard_normal((1 << Q, 2)).astype(np.float32)
    got = ste.make_hyb_codebook_gpu(lut, Q=Q, L_bits=L).cpu().numpy()
    np.testing.assert_array_equal(got, hyb_codebook(lut, Q=Q, L=L))


def test_hyb_codebook_errors(cuda_ok):
    from quant_2bit_b200 import ste
    with pytest.raises(AssertionError):
        ste.make_hyb_codebook_gpu(np.zeros((64, 2), np.float32), Q=9)
    with pytest.raises(AssertionError):
        ste.make_hyb_codebook_gpu(np.zeros((1 << 16, 2), np.float32), Q=16)
    with pytest.raises(RuntimeError):
        ste.make_hyb_codebook_gpu(np.zeros((512, 2), np.float32), device="cpu")
