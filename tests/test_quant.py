"""Caller-side layer (quant_2bit_b200.quant, .hook): sign vectors and tile
order against the reference's outputs (tests/golden/rht.npz), the hook
against an importable reference checkout, and (GPU) the whole quantizer
wrapper, forward and gradient, against the reference's algorithm restated in
torch on CPU (the native RHT kernels themselves: tests/test_gpu_rht.py)."""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT
from oracle import torch_port


def _rht():
    return dict(np.load(os.path.join(GOLDEN, "rht.npz")))


def test_sign_vectors_match_reference():
    from quant_2bit_b200.quant import make_sign_vector
    d = _rht()
    np.testing.assert_array_equal(make_sign_vector(32, 5), d["sign_l"])
    np.testing.assert_array_equal(make_sign_vector(64, 6), d["sign_r"])


def test_tile_order_matches_reference_and_round_trips():
    from quant_2bit_b200.quant import _tile_for_viterbi_gpu, _untile_from_viterbi_gpu
    d = _rht()
    # the reference tiles in float32 (src/qat/ste.py:96-98)
    Wt = torch.tensor(d["W_rht"].astype(np.float32))
    seqs, info = _tile_for_viterbi_gpu(Wt)
    np.testing.assert_array_equal(seqs.numpy(), d["tiles"])
    assert tuple(info) == tuple(d["info"])
    assert torch.equal(_untile_from_viterbi_gpu(seqs, info, Wt.shape), Wt)


def test_hook_patches_reference_modules():
    # the reference's own package, installed unmodified in baseline/_ref
    ref = os.environ.get("QUANT2BIT_REFERENCE", os.path.join(ROOT, "baseline", "_ref"))
    if not os.path.isdir(os.path.join(ref, "src", "bcjr")):
        pytest.skip("reference install not present")
    sys.path.insert(0, ref)
    try:
        import src.bcjr.bcjr_quant as bq
        import src.qat.ste as ste
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference not importable: {e}")
    import quant_2bit_b200.hook as hook
    from quant_2bit_b200 import quant
    orig = bq._bcjr_chunk_forward
    try:
        names = hook.install()
        assert "src.bcjr.bcjr_quant._bcjr_chunk_forward" in names
        assert "src.bcjr.bcjr_quant.bcjr_quantize_weight" in names
        assert bq._bcjr_chunk_forward is quant._bcjr_chunk_forward
        assert bq.bcjr_quantize_weight is quant.bcjr_quantize_weight
        from quant_2bit_b200 import ste as qste
        assert ste.TrellisQuantSTE is qste.TrellisQuantSTE
        assert ste.viterbi_encode_chunked is qste.viterbi_encode_chunked
        assert ste.make_hyb_codebook_gpu is qste.make_hyb_codebook_gpu
        assert bq.bcjr_quantize_tiles is quant.bcjr_quantize_tiles
        if not getattr(ste, "_HAS_FHT", False):
            assert bq.apply_rht_gpu is quant.apply_rht_gpu
    finally:
        hook.uninstall()
    assert bq._bcjr_chunk_forward is orig


@pytest.mark.gpu
def test_quantize_weight_matches_reference_pipeline(cuda_ok):
    """bcjr_quantize_weight (RHT -> RMS scale -> tile -> BCJR -> untile ->
    inverse RHT) and its gradient, against the same pipeline built on the
    reference's eager BCJR (torch port, fp64, CPU)."""
    from quant_2bit_b200 import quant
    L, k, V, T = 8, 2, 1, 0.6
    rng = np.random.default_rng(3)
    W = rng.standard_normal((32, 64)).astype(np.float32)
    cb = rng.standard_normal((1 << L, V)).astype(np.float32)
    sl, sr = quant.make_sign_vector(32, 1), quant.make_sign_vector(64, 2)
    G = rng.standard_normal((32, 64)).astype(np.float32)

    dev = torch.device("cuda")
    Wd = torch.tensor(W, device=dev, requires_grad=True)
    Wq = quant.bcjr_quantize_weight(Wd, torch.tensor(sl, device=dev), torch.tensor(sr, device=dev),
                                    torch.tensor(cb, device=dev),
                                    torch.tensor(T, device=dev))
    (Wq * torch.tensor(G, device=dev)).sum().backward()

    Wr = torch.tensor(W, dtype=torch.float64, requires_grad=True)
    s_l, s_r = torch.tensor(sl, dtype=torch.float64), torch.tensor(sr, dtype=torch.float64)
    Wt = torch_port.apply_rht(Wr, s_l, s_r)
    scale = Wt.detach().pow(2).mean().sqrt()
    seqs, info = quant._tile_for_viterbi_gpu(Wt / scale)
    soft, _ = torch_port.bcjr_forward_backward(seqs.reshape(seqs.shape[0], -1, V),
                                               torch.tensor(cb, dtype=torch.float64), T, L, k, V)
    Wq_ref = torch_port.apply_inverse_rht(
        quant._untile_from_viterbi_gpu(soft.reshape(seqs.shape), info, W.shape) * scale, s_l, s_r)
    (Wq_ref * torch.tensor(G, dtype=torch.float64)).sum().backward()
    np.testing.assert_allclose(Wq.detach().cpu().numpy(), Wq_ref.detach().numpy(),
                               rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(Wd.grad.cpu().numpy(), Wr.grad.numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
def test_quantize_layer_equals_per_weight(cuda_ok):
    """bcjr_quantize_layer (all weights' tiles in one BCJR launch per direction)
    gives bitwise the results and gradients of bcjr_quantize_weight per weight:
    per-sequence results do not depend on the batch."""
    from quant_2bit_b200 import quant
    rng = np.random.default_rng(8)
    cb = torch.tensor(rng.standard_normal((65536, 2)).astype(np.float32), device="cuda")
    T = torch.tensor(0.4, device="cuda")
    shapes = [(64, 32), (16, 128), (32, 32)]
    Ws = [torch.tensor(rng.standard_normal(s).astype(np.float32), device="cuda") for s in shapes]
    sls = [torch.tensor(quant.make_sign_vector(m, 10 + i), device="cuda") for i, (m, n) in enumerate(shapes)]
    srs = [torch.tensor(quant.make_sign_vector(n, 20 + i), device="cuda") for i, (m, n) in enumerate(shapes)]
    Gs = [torch.tensor(rng.standard_normal(s).astype(np.float32), device="cuda") for s in shapes]
    xs = [W.clone().requires_grad_(True) for W in Ws]
    outs = quant.bcjr_quantize_layer(xs, sls, srs, cb, T)
    sum((o * g).sum() for o, g in zip(outs, Gs)).backward()
    for W, sl, sr, G, o, x in zip(Ws, sls, srs, Gs, outs, xs):
        y = W.clone().requires_grad_(True)
        ref = quant.bcjr_quantize_weight(y, sl, sr, cb, T)
        (ref * G).sum().backward()
        assert torch.equal(o.detach(), ref.detach())
        assert torch.equal(x.grad, y.grad)


def test_python_temperature_must_be_positive_and_finite():
    """A python-number T is checked on the host (ValueError), with no device
    access; a device T is checked by the kernels (NaN outputs)."""
    import torch
    from quant_2bit_b200 import bcjr
    for T in (0.0, -1.0, float("nan"), float("inf"), -0.0):
        with pytest.raises(ValueError):
            bcjr._temperature(T, torch.device("cpu"))
    assert float(bcjr._temperature(0.5, torch.device("cpu"))) == 0.5
