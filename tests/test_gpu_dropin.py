"""GPU tests of the caller-level drop-in.

The reference's own QuantizedLinear(quant_mode="bcjr") and
QATDenseDecoderLayer, imported unmodified from the reference's install in
baseline/_ref, run their BCJR quantizer on this library's kernels once
quant_2bit_b200.hook.install() has patched the reference's module attributes
(src/qat/quantized_linear.py:204-211 -> src/bcjr/bcjr_quant.py:159-178;
src/qat/qat_dense_decoder_layer.py:39-55).  The QuantizedLinear result is
checked against a fixture made by the reference's own
bcjr_quantize_weight_rotated on CPU (tests/golden/make_golden.py --only
dropin).  Skipped when the install is absent."""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT, hyb_codebook, parity_report

pytestmark = pytest.mark.gpu
REF = os.path.join(ROOT, "baseline", "_ref")


@pytest.fixture(scope="module")
def reference():
    if not os.path.isdir(os.path.join(REF, "src", "qat")):
        pytest.skip("the reference's install (baseline/_ref) is absent")
    sys.path.insert(0, REF)
    try:
        import src.qat.quantized_linear as ql
        import src.qat.qat_dense_decoder_layer as qdl
        from quant_2bit_b200 import hook
        patched = hook.install()
        yield ql, qdl, patched
        hook.uninstall()
    finally:
        sys.path.remove(REF)


def test_quantized_linear_bcjr_matches_reference_fixture(cuda_ok, reference):
    """QuantizedLinear(32 x 64, HYB (65536, 2) codebook, T_temp a CUDA
    buffer) forward and backward: W_q (its cache), y and W_latent.grad
    elementwise against the reference's fp64 and fp32 results at 1e-4
    relative / 1e-5 absolute."""
    ql, _, patched = reference
    assert "src.qat.quantized_linear.bcjr_quantize_weight" in patched
    d = dict(np.load(os.path.join(GOLDEN, "dropin_qlinear_T0.5.npz")))
    dev = torch.device("cuda")
    cb = torch.tensor(hyb_codebook(d["lut"]), device=dev)
    m, n = int(d["m"]), int(d["n"])
    lin = ql.QuantizedLinear(n, m, cb, seed=int(d["seed"]), quant_mode="bcjr",
                             T_init=float(d["T"]), device="cuda")
    assert lin.T_temp.is_cuda
    np.testing.assert_array_equal(lin.sign_l.cpu().numpy(), d["sign_l"])
    np.testing.assert_array_equal(lin.sign_r.cpu().numpy(), d["sign_r"])
    with torch.no_grad():
        lin.W_latent.copy_(torch.tensor(d["W"]))
        lin.bias.copy_(torch.tensor(d["bias"]))
    y = lin(torch.tensor(d["x"], device=dev))
    (y * torch.tensor(d["gy"], device=dev)).sum().backward()
    torch.cuda.synchronize()
    for ours, key in ((lin._W_q_cache, "Wq"), (y, "y"), (lin.W_latent.grad, "grad")):
        rep = parity_report(ours.detach().cpu().numpy(), d[key + "32"], d[key + "64"])
        assert rep["vs64"], (key, rep)
        assert rep["vs32"], (key, rep)


def test_qat_dense_decoder_layer_runs_on_the_kernels(cuda_ok, reference):
    """A one-layer QATDenseDecoderLayer (tiny Llama config: hidden 64,
    intermediate 128, 2 heads of 32, 1 KV head) with every projection in
    BCJR mode: forward and backward run, every W_latent gets a finite,
    non-zero gradient, and every projection's cached W_q is bitwise this
    library's bcjr_quantize_weight of that projection's own weight."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding
    from quant_2bit_b200 import quant
    _, qdl, _ = reference
    torch.manual_seed(0)
    dev = torch.device("cuda")
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_attention_heads=2,
                      num_key_value_heads=1, head_dim=32, max_position_embeddings=64,
                      attn_implementation="eager")
    layer = LlamaDecoderLayer(cfg, 0).to(dev)
    lut = np.random.default_rng(3).standard_normal((512, 2)).astype(np.float32)
    cb = torch.tensor(hyb_codebook(lut), device=dev)
    qlayer = qdl.QATDenseDecoderLayer(layer, cb, cfg)
    T = 0.5
    for _, lin in qlayer._all_qls():
        lin.set_quant_mode("bcjr")
        lin.set_temperature(T)
    x = torch.randn(2, 8, 64, device=dev)
    pos = torch.arange(8, device=dev)[None].expand(2, -1)
    cos, sin = LlamaRotaryEmbedding(cfg, device=dev)(x, pos)
    out = qlayer(x, position_embeddings=(cos, sin), position_ids=pos)
    out = out[0] if isinstance(out, tuple) else out
    out.pow(2).mean().backward()
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    Tt = torch.tensor(T, device=dev)
    for name, lin in qlayer._all_qls():
        g = lin.W_latent.grad
        assert g is not None and torch.isfinite(g).all() and g.abs().max() > 0, name
        with torch.no_grad():
            Wq = quant.bcjr_quantize_weight(lin.W_latent, lin.sign_l, lin.sign_r, cb, Tt)
        assert torch.equal(Wq, lin._W_q_cache), name
