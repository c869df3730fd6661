"""Route an imported copy of the reference (quant-2bit's ``src`` package) to
the sm_100a BCJR kernels, so its own callers run unmodified.

    import quant_2bit_b200.hook as hook
    hook.install()          # after `src` is importable

What is replaced (module attributes, looked up by the reference at call time):

* src.bcjr.bcjr_quant._bcjr_chunk_forward and bcjr_quantize_tiles
  (src/bcjr/bcjr_quant.py:63-122): every quantizer call --
  QuantizedLinear._compute_W_q (src/qat/quantized_linear.py:204-211) and so
  every QATDenseDecoderLayer projection -- goes through one launch of
  BcjrForwardBackwardMonolithic;
* src.bcjr.bcjr_quant.bcjr_quantize_weight and the name
  src.qat.quantized_linear imported from it (src/bcjr/bcjr_quant.py:159-178,
  src/qat/quantized_linear.py:41): RHT, RMS scale and tiling on both sides
  of the op run as native kernels;
* the hard quantizer of src.qat.ste (viterbi_encode_chunked,
  quantize_forward_gpu[_no_rht], TrellisQuantSTE[_IP]; src/qat/ste.py:58-356)
  and the names src.qat.quantized_linear and src.bcjr.anneal import from it:
  Viterbi encode, RHT, scale and tiling as native kernels; and
  make_hyb_codebook_gpu (src/qat/ste.py:376-392), the HYB codebook built
  from its LUT by one kernel;
* src.bcjr.bcjr_monolithic.BcjrForwardBackwardMonolithic and
  bcjr_forward_backward_monolithic (src/bcjr/bcjr_monolithic.py:157-262);
* src.bcjr.bcjr_quant.apply_rht_gpu / apply_inverse_rht_gpu and the same
  names in src.qat.ste, when the fast_hadamard_transform extension the
  reference needs is not installed (src/qat/ste.py:34-38, :118).

``uninstall()`` restores the originals.  Nothing here runs on import.
"""
import importlib

from . import bcjr as _bcjr
from . import quant as _quant
from . import ste as _ste

_saved = {}


def _patch(module, name, value):
    if (module.__name__, name) not in _saved:
        _saved[(module.__name__, name)] = (module, getattr(module, name, None))
    setattr(module, name, value)


def install(patch_rht=None):
    """Patch the reference modules; returns the list of patched names."""
    bq = importlib.import_module("src.bcjr.bcjr_quant")
    bm = None
    try:
        bm = importlib.import_module("src.bcjr.bcjr_monolithic")
    except Exception:       # imports triton at module load; optional
        bm = None
    ste = importlib.import_module("src.qat.ste")
    _patch(bq, "_bcjr_chunk_forward", _quant._bcjr_chunk_forward)
    _patch(bq, "bcjr_quantize_tiles", _quant.bcjr_quantize_tiles)
    _patch(bq, "bcjr_quantize_weight", _quant.bcjr_quantize_weight)
    for name in ("viterbi_encode_chunked", "quantize_forward_gpu", "quantize_forward_gpu_no_rht",
                 "TrellisQuantSTE", "TrellisQuantSTE_IP", "make_hyb_codebook_gpu"):
        _patch(ste, name, getattr(_ste, name))
    for modname, names in (("src.qat.quantized_linear",
                            ("bcjr_quantize_weight", "TrellisQuantSTE", "TrellisQuantSTE_IP")),
                           ("src.bcjr.anneal", ("TrellisQuantSTE",))):
        try:
            mod = importlib.import_module(modname)
        except Exception:   # optional: its imports may need packages not present
            continue
        for name in names:
            if hasattr(mod, name):
                _patch(mod, name, getattr(_ste, name, None) or getattr(_quant, name))
    if bm is not None:
        _patch(bm, "BcjrForwardBackwardMonolithic", _bcjr.BcjrForwardBackwardMonolithic)
        _patch(bm, "bcjr_forward_backward_monolithic", _bcjr.bcjr_forward_backward_monolithic)
    if patch_rht is None:
        patch_rht = not getattr(ste, "_HAS_FHT", False)
    if patch_rht:
        for mod in (bq, ste):
            _patch(mod, "apply_rht_gpu", _quant.apply_rht_gpu)
            _patch(mod, "apply_inverse_rht_gpu", _quant.apply_inverse_rht_gpu)
    return sorted(f"{m}.{n}" for (m, n) in _saved)


def uninstall():
    for (_, name), (module, value) in list(_saved.items()):
        setattr(module, name, value)
    _saved.clear()
