import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: long-running")


def hyb_codebook(lut, Q=9, L=16):
    """(2^L, 2) HYB codebook from a (2^Q, 2) LUT: Klimov-Shamir hash x*x + x
    (mod 2^32), LUT row (x >> (15 - Q)) & (2^Q - 1), second component negated
    when bit 15 of the hash is set (the reference's HYB code,
    src/codes/ref.py:99-114, src/qat/ste.py:376-392)."""
    s = np.arange(1 << L, dtype=np.uint64)
    x = (s * s + s) & np.uint64(0xFFFFFFFF)
    idx = ((x >> np.uint64(15 - Q)) & np.uint64((1 << Q) - 1)).astype(np.int64)
    out = np.asarray(lut, dtype=np.float32)[idx].copy()
    flip = (x & np.uint64(1 << 15)) != 0
    out[flip, 1] = -out[flip, 1]
    return out


def load_golden(name):
    """A fixture written by tests/golden/make_golden.py (reference outputs).
    Large codebooks live in shared files (l16_cb.npy, l16v2_cb.npy); a HYB
    fixture carries its LUT, and the codebook is rebuilt from it and checked
    against the reference decoder's rows stored with it."""
    d = dict(np.load(os.path.join(GOLDEN, name)))
    if "cb" not in d and "lut" in d:
        d["cb"] = hyb_codebook(d["lut"])
        if "cb_rows" in d:
            assert np.array_equal(d["cb"][d["cb_rows"]], d["cb_at_rows"])
    elif "cb" not in d:
        shared = "l16v2_cb.npy" if name.startswith("l16v2_") else "l16_cb.npy"
        d["cb"] = np.load(os.path.join(GOLDEN, shared))
    for key in ("L", "k", "V"):
        d[key] = int(d[key])
    if "T" in d:
        d["T"] = float(d["T"])
    return d


def golden_names(pattern):
    return sorted(os.path.basename(p) for p in glob.glob(os.path.join(GOLDEN, pattern)))


def parity_report(ours, ref32, ref64, rtol=1e-4, atol=1e-5):
    """Distances used by every parity test (tolerance of the north star:
    1e-4 relative, 1e-5 absolute).

    * ``vs64``:  elementwise allclose(ours, fp64 reference run, rtol, atol).
    * ``vs32``:  elementwise |ours - ref32| <= atol + rtol |ref32| + |ref32 - ref64|,
      i.e. within tolerance of the reference's fp32 output up to that output's
      own rounding error (which exceeds the tolerance at low T).
    * ``norm32``: max|ours - ref32| / max|ref32| (the metric of the reference's
      own parity scripts, src/tripwires/test_bcjr_triton_parity.py:28,46).
    """
    ours = np.asarray(ours, dtype=np.float64)
    ref32 = np.asarray(ref32, dtype=np.float64)
    ref64 = np.asarray(ref64, dtype=np.float64)
    own = np.abs(ref32 - ref64)
    vs64 = np.abs(ours - ref64) <= atol + rtol * np.abs(ref64)
    vs32 = np.abs(ours - ref32) <= atol + rtol * np.abs(ref32) + own
    norm32 = np.abs(ours - ref32).max() / max(np.abs(ref32).max(), 1e-30)
    return {
        "vs64": bool(vs64.all()),
        "vs32": bool(vs32.all()),
        "norm32": float(norm32),
        "max_err64": float(np.abs(ours - ref64).max()),
        "max_err32": float(np.abs(ours - ref32).max()),
        "ref_own_err": float(own.max()),
    }


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip("needs sm_100")
    return True
