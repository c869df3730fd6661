"""CPU tests of the C ABI: the library builds, loads and exports every symbol
that include/bcjr_b200.h declares; host-side validation works without a GPU
(no compute call is made here)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "bcjr_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"BCJR_API\s+[\w\s\*]+?\b(bcjr_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from quant_2bit_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for name in ("bcjr_fb_forward", "bcjr_fb_backward", "bcjr_workspace_bytes",
                 "bcjr_fb_internals", "bcjr_check_shape", "bcjr_status_string"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_python_binding_covers_every_declared_symbol():
    from quant_2bit_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_only_declared_symbols_are_exported():
    """-fvisibility=hidden: the dynamic symbol table holds the C ABI only
    (plus the CUDA runtime's own hidden-by-default internals)."""
    from quant_2bit_b200 import _lib
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH],
                         capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r"\b(bcjr_\w+)\b", out)))
    assert exported == declared_symbols()


def test_shape_validation_without_gpu(lib):
    ok = lib.bcjr_check_shape(4, 256, 16, 2, 1)
    assert ok == 0
    assert lib.bcjr_check_shape(4, 256, 16, 2, 2) == 0           # b = 4
    assert lib.bcjr_check_shape(4, 0, 16, 2, 1) == 1             # N = 0
    assert lib.bcjr_check_shape(-1, 8, 16, 2, 1) == 1            # B < 0
    assert lib.bcjr_check_shape(4, 8, 17, 2, 1) == 2             # L > 16
    assert lib.bcjr_check_shape(4, 8, 3, 2, 2) == 2              # L < kV
    assert lib.bcjr_check_shape(4, 8, 16, 3, 2) == 2             # kV = 6
    assert lib.bcjr_check_shape(0, 8, 16, 2, 1) == 0             # empty batch is valid


def test_viterbi_launch_count_shape_checks(lib):
    """bcjr_viterbi_launches: 0 for an empty batch, a negative status code
    for a shape the encoder does not build (no device work either way)."""
    assert lib.bcjr_viterbi_launches(0, 128, 16, 2, 2) == 0
    assert lib.bcjr_viterbi_launches(4, 0, 16, 2, 1) == -1       # N = 0
    assert lib.bcjr_viterbi_launches(4, 8, 16, 3, 2) == -2       # kV = 6


def test_status_strings(lib):
    for code in range(0, 9):
        assert lib.bcjr_status_string(code).decode()
    assert lib.bcjr_version() >= 100


def test_workspace_query_without_gpu_returns_zero(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert lib.bcjr_workspace_bytes(4, 256, 16, 2, 1, 1) == 0


def test_ops_refuse_cpu_tensors():
    import torch
    from quant_2bit_b200 import bcjr_forward_backward
    w = torch.randn(2, 8, 1)
    cb = torch.randn(256, 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        bcjr_forward_backward(w, cb, 1.0, L=8, k=2, V=1)


def test_test_options_are_set_through_the_abi_not_the_environment(lib):
    """Fault injection and kernel forcing are process-wide switches set by
    bcjr_set_test_option (0 by default); the library reads no environment
    variable on any path (no stray export can change a result)."""
    from quant_2bit_b200 import _lib
    for opt in (_lib.OPT_TEST_DROP_SENDS, _lib.OPT_FORCE_GENERIC, _lib.OPT_L16_FORWARD_CLUSTER,
                _lib.OPT_L16_BACKWARD_CLUSTER):
        assert lib.bcjr_set_test_option(opt, 0) == 0
        with _lib.test_option(opt, 1):
            assert lib.bcjr_set_test_option(opt, 1) == 1
        assert lib.bcjr_set_test_option(opt, 0) == 0
    assert lib.bcjr_set_test_option(0, 1) == -1
    assert lib.bcjr_set_test_option(99, 1) == -1
    csrc = os.path.join(ROOT, "quant_2bit_b200", "csrc")
    for name in os.listdir(csrc):
        text = open(os.path.join(csrc, name)).read()
        assert "getenv" not in text, name


def test_reserved_sms_setter(lib):
    """bcjr_set_reserved_sms: process-wide, 0 by default, 0..64, returns the
    previous value (host-only; no GPU call)."""
    from quant_2bit_b200 import _lib
    assert lib.bcjr_set_reserved_sms(0) == 0
    with _lib.reserved_sms(8):
        assert lib.bcjr_set_reserved_sms(8) == 8
    assert lib.bcjr_set_reserved_sms(0) == 0
    assert lib.bcjr_set_reserved_sms(-1) == -1
    assert lib.bcjr_set_reserved_sms(65) == -1
    with pytest.raises(ValueError):
        with _lib.reserved_sms(100):
            pass
