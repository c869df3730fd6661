"""ctypes binding of libbcjr_b200.so (the C ABI in include/bcjr_b200.h).

The product path has no fallback: if the library is missing or fails to
load, every op raises.  Pointers handed to the library come from torch CUDA
tensors; the stream is the caller's current torch stream.
"""
import contextlib
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbcjr_b200.so")

BCJR_OK = 0
BCJR_ERR_BAD_SHAPE = 1
BCJR_ERR_UNSUPPORTED = 2
BCJR_ERR_NULL_POINTER = 3
BCJR_ERR_ALIGNMENT = 4
BCJR_ERR_WORKSPACE = 5
BCJR_ERR_LAUNCH = 6
BCJR_ERR_DEVICE = 7
BCJR_ERR_TIMEOUT = 8
WS_FORWARD, WS_BACKWARD, WS_INTERNALS = 1, 2, 4
# bcjr_set_test_option switches (tests and diagnostics only)
OPT_TEST_DROP_SENDS = 1
OPT_FORCE_GENERIC = 2
OPT_L16_FORWARD_CLUSTER = 3
OPT_L16_BACKWARD_CLUSTER = 4

# Every symbol include/bcjr_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
SIGNATURES = {
    "bcjr_version": ([], _I),
    "bcjr_set_test_option": ([_I, _I], _I),
    "bcjr_set_reserved_sms": ([_I], _I),
    "bcjr_status_string": ([_I], ctypes.c_char_p),
    "bcjr_workspace_bytes": ([_I, _I, _I, _I, _I, _I], _SZ),
    "bcjr_check_shape": ([_I, _I, _I, _I, _I], _I),
    "bcjr_kernel_launches": ([_I, _I, _I, _I, _I, _I], _I),
    "bcjr_fb_forward": ([_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _SZ, _P], _I),
    "bcjr_fb_backward": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _SZ, _P], _I),
    "bcjr_fb_internals": ([_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P], _I),
    "bcjr_ws_status": ([_P, _P], _I),
    "bcjr_fb_forward_noalloc": ([_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P], _I),
    "bcjr_rht_workspace_bytes": ([_I, _I], _SZ),
    "bcjr_rht": ([_P, _P, _P, _I, _I, _I, _P, _P, _SZ, _P], _I),
    "bcjr_rht_tile": ([_P, _P, _P, _I, _I, _P, _P, _P, _P, _SZ, _P], _I),
    "bcjr_untile_irht": ([_P, _P, _P, _I, _I, _P, _P, _P, _SZ, _P], _I),
    "bcjr_viterbi_workspace_bytes": ([_I, _I, _I, _I, _I], _SZ),
    "bcjr_viterbi_launches": ([_I, _I, _I, _I, _I], _I),
    "bcjr_viterbi": ([_P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _SZ, _P], _I),
    "bcjr_hyb_codebook": ([_P, _I, _I, _P, _P], _I),
    "bcjr_probe_mufu": ([_P, _I, ctypes.POINTER(ctypes.c_double), _P], _I),
}

_lib = None


class BcjrError(RuntimeError):
    """A non-zero status from the library."""

    def __init__(self, status, what):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


def load(path=LIB_PATH):
    """Load the shared library once; raise ImportError when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"libbcjr_b200.so not found at {path}; build it with "
            "`python -m quant_2bit_b200.build` (there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def status_string(status):
    return load().bcjr_status_string(int(status)).decode()


def check(status, what):
    if status == BCJR_OK:
        return
    if status == BCJR_ERR_BAD_SHAPE:
        # The reference asserts on shapes (forward_backward.py:206-207).
        raise AssertionError(f"{what}: {status_string(status)}")
    if status == BCJR_ERR_UNSUPPORTED:
        raise ValueError(f"{what}: {status_string(status)}")
    raise BcjrError(status, what)


@contextlib.contextmanager
def test_option(option, value):
    """Set a bcjr_set_test_option switch for the duration of a block (tests
    and diagnostics; the library reads no environment)."""
    lib = load()
    old = lib.bcjr_set_test_option(option, int(value))
    if old < 0:
        raise ValueError(f"unknown test option {option}")
    try:
        yield
    finally:
        lib.bcjr_set_test_option(option, old)


@contextlib.contextmanager
def reserved_sms(n):
    """Leave `n` SMs free of the persistent cluster kernels for the duration
    of a block (bcjr_set_reserved_sms), e.g. for collectives that overlap
    them."""
    lib = load()
    old = lib.bcjr_set_reserved_sms(int(n))
    if old < 0:
        raise ValueError(f"reserved SMs must be in 0..64, got {n}")
    try:
        yield
    finally:
        lib.bcjr_set_reserved_sms(old)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def workspace(B, N, L, k, V, flags, device):
    """Allocate the workspace for these entry points (torch caching allocator)."""
    lib = load()
    with torch.cuda.device(device):
        n = lib.bcjr_workspace_bytes(B, N, L, k, V, flags)
    if n == 0:
        check(lib.bcjr_check_shape(B, N, L, k, V) or BCJR_ERR_UNSUPPORTED, "bcjr_workspace_bytes")
    return torch.empty(n, dtype=torch.uint8, device=device)


def measure_mufu_gops(device, iters=8192, repeats=3):
    """Measured MUFU (ex2) throughput of this GPU in Gop/s: the best of
    `repeats` timed launches of bcjr_probe_mufu on the current stream."""
    lib = load()
    out = torch.zeros(1, dtype=torch.float32, device=device)
    ops = ctypes.c_double(0.0)
    stream = torch.cuda.current_stream(device)
    best = None
    for r in range(repeats + 1):          # the first launch warms up
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        check(lib.bcjr_probe_mufu(ptr(out), int(iters), ctypes.byref(ops),
                                  ctypes.c_void_p(stream.cuda_stream)), "bcjr_probe_mufu")
        e1.record(stream)
        e1.synchronize()
        if r:
            g = ops.value / (e0.elapsed_time(e1) / 1e3) / 1e9
            best = g if best is None else max(best, g)
    return best
