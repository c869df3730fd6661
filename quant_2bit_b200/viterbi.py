"""Hard (min-sum) Viterbi encoder on the sm_100a kernels.

Mirrors src/viterbi/cuda_kernel.py:147-220 (``viterbi_encode_v_batched_cuda``,
hardcoded there to L=16, k=2, V=2) for any trellis the library builds
(kV <= 4, V <= 2, kV <= L <= 16): L from the codebook's rows, V from its
columns.  Results are bit-identical to the reference's exact-arithmetic
encoder viterbi_encode_v (src/viterbi/encode.py:258-310) on the same inputs.
There is no CPU path: CPU tensors raise.
"""
import math

import numpy as np
import torch

from . import _lib


def viterbi_encode_batched(sequences, codebook, L, k, V):
    """sequences (B, T) fp32 CUDA, T = N V; codebook (2^L, V).
    Returns (bitstreams (B, N) int32, start_states (B,) int32,
    recons (B, T) fp32, mses (B,) fp32)."""
    if not (sequences.is_cuda and codebook.is_cuda):
        raise RuntimeError("the Viterbi kernel needs CUDA tensors (there is no CPU path)")
    assert sequences.dim() == 2, "sequences must be (B, T)"
    assert codebook.shape == (1 << L, V), f"codebook must be ({1 << L}, {V})"
    B, T = sequences.shape
    assert T % V == 0, f"T={T} must be divisible by V={V}"
    N = T // V
    seq = sequences.detach().float().contiguous()
    cb = codebook.detach().float().contiguous()
    dev = seq.device
    bits = torch.empty((B, N), dtype=torch.int32, device=dev)
    starts = torch.empty((B,), dtype=torch.int32, device=dev)
    recons = torch.empty((B, T), dtype=torch.float32, device=dev)
    mses = torch.empty((B,), dtype=torch.float32, device=dev)
    if B == 0:
        return bits, starts, recons, mses
    lib = _lib.load()
    with torch.cuda.device(dev):
        nbytes = lib.bcjr_viterbi_workspace_bytes(B, N, L, k, V)
    if nbytes == 0:
        _lib.check(lib.bcjr_check_shape(B, N, L, k, V) or _lib.BCJR_ERR_UNSUPPORTED,
                   "bcjr_viterbi_workspace_bytes")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    P = _lib.ptr
    _lib.check(lib.bcjr_viterbi(P(seq), P(cb), B, N, L, k, V, P(bits), P(starts), P(recons),
                                P(mses), P(ws), ws.numel(), _lib.stream_ptr(dev)), "bcjr_viterbi")
    return bits, starts, recons, mses


def viterbi_encode_v_batched_cuda(sequences, codebook, k=2):
    """Batched Viterbi encoder (src/viterbi/cuda_kernel.py:147-220): L from
    the codebook's rows, V from its columns, k bits per dimension."""
    L = int(round(math.log2(codebook.shape[0])))
    V = codebook.shape[1] if codebook.dim() == 2 else 1
    return viterbi_encode_batched(sequences, codebook.reshape(1 << L, V), L, k, V)


def viterbi_encode(sequence, L, k, decode_fn, return_trace=False):
    """The V=1 encoder of src/viterbi/encode.py:47-90 (one sequence, numpy in
    and out) on the sm_100a kernels: (bitstream int32 (T,), start_state int,
    recon float32 (T,), mse float), bit-identical to the reference's for a
    float32 sequence (its arithmetic is fp32 then).  decode_fn maps a uint32
    array of states to their codewords, as in the reference.  The per-step
    cost trace (return_trace=True) is not kept by the kernels."""
    if return_trace:
        raise NotImplementedError("return_trace: the kernels keep no per-step cost rows")
    if not torch.cuda.is_available():
        raise RuntimeError("the Viterbi kernel needs a CUDA device (there is no CPU path)")
    states = np.arange(1 << L, dtype=np.uint32)
    cb = torch.tensor(np.asarray(decode_fn(states), dtype=np.float32).reshape(1 << L, 1),
                      device="cuda")
    seq = torch.tensor(np.asarray(sequence, dtype=np.float32).reshape(1, -1), device="cuda")
    bits, starts, recons, mses = viterbi_encode_batched(seq, cb, L, k, 1)
    return (bits[0].cpu().numpy(), int(starts[0]), recons[0].cpu().numpy(), float(mses[0]))


__all__ = ["viterbi_encode", "viterbi_encode_batched", "viterbi_encode_v_batched_cuda"]
