"""BCJR forward-backward on B200: the reference's autograd API over the C ABI.

Drop-in replacements (same names, arguments, return values and assertion
behaviour) for

* ``BcjrForwardBackwardMonolithic`` and ``bcjr_forward_backward_monolithic``
  (src/bcjr/bcjr_monolithic.py:157-262),
* ``bcjr_forward_backward`` (src/bcjr/forward_backward.py:190-232),
* ``build_pred_succ_tables`` (src/bcjr/forward_backward.py:62-86).

Every op runs the sm_100a kernels of libbcjr_b200.so on the caller's current
CUDA stream.  There is no CPU path: CPU tensors raise.  The pred/succ tables
are accepted positionally, as the reference's callers pass them, but the
kernels derive the topology from (L, k, V); only the tables' width (2^kV) is
read, to recover k when the caller does not pass it.
"""
import math

import torch

from . import _lib

L_BITS = 16
K_BITS = 2
V_DIM = 2


def build_pred_succ_tables(L=L_BITS, k=K_BITS, V=V_DIM, device="cuda"):
    """(preds, succs) int64 tables, (2^L, 2^kV) each, as the reference builds
    them (forward_backward.py:62-86):
    preds[s, p] = (p << (L - kV)) | (s >> kV);  succs[s, c] = ((s << kV) | c) & mask."""
    S = 1 << L
    b = k * V
    nb = 1 << b
    mask = S - 1
    s = torch.arange(S, dtype=torch.int64, device=device)
    c = torch.arange(nb, dtype=torch.int64, device=device)
    preds = (c.unsqueeze(0) << (L - b)) | (s >> b).unsqueeze(1)
    succs = ((s.unsqueeze(1) << b) & mask) | c.unsqueeze(0)
    return preds, succs


def _require_cuda(t, name):
    if not (torch.is_tensor(t) and t.is_cuda):
        raise RuntimeError(
            f"quant_2bit_b200: `{name}` must be a CUDA tensor (the B200 kernels "
            "have no CPU fallback)")


def _temperature(T_temp, device):
    """Device fp32 scalar for T (the kernels read T on the device; a python
    float becomes a 0-d tensor as in forward_backward.py:212-213).

    A python number must be positive and finite (ValueError otherwise; the
    reference divides by it unchecked, forward_backward.py:101).  A tensor T
    is not read on the host (that would synchronise): the kernels write NaN
    into every output when the T they read is not positive."""
    if torch.is_tensor(T_temp):
        T = T_temp.detach()
        if T.device != device or T.dtype != torch.float32:
            T = T.to(device=device, dtype=torch.float32)
        return T.reshape(()).contiguous()
    Tf = float(T_temp)
    if not (Tf > 0.0 and math.isfinite(Tf)):
        raise ValueError(f"temperature must be positive and finite, got {T_temp!r}")
    return torch.tensor(Tf, dtype=torch.float32, device=device)


def _infer_L_k_V(sequences, codebook, preds, k):
    S = codebook.shape[0]
    L = int(round(math.log2(S))) if S > 0 else -1
    assert S > 0 and (1 << L) == S, f"codebook rows {S} is not a power of two"
    V = sequences.shape[-1]
    if k is None:
        if preds is not None and torch.is_tensor(preds) and preds.dim() == 2:
            nb = preds.shape[1]
            b = int(round(math.log2(nb)))
            assert (1 << b) == nb and b % V == 0, f"preds width {nb} does not match V={V}"
            k = b // V
        else:
            k = K_BITS
    return L, k, V


def _forward(seq, cb, T, L, k, V, want_logZ=True, out=None):
    B, N, _ = seq.shape
    dev = seq.device
    if out is None:
        soft = torch.empty((B, N, V), dtype=torch.float32, device=dev)
    else:
        assert out.shape == (B, N, V) and out.dtype == torch.float32 and out.is_contiguous() \
            and out.device == dev, "out must be a contiguous float32 (B, N, V) tensor on the input's device"
        soft = out
    logZ = torch.empty((B,), dtype=torch.float32, device=dev) if want_logZ else None
    if B == 0:
        return soft, logZ
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = _lib.workspace(B, N, L, k, V, _lib.WS_FORWARD, dev)
        st = lib.bcjr_fb_forward(_lib.ptr(seq), _lib.ptr(cb), _lib.ptr(T), B, N, L, k, V,
                                 _lib.ptr(soft), _lib.ptr(logZ), _lib.ptr(ws), ws.numel(),
                                 _lib.stream_ptr(dev))
    _lib.check(st, "bcjr_fb_forward")
    return soft, logZ


def _backward(seq, cb, T, soft, grad_soft, L, k, V):
    B, N, _ = seq.shape
    dev = seq.device
    d_seq = torch.empty((B, N, V), dtype=torch.float32, device=dev)
    if B == 0:
        return d_seq
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = _lib.workspace(B, N, L, k, V, _lib.WS_BACKWARD, dev)
        st = lib.bcjr_fb_backward(_lib.ptr(seq), _lib.ptr(cb), _lib.ptr(T), _lib.ptr(soft),
                                  _lib.ptr(grad_soft), B, N, L, k, V, _lib.ptr(d_seq),
                                  _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(st, "bcjr_fb_backward")
    return d_seq


def _internals(seq, cb, T, L, k, V):
    B, N, _ = seq.shape
    dev = seq.device
    S = 1 << L
    P = torch.empty((B, N, S), dtype=torch.float32, device=dev)
    la = torch.empty_like(P)
    lb = torch.empty_like(P)
    if B == 0:
        return P, la, lb
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = _lib.workspace(B, N, L, k, V, _lib.WS_INTERNALS, dev)
        st = lib.bcjr_fb_internals(_lib.ptr(seq), _lib.ptr(cb), _lib.ptr(T), B, N, L, k, V,
                                   _lib.ptr(P), _lib.ptr(la), _lib.ptr(lb),
                                   _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(st, "bcjr_fb_internals")
    return P, la, lb


def _prep(sequences, codebook, T_temp):
    _require_cuda(sequences, "sequences")
    _require_cuda(codebook, "codebook")
    assert sequences.dim() == 3, "sequences must be (B, N, V)"
    seq = sequences.detach().contiguous()
    cb = codebook.detach().contiguous()
    T = _temperature(T_temp, seq.device)
    return seq, cb, T


class BcjrForwardBackwardMonolithic(torch.autograd.Function):
    """One autograd node for the whole BCJR forward-backward
    (src/bcjr/bcjr_monolithic.py:157-243).  forward -> soft (B, N, V);
    backward -> (d_sequences, None, None, None, None).  Saves only the inputs
    and the (B, N, V) output, never (B, N, 2^L) tensors."""

    @staticmethod
    def forward(ctx, sequences, codebook, T_temp, preds, succs):
        assert sequences.dtype == torch.float32
        assert codebook.dtype == torch.float32
        L, k, V = _infer_L_k_V(sequences, codebook, preds, None)
        assert codebook.shape == (1 << L, V)
        seq, cb, T = _prep(sequences, codebook, T_temp)
        soft, _ = _forward(seq, cb, T, L, k, V, want_logZ=False)
        ctx.save_for_backward(seq, cb, T, soft)
        ctx.dims = (L, k, V)
        return soft

    @staticmethod
    def backward(ctx, grad_soft):
        seq, cb, T, soft = ctx.saved_tensors
        L, k, V = ctx.dims
        d_seq = _backward(seq, cb, T, soft, grad_soft.contiguous().float(), L, k, V)
        return d_seq, None, None, None, None


class _BcjrSoftLogZ(torch.autograd.Function):
    """(soft, log_Z) with gradients through both, for the eager-compatible
    ``bcjr_forward_backward``.  d log_Z / d w_u = (2/T) sum_s P_u(s) (c(s) - w_u)
    = (2/T) (soft_u - w_u), since the marginals at every step sum to one."""

    @staticmethod
    def forward(ctx, sequences, codebook, T_temp, L, k, V):
        seq, cb, T = _prep(sequences, codebook, T_temp)
        soft, logZ = _forward(seq, cb, T, L, k, V, want_logZ=True)
        ctx.save_for_backward(seq, cb, T, soft)
        ctx.dims = (L, k, V)
        # an output that the loss does not use gets None, not a zero tensor
        # (no eager kernels for an unused log Z)
        ctx.set_materialize_grads(False)
        return soft, logZ

    @staticmethod
    def backward(ctx, grad_soft, grad_logZ):
        seq, cb, T, soft = ctx.saved_tensors
        L, k, V = ctx.dims
        if grad_soft is not None:
            d_seq = _backward(seq, cb, T, soft, grad_soft.contiguous().float(), L, k, V)
        else:
            d_seq = torch.zeros_like(seq)
        if grad_logZ is not None:
            d_seq = d_seq + (2.0 / T) * grad_logZ.view(-1, 1, 1) * (soft - seq)
        return d_seq, None, None, None, None, None


def bcjr_forward_backward(sequences, codebook, T_temp, L=L_BITS, k=K_BITS, V=V_DIM,
                          preds=None, succs=None, return_internals=False):
    """Eager-compatible entry (src/bcjr/forward_backward.py:190-232).

    Returns (soft, log_Z), or (soft, log_Z, P, log_alpha, log_beta) when
    ``return_internals`` (those three are (B, N, 2^L), detached; the
    reference's only consumer, anneal.entropy_diagnostic, runs under no_grad).
    """
    assert sequences.dim() == 3 and sequences.shape[-1] == V
    assert codebook.shape == (1 << L, V)
    soft, logZ = _BcjrSoftLogZ.apply(sequences.float(), codebook.float(), T_temp, L, k, V)
    if return_internals:
        seq, cb, T = _prep(sequences.float(), codebook.float(), T_temp)
        P, la, lb = _internals(seq, cb, T, L, k, V)
        return soft, logZ, P, la, lb
    return soft, logZ


def bcjr_forward_backward_monolithic(sequences, codebook, T_temp, L=L_BITS, k=K_BITS,
                                     V=V_DIM, preds=None, succs=None,
                                     return_internals=False):
    """Drop-in for src/bcjr/bcjr_monolithic.py:246-262: returns (soft, None).

    Unlike the reference (whose Triton kernels hard-code 16 predecessors), any
    (L, k, V) the library supports is accepted; L comes from the codebook and
    k from the tables' width when tables are given."""
    if preds is not None:
        L, k, V = _infer_L_k_V(sequences, codebook, preds, None)
    soft = _MonolithicKV.apply(sequences.float(), codebook.float(), T_temp, L, k, V)
    return soft, None


class _MonolithicKV(torch.autograd.Function):
    """BcjrForwardBackwardMonolithic with explicit (L, k, V)."""

    @staticmethod
    def forward(ctx, sequences, codebook, T_temp, L, k, V):
        assert codebook.shape == (1 << L, V)
        seq, cb, T = _prep(sequences, codebook, T_temp)
        soft, _ = _forward(seq, cb, T, L, k, V, want_logZ=False)
        ctx.save_for_backward(seq, cb, T, soft)
        ctx.dims = (L, k, V)
        return soft

    @staticmethod
    def backward(ctx, grad_soft):
        seq, cb, T, soft = ctx.saved_tensors
        L, k, V = ctx.dims
        d_seq = _backward(seq, cb, T, soft, grad_soft.contiguous().float(), L, k, V)
        return d_seq, None, None, None, None, None


def bcjr_soft_forward(sequences, codebook, T_temp, L, k, V, out=None, want_logZ=True):
    """Forward only, no autograd: (soft, log_Z) for inference-style callers.
    ``out``: a contiguous (B, N, V) float32 tensor to write soft into (for
    instance rows of a larger buffer); log_Z is None unless ``want_logZ``."""
    seq, cb, T = _prep(sequences.float(), codebook.float(), T_temp)
    return _forward(seq, cb, T, L, k, V, want_logZ=want_logZ, out=out)


def bcjr_soft_backward(sequences, codebook, T_temp, soft, grad_soft, L, k, V):
    """Backward only, no autograd: d_sequences for a given upstream gradient."""
    seq, cb, T = _prep(sequences.float(), codebook.float(), T_temp)
    return _backward(seq, cb, T, soft.contiguous(), grad_soft.contiguous().float(), L, k, V)
