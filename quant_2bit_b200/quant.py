"""Caller side of the BCJR op: the reference's quantizer wrapper, routed to the
sm_100a kernels.

Mirrors src/bcjr/bcjr_quant.py (``_bcjr_chunk_forward``, ``bcjr_quantize_tiles``,
``bcjr_quantize_weight_rotated``, ``bcjr_quantize_weight``) and the helpers it
uses from src/qat/ste.py (tiling, GPU RHT) and src/rht/transform.py (sign
vectors), with the same names, arguments and return values, so that
QuantizedLinear-style callers can switch by changing an import.

Differences that do not change results:
* ``chunk_size`` / ``use_checkpoint`` are accepted and ignored: the op keeps
  no per-tile (N, 2^L) buffers (the reference chunks to bound those, and
  checkpoints to drop them), so every tile goes through one launch.
* The randomized Hadamard transform, RMS scale and tiling run as native
  kernels (csrc/bcjr_rht.cu) instead of the un-vendored
  fast_hadamard_transform extension the reference requires
  (src/qat/ste.py:34-38, :118): same unnormalised transform, same 1/sqrt(mn)
  scaling (src/rht/transform.py:65-126), same detached RMS scale and tile
  order.  ``bcjr_quantize_weight`` runs RHT + scale + tile as one call and
  untile + rescale + inverse RHT as another; each is the other's adjoint, so
  their backward passes are the same two calls.
"""
import math

import numpy as np
import torch

from . import _lib
from .bcjr import (K_BITS, L_BITS, V_DIM, BcjrForwardBackwardMonolithic,
                   build_pred_succ_tables)

TX = 16
TY = 16
BCJR_CHUNK = 8


def make_sign_vector(n, seed):
    """Random +-1 vector of length n (src/rht/transform.py:59-62, same RNG)."""
    rng = np.random.default_rng(seed)
    return rng.choice([-1.0, 1.0], size=n).astype(np.float32)


def _rht_args(W, sign_l, sign_r):
    if not (W.is_cuda and sign_l.is_cuda and sign_r.is_cuda):
        raise RuntimeError("the RHT kernels need CUDA tensors (there is no CPU path)")
    assert W.dim() == 2, "W must be (m, n)"
    m, n = W.shape
    for v, name in ((m, "m"), (n, "n")):
        assert v >= 16 and v <= 32768 and v & (v - 1) == 0, \
            f"FWHT length must be a power of 2 in [16, 32768], got {name}={v}"
    assert sign_l.numel() == m and sign_r.numel() == n, "sign vectors must have lengths m and n"
    return (W.detach().float().contiguous(), sign_l.detach().float().contiguous().view(-1),
            sign_r.detach().float().contiguous().view(-1), m, n)


def _rht_ws(m, n, device):
    lib = _lib.load()
    nbytes = lib.bcjr_rht_workspace_bytes(m, n)
    if nbytes == 0:
        raise ValueError(f"unsupported RHT shape ({m}, {n})")
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _rht_call(W, sl, sr, m, n, inverse):
    lib = _lib.load()
    out = torch.empty((m, n), dtype=torch.float32, device=W.device)
    ws = _rht_ws(m, n, W.device)
    P = _lib.ptr
    _lib.check(lib.bcjr_rht(P(W), P(sl), P(sr), m, n, int(inverse), P(out), P(ws), ws.numel(),
                            _lib.stream_ptr(W.device)), "bcjr_rht")
    return out


def _tile_call(W, sl, sr, m, n, mu=None):
    """(seqs (m n / 256, 256), rms) = tile(RHT(W)) * mu; mu = 1 / rms if None."""
    lib = _lib.load()
    seqs = torch.empty((m * n // 256, 256), dtype=torch.float32, device=W.device)
    rms = torch.empty((), dtype=torch.float32, device=W.device)
    ws = _rht_ws(m, n, W.device)
    P = _lib.ptr
    _lib.check(lib.bcjr_rht_tile(P(W), P(sl), P(sr), m, n, P(mu) if mu is not None else None,
                                 P(seqs), P(rms), P(ws), ws.numel(), _lib.stream_ptr(W.device)),
               "bcjr_rht_tile")
    return seqs, rms


def _untile_call(S, sl, sr, m, n, s):
    """RHT^-1(untile(S) * s)."""
    lib = _lib.load()
    out = torch.empty((m, n), dtype=torch.float32, device=S.device)
    ws = _rht_ws(m, n, S.device)
    P = _lib.ptr
    _lib.check(lib.bcjr_untile_irht(P(S), P(sl), P(sr), m, n, P(s), P(out), P(ws), ws.numel(),
                                    _lib.stream_ptr(S.device)), "bcjr_untile_irht")
    return out


class _Rht(torch.autograd.Function):
    """RHT (inverse=False) or its inverse; orthogonal, so each one's backward
    is the other."""

    @staticmethod
    def forward(ctx, W, sign_l, sign_r, inverse):
        Wc, sl, sr, m, n = _rht_args(W, sign_l, sign_r)
        ctx.save_for_backward(sl, sr)
        ctx.inverse = inverse
        return _rht_call(Wc, sl, sr, m, n, inverse)

    @staticmethod
    def backward(ctx, g):
        sl, sr = ctx.saved_tensors
        m, n = g.shape
        return _rht_call(g.float().contiguous(), sl, sr, m, n, not ctx.inverse), None, None, None


class _RhtTile(torch.autograd.Function):
    """(seqs, rms) = (tile(RHT(W)) / rms, rms), rms = RMS(RHT(W)) detached."""

    @staticmethod
    def forward(ctx, W, sign_l, sign_r):
        Wc, sl, sr, m, n = _rht_args(W, sign_l, sign_r)
        seqs, rms = _tile_call(Wc, sl, sr, m, n)
        mu = 1.0 / rms
        ctx.save_for_backward(sl, sr, mu)
        ctx.mn = (m, n)
        ctx.mark_non_differentiable(rms)
        return seqs, rms

    @staticmethod
    def backward(ctx, g_seqs, g_rms):
        sl, sr, mu = ctx.saved_tensors
        m, n = ctx.mn
        return _untile_call(g_seqs.float().contiguous(), sl, sr, m, n, mu), None, None


class _UntileIrht(torch.autograd.Function):
    """W = RHT^-1(untile(S) * s), s a detached device scalar."""

    @staticmethod
    def forward(ctx, S, sign_l, sign_r, s, m, n):
        sl = sign_l.detach().float().contiguous().view(-1)
        sr = sign_r.detach().float().contiguous().view(-1)
        s = s.detach().float().contiguous()
        ctx.save_for_backward(sl, sr, s)
        ctx.mn = (m, n)
        return _untile_call(S.float().contiguous(), sl, sr, m, n, s)

    @staticmethod
    def backward(ctx, g):
        sl, sr, s = ctx.saved_tensors
        m, n = ctx.mn
        seqs, _ = _tile_call(g.float().contiguous(), sl, sr, m, n, mu=s)
        return seqs, None, None, None, None, None


def apply_rht_gpu(W, sign_l, sign_r):
    """W~ = H_m diag(sign_l) W diag(sign_r) H_n / sqrt(mn) (src/qat/ste.py:113-125),
    differentiable."""
    return _Rht.apply(W, sign_l, sign_r, False)


def apply_inverse_rht_gpu(W_tilde, sign_l, sign_r):
    """Inverse of apply_rht_gpu (src/qat/ste.py:128-135), differentiable."""
    return _Rht.apply(W_tilde, sign_l, sign_r, True)


def _tile_for_viterbi_gpu(W, Tx=TX, Ty=TY):
    """(m, n) -> (B, Tx*Ty): sequence j*(m/Tx) + i is the row-major block at
    rows Tx*i.., cols Ty*j.. (src/qat/ste.py:138-149)."""
    m, n = W.shape
    assert m % Tx == 0 and n % Ty == 0
    n_row_blocks, n_col_blocks = m // Tx, n // Ty
    seqs = W.reshape(m, n_col_blocks, Ty).permute(1, 0, 2).reshape(n_col_blocks * n_row_blocks,
                                                                     Tx * Ty)
    return seqs, (n_row_blocks, n_col_blocks)


def _untile_from_viterbi_gpu(recons, shape_info, shape_mn, Tx=TX, Ty=TY):
    """Inverse of _tile_for_viterbi_gpu (src/qat/ste.py:152-159)."""
    n_row_blocks, n_col_blocks = shape_info
    m, n = shape_mn
    return recons.reshape(n_col_blocks, m, Ty).permute(1, 0, 2).reshape(m, n)


def _bcjr_chunk_forward(sequences_chunk, codebook, T_temp, preds, succs):
    """One BCJR call -> soft (B, N, V) (src/bcjr/bcjr_quant.py:63-82)."""
    return BcjrForwardBackwardMonolithic.apply(sequences_chunk, codebook, T_temp, preds, succs)


def bcjr_quantize_tiles(sequences, codebook, T_temp, preds, succs,
                        chunk_size=BCJR_CHUNK, use_checkpoint=True):
    """BCJR over all (B, N, V) tiles in one launch (src/bcjr/bcjr_quant.py:85-122;
    chunk_size and use_checkpoint accepted for compatibility)."""
    return _bcjr_chunk_forward(sequences.float().contiguous(), codebook.float().contiguous(),
                               T_temp, preds, succs)


def bcjr_quantize_weight_rotated(W_rotated, codebook, T_temp, preds, succs,
                                 chunk_size=BCJR_CHUNK, Tx=TX, Ty=TY):
    """RMS-scale (detached), tile, BCJR, untile, rescale
    (src/bcjr/bcjr_quant.py:125-156)."""
    m, n = W_rotated.shape
    V = codebook.shape[1]
    W_scale = W_rotated.detach().pow(2).mean().sqrt().clamp(min=1e-30)
    W_unit = W_rotated / W_scale
    seqs_flat, shape_info = _tile_for_viterbi_gpu(W_unit, Tx=Tx, Ty=Ty)
    B, T_seq = seqs_flat.shape
    sequences = seqs_flat.reshape(B, T_seq // V, V)
    soft = bcjr_quantize_tiles(sequences, codebook, T_temp, preds, succs, chunk_size=chunk_size)
    W_q_unit = _untile_from_viterbi_gpu(soft.reshape(B, T_seq), shape_info, (m, n), Tx, Ty)
    return W_q_unit * W_scale


def bcjr_quantize_weight(W_latent, sign_l, sign_r, codebook, T_temp, preds=None, succs=None,
                         chunk_size=BCJR_CHUNK, Tx=TX, Ty=TY):
    """RHT, BCJR quantize, inverse RHT (src/bcjr/bcjr_quant.py:159-178).  The
    pred/succ tables default to the codebook's trellis (L from its rows, V
    from its columns, k = 2).  With the default 16x16 tiles the RHT, RMS scale
    and tiling run as one native call and the untile, rescale and inverse RHT
    as another."""
    if preds is None or succs is None:
        L = int(round(math.log2(codebook.shape[0])))
        preds, succs = build_pred_succ_tables(L=L, k=K_BITS, V=codebook.shape[1],
                                              device=W_latent.device)
    if Tx != TX or Ty != TY:
        W_tilde = apply_rht_gpu(W_latent, sign_l, sign_r)
        W_tilde_q = bcjr_quantize_weight_rotated(W_tilde, codebook, T_temp, preds, succs,
                                                 chunk_size=chunk_size, Tx=Tx, Ty=Ty)
        return apply_inverse_rht_gpu(W_tilde_q, sign_l, sign_r)
    m, n = W_latent.shape
    V = codebook.shape[1]
    seqs, rms = _RhtTile.apply(W_latent, sign_l, sign_r)
    B = seqs.shape[0]
    soft = bcjr_quantize_tiles(seqs.view(B, (TX * TY) // V, V), codebook, T_temp, preds, succs,
                               chunk_size=chunk_size)
    return _UntileIrht.apply(soft.reshape(B, TX * TY), sign_l, sign_r, rms, m, n)


def bcjr_quantize_layer(weights, signs_l, signs_r, codebook, T_temp, preds=None, succs=None):
    """bcjr_quantize_weight for several weights at once (e.g. the 7 projections
    of a decoder layer, or the experts of an MoE layer), with one BCJR launch
    per direction for all their tiles: each weight is rotated, scaled and
    tiled by itself (its own RMS scale and sign vectors, as
    bcjr_quantize_weight does), the tiles of all weights go through the op
    together, and each weight is untiled and rotated back.  Returns the list
    of quantized weights; gradients flow to every weight."""
    assert len(weights) == len(signs_l) == len(signs_r)
    if preds is None or succs is None:
        L = int(round(math.log2(codebook.shape[0])))
        preds, succs = build_pred_succ_tables(L=L, k=K_BITS, V=codebook.shape[1],
                                              device=weights[0].device)
    V = codebook.shape[1]
    tiles, scales, counts = [], [], []
    for W, sl, sr in zip(weights, signs_l, signs_r):
        seqs, rms = _RhtTile.apply(W, sl, sr)
        tiles.append(seqs)
        scales.append(rms)
        counts.append(seqs.shape[0])
    allseq = torch.cat(tiles, dim=0)
    Bt = allseq.shape[0]
    soft = bcjr_quantize_tiles(allseq.view(Bt, (TX * TY) // V, V), codebook, T_temp, preds, succs)
    out = []
    for part, W, sl, sr, rms in zip(torch.split(soft.reshape(Bt, TX * TY), counts, dim=0), weights,
                                    signs_l, signs_r, scales):
        m, n = W.shape
        out.append(_UntileIrht.apply(part, sl, sr, rms, m, n))
    return out


__all__ = [
    "TX", "TY", "BCJR_CHUNK", "L_BITS", "K_BITS", "V_DIM", "make_sign_vector",
    "apply_rht_gpu", "apply_inverse_rht_gpu", "_tile_for_viterbi_gpu",
    "_untile_from_viterbi_gpu", "_bcjr_chunk_forward", "bcjr_quantize_tiles",
    "bcjr_quantize_weight_rotated", "bcjr_quantize_weight", "bcjr_quantize_layer",
]
