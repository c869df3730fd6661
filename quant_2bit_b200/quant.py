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
* The randomized Hadamard transform uses a torch fast Walsh-Hadamard
  transform (``fwht``) instead of the un-vendored fast_hadamard_transform
  extension the reference requires (src/qat/ste.py:34-38, :118); same
  unnormalised transform, same 1/sqrt(mn) scaling (src/rht/transform.py:65-126).
"""
import math

import numpy as np
import torch

from .bcjr import (K_BITS, L_BITS, V_DIM, BcjrForwardBackwardMonolithic,
                   build_pred_succ_tables)

TX = 16
TY = 16
BCJR_CHUNK = 8


def make_sign_vector(n, seed):
    """Random +-1 vector of length n (src/rht/transform.py:59-62, same RNG)."""
    rng = np.random.default_rng(seed)
    return rng.choice([-1.0, 1.0], size=n).astype(np.float32)


def fwht(x):
    """Unscaled fast Walsh-Hadamard transform along the last axis (length a
    power of two), in the butterfly order of src/rht/transform.py:26-40."""
    n = x.shape[-1]
    assert n > 0 and (n & (n - 1)) == 0, f"FWHT length must be a power of 2, got {n}"
    shape = x.shape
    y = x.reshape(-1, n)
    h = 1
    while h < n:
        y = y.view(-1, n // (2 * h), 2, h)
        a, b = y[:, :, 0, :], y[:, :, 1, :]
        y = torch.stack((a + b, a - b), dim=2)
        h *= 2
    return y.reshape(shape)


def apply_rht_gpu(W, sign_l, sign_r):
    """W~ = H_m diag(sign_l) W diag(sign_r) H_n / sqrt(mn) (src/qat/ste.py:113-125)."""
    m, n = W.shape
    Wr = fwht(W * sign_r.unsqueeze(0))
    Wl = fwht((Wr * sign_l.unsqueeze(1)).transpose(0, 1).contiguous()).transpose(0, 1)
    return Wl / math.sqrt(m * n)


def apply_inverse_rht_gpu(W_tilde, sign_l, sign_r):
    """Inverse of apply_rht_gpu (src/qat/ste.py:128-135)."""
    m, n = W_tilde.shape
    Wr = fwht(W_tilde) * sign_r.unsqueeze(0)
    Wl = fwht(Wr.transpose(0, 1).contiguous()).transpose(0, 1) * sign_l.unsqueeze(1)
    return Wl / math.sqrt(m * n)


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
    from its columns, k = 2)."""
    if preds is None or succs is None:
        L = int(round(math.log2(codebook.shape[0])))
        preds, succs = build_pred_succ_tables(L=L, k=K_BITS, V=codebook.shape[1],
                                              device=W_latent.device)
    W_tilde = apply_rht_gpu(W_latent, sign_l, sign_r)
    W_tilde_q = bcjr_quantize_weight_rotated(W_tilde, codebook, T_temp, preds, succs,
                                             chunk_size=chunk_size, Tx=Tx, Ty=Ty)
    return apply_inverse_rht_gpu(W_tilde_q, sign_l, sign_r)


__all__ = [
    "TX", "TY", "BCJR_CHUNK", "L_BITS", "K_BITS", "V_DIM", "make_sign_vector", "fwht",
    "apply_rht_gpu", "apply_inverse_rht_gpu", "_tile_for_viterbi_gpu",
    "_untile_from_viterbi_gpu", "_bcjr_chunk_forward", "bcjr_quantize_tiles",
    "bcjr_quantize_weight_rotated", "bcjr_quantize_weight",
]
