"""CPU oracle (test infrastructure only; the product never imports it) for the
caller side of the op: randomized Hadamard transform, RMS scale and 16x16
tiling, restated in numpy from the reference:

* Walsh-Hadamard transform, unscaled, butterflies of span h = 1, 2, 4, ...
  (src/rht/transform.py:24-40);
* apply_rht / apply_inverse_rht with the 1/sqrt(mn) scaling
  (src/rht/transform.py:65-126);
* RMS scale clamp(min=1e-30) of the rotated weight
  (src/bcjr/bcjr_quant.py:125-141);
* tile / untile order of _tile_for_viterbi_gpu / _untile_from_viterbi_gpu
  (src/qat/ste.py:138-159).

Pinned against the reference's own outputs in tests/golden/rht.npz.
Computes in float64 unless asked otherwise.
"""
import numpy as np


def fwht(x):
    """Unscaled Walsh-Hadamard transform along the last axis (power of two)."""
    x = np.array(x, dtype=np.float64 if np.asarray(x).dtype != np.float32 else np.float32)
    n = x.shape[-1]
    assert n > 0 and n & (n - 1) == 0, n
    lead = x.shape[:-1]
    h = 1
    while h < n:
        y = x.reshape(lead + (n // (2 * h), 2, h))
        a = y[..., 0, :].copy()
        b = y[..., 1, :].copy()
        y[..., 0, :] = a + b
        y[..., 1, :] = a - b
        x = y.reshape(lead + (n,))
        h *= 2
    return x


def apply_rht(W, sign_l, sign_r, dtype=np.float64):
    """H_m diag(sign_l) W diag(sign_r) H_n / sqrt(m n)."""
    W = np.asarray(W, dtype=dtype)
    m, n = W.shape
    Wr = fwht(W * np.asarray(sign_r, dtype)[None, :])
    Wl = fwht((Wr * np.asarray(sign_l, dtype)[:, None]).T).T
    return Wl / np.sqrt(m * n)


def apply_inverse_rht(Wt, sign_l, sign_r, dtype=np.float64):
    """diag(sign_l) H_m Wt H_n diag(sign_r) / sqrt(m n)."""
    Wt = np.asarray(Wt, dtype=dtype)
    m, n = Wt.shape
    Wr = fwht(Wt) * np.asarray(sign_r, dtype)[None, :]
    Wl = fwht(Wr.T).T * np.asarray(sign_l, dtype)[:, None]
    return Wl / np.sqrt(m * n)


def rms_scale(Wt):
    """max(sqrt(mean(Wt^2)), 1e-30)."""
    return max(float(np.sqrt(np.mean(np.asarray(Wt, np.float64) ** 2))), 1e-30)


def tile(W, Tx=16, Ty=16):
    """(m, n) -> (m n / (Tx Ty), Tx Ty): sequence j (m/Tx) + i holds the
    row-major block at rows Tx i.., cols Ty j.."""
    W = np.asarray(W)
    m, n = W.shape
    out = np.empty(((m // Tx) * (n // Ty), Tx * Ty), dtype=W.dtype)
    for j in range(n // Ty):
        for i in range(m // Tx):
            out[j * (m // Tx) + i] = W[Tx * i:Tx * (i + 1), Ty * j:Ty * (j + 1)].reshape(-1)
    return out


def untile(S, m, n, Tx=16, Ty=16):
    """Inverse of tile."""
    S = np.asarray(S)
    out = np.empty((m, n), dtype=S.dtype)
    for j in range(n // Ty):
        for i in range(m // Tx):
            out[Tx * i:Tx * (i + 1), Ty * j:Ty * (j + 1)] = S[j * (m // Tx) + i].reshape(Tx, Ty)
    return out


def rht_tile(W, sign_l, sign_r, mu=None):
    """(tile(RHT(W)) * mu, rms) with mu = 1 / rms when not given."""
    Wt = apply_rht(W, sign_l, sign_r)
    rms = rms_scale(Wt)
    if mu is None:
        mu = 1.0 / rms
    return tile(Wt * mu), rms


def untile_irht(S, sign_l, sign_r, m, n, s):
    """RHT^-1(untile(S) * s)."""
    return apply_inverse_rht(untile(np.asarray(S, np.float64), m, n) * s, sign_l, sign_r)
