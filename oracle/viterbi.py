"""CPU oracle (test infrastructure only; the product never imports it) for the
hard Viterbi encoder: a vectorised numpy restatement of the reference's
viterbi_encode_v (src/viterbi/encode.py:258-310), batched over sequences.

Same arithmetic as the reference, in float32: d = c - w, local cost
d0*d0 (+ d1*d1), cum_t(s) = min over the 2^kV predecessors of cum_{t-1}
plus local cost, lowest predecessor index on ties, lowest final state on
ties, walk back through the per-state backpointers
preds[s, best] = (best << (L - kV)) | (s >> kV).
Pinned against the reference's own outputs in tests/golden/viterbi_*.npz.
"""
import numpy as np


def viterbi(seqs, cb, L, k, V):
    """seqs (B, N*V), cb (2^L, V) -> (bits (B, N), starts (B,), recons
    (B, N*V), mses (B,)), numpy int32 / float32."""
    seqs = np.asarray(seqs, np.float32)
    cb = np.asarray(cb, np.float32).reshape(1 << L, V)
    B, T = seqs.shape
    N = T // V
    b = k * V
    S, NP = 1 << L, 1 << b
    G = S >> b
    tops = np.arange(S) >> b
    w = seqs.reshape(B, N, V)
    cum = np.zeros((B, S), np.float32)
    best = np.zeros((N, B, G), np.int32)
    for t in range(N):
        local = np.zeros((B, S), np.float32)
        for v in range(V):
            d = cb[None, :, v] - w[:, t, v][:, None]
            local = d * d if v == 0 else local + d * d
        c3 = cum.reshape(B, NP, G)
        best[t] = c3.argmin(axis=1)
        cum = c3.min(axis=1)[:, tops] + local
    final = cum.argmin(axis=1)
    walk = np.zeros((B, N), np.int64)
    walk[:, N - 1] = final
    rows = np.arange(B)
    for t in range(N - 1, 0, -1):
        h = walk[:, t] >> b
        walk[:, t - 1] = (best[t][rows, h].astype(np.int64) << (L - b)) | h
    h0 = walk[:, 0] >> b
    starts = ((best[0][rows, h0].astype(np.int64) << (L - b)) | h0).astype(np.int32)
    bits = (walk & (NP - 1)).astype(np.int32)
    recons = cb[walk].reshape(B, T)
    mses = ((recons.astype(np.float64) - seqs) ** 2).mean(axis=1).astype(np.float32)
    return bits, starts, recons, mses
