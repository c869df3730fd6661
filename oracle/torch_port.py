"""Torch (CPU) restatement of the reference's eager BCJR path.

TEST INFRASTRUCTURE ONLY: the timed CPU baseline of bench.py (``--impl
reference`` and the ``cpu_baseline`` object) and a cross-check in tests/.
The reference package itself cannot travel to the GPU box, so this module
restates its eager algorithm with the same torch operations in the same
order:

* tables           src/bcjr/forward_backward.py:62-86
* local energy     src/bcjr/forward_backward.py:89-103
* alpha / beta     src/bcjr/forward_backward.py:106-187 (per-step
                   torch.utils.checkpoint when grad is on, :141-153, :173-185)
* log Z, P, soft   src/bcjr/forward_backward.py:219-232
and autograd for the backward, as the reference does.  tests/test_oracle.py
checks that it reproduces the reference's golden outputs.
"""
import torch
import torch.utils.checkpoint as _ckpt


def build_pred_succ_tables(L, k, V, device="cpu"):
    S = 1 << L
    b = k * V
    nb = 1 << b
    mask = S - 1
    s = torch.arange(S, dtype=torch.int64, device=device)
    c = torch.arange(nb, dtype=torch.int64, device=device)
    preds = (c.unsqueeze(0) << (L - b)) | (s >> b).unsqueeze(1)
    succs = ((s.unsqueeze(1) << b) & mask) | c.unsqueeze(0)
    return preds, succs


def _local(seq, cb, T):
    cb_sq = (cb * cb).sum(dim=-1)
    dot = torch.einsum("bnv,sv->bns", seq, cb)
    w_sq = (seq * seq).sum(dim=-1, keepdim=True)
    return -(cb_sq.view(1, 1, -1) - 2.0 * dot + w_sq) / T


def _alpha_step(prev, loc_t, preds):
    return loc_t + torch.logsumexp(prev[:, preds], dim=-1)


def _beta_step(nxt, loc_next, succs):
    return torch.logsumexp(loc_next[:, succs] + nxt[:, succs], dim=-1)


def bcjr_forward_backward(seq, cb, T, L, k, V, use_checkpoint=True):
    """(soft, log_Z) with autograd, as the reference's eager function."""
    preds, succs = build_pred_succ_tables(L, k, V, device=seq.device)
    if not torch.is_tensor(T):
        T = torch.tensor(float(T), dtype=seq.dtype)
    loc = _local(seq, cb, T)
    B, N, S = loc.shape
    ck = use_checkpoint and loc.requires_grad
    a = torch.zeros((B, S), dtype=loc.dtype)
    outs = []
    for t in range(N):
        if ck:
            a = _ckpt.checkpoint(_alpha_step, a, loc[:, t], preds, use_reentrant=False)
        else:
            a = _alpha_step(a, loc[:, t], preds)
        outs.append(a)
    la = torch.stack(outs, dim=1)
    bt = torch.zeros((B, S), dtype=loc.dtype)
    rev = [bt]
    for t in range(N - 2, -1, -1):
        if ck:
            bt = _ckpt.checkpoint(_beta_step, bt, loc[:, t + 1], succs, use_reentrant=False)
        else:
            bt = _beta_step(bt, loc[:, t + 1], succs)
        rev.append(bt)
    lb = torch.stack(rev[::-1], dim=1)
    logZ = torch.logsumexp(la[:, -1], dim=-1)
    P = (la + lb - logZ.view(-1, 1, 1)).exp()
    soft = torch.einsum("bns,sv->bnv", P, cb)
    return soft, logZ


def fwd_bwd(seq, cb, T, L, k, V, grad_soft=None, chunk=8):
    """One forward + backward over ``seq`` in chunks of ``chunk`` sequences
    (the reference default BCJR_CHUNK=8, src/bcjr/bcjr_quant.py:60); upstream
    gradient of ones when ``grad_soft`` is None.  Returns (soft, logZ, d_seq)."""
    softs, lzs, grads = [], [], []
    for i in range(0, seq.shape[0], chunk):
        x = seq[i:i + chunk].detach().clone().requires_grad_(True)
        soft, lz = bcjr_forward_backward(x, cb, T, L, k, V)
        g = torch.ones_like(soft) if grad_soft is None else grad_soft[i:i + chunk]
        (soft * g).sum().backward()
        softs.append(soft.detach())
        lzs.append(lz.detach())
        grads.append(x.grad)
    return torch.cat(softs), torch.cat(lzs), torch.cat(grads)


def internals(seq, cb, T, L, k, V):
    """(P, log_alpha, log_beta), each (B, N, 2^L), exactly as the reference's
    return_internals=True path builds them (forward_backward.py:215-231)."""
    preds, succs = build_pred_succ_tables(L, k, V, device=seq.device)
    if not torch.is_tensor(T):
        T = torch.tensor(float(T), dtype=seq.dtype)
    loc = _local(seq, cb, T)
    B, N, S = loc.shape
    a = torch.zeros((B, S), dtype=loc.dtype)
    outs = []
    for t in range(N):
        a = _alpha_step(a, loc[:, t], preds)
        outs.append(a)
    la = torch.stack(outs, dim=1)
    bt = torch.zeros((B, S), dtype=loc.dtype)
    rev = [bt]
    for t in range(N - 2, -1, -1):
        bt = _beta_step(bt, loc[:, t + 1], succs)
        rev.append(bt)
    lb = torch.stack(rev[::-1], dim=1)
    logZ = torch.logsumexp(la[:, -1], dim=-1)
    P = (la + lb - logZ.view(-1, 1, 1)).exp()
    return P, la, lb


# ---------------------------------------------------------------------------
# Caller side (differentiable torch restatement, for the wrapper's gradient
# checks): randomized Hadamard transform of src/rht/transform.py:24-126 and
# the rotated pipeline of src/bcjr/bcjr_quant.py:125-178.

def fwht(x):
    """Unscaled Walsh-Hadamard transform along the last axis (power of two)."""
    n = x.shape[-1]
    shape = x.shape
    y = x.reshape(-1, n)
    h = 1
    while h < n:
        y = y.reshape(-1, n // (2 * h), 2, h)
        a, b = y[:, :, 0, :], y[:, :, 1, :]
        y = torch.stack((a + b, a - b), dim=2)
        h *= 2
    return y.reshape(shape)


def apply_rht(W, sign_l, sign_r):
    m, n = W.shape
    Wr = fwht(W * sign_r.unsqueeze(0))
    Wl = fwht((Wr * sign_l.unsqueeze(1)).transpose(0, 1)).transpose(0, 1)
    return Wl / (m * n) ** 0.5


def apply_inverse_rht(Wt, sign_l, sign_r):
    m, n = Wt.shape
    Wr = fwht(Wt) * sign_r.unsqueeze(0)
    Wl = fwht(Wr.transpose(0, 1)).transpose(0, 1) * sign_l.unsqueeze(1)
    return Wl / (m * n) ** 0.5
