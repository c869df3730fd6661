"""Tile-sharded BCJR across GPUs (one process per GPU, torch.distributed).

Sequences (16x16 weight tiles) are independent in both directions of the
recursion, so rank r of R takes the contiguous range
``[r * B // R, (r + 1) * B // R)`` and computes it with no communication.
Only reassembly needs a collective: the soft codewords of all ranks are
gathered with one ``all_gather_into_tensor`` (NCCL over NVLink on B200; the
reference has no multi-GPU path, src/bcjr/bcjr_quant.py:85-122 only chunks
tiles on one device).  In the reference's tile order (src/qat/ste.py:138-149)
a contiguous range of sequences is a contiguous slab of column blocks of W,
so concatenation in rank order restores the full (B, N, V) tensor.  The
backward gathers d_sequences the same way, for callers whose latent weight is
replicated on every rank.

Shards are padded to ceil(B / R) rows for the collective (all ranks
contribute equal sizes); padded rows are never computed and are dropped on
reassembly.  ``compute`` lets tests substitute a CPU function; the default is
the sm_100a kernels and has no CPU fallback.
"""
import torch
import torch.distributed as dist

from . import bcjr as _bcjr


def shard_range(B, world, rank):
    """Contiguous, balanced range of sequences owned by ``rank``."""
    return (rank * B) // world, ((rank + 1) * B) // world


def _pad_rows(x, rows):
    if x.shape[0] == rows:
        return x.contiguous()
    pad = torch.zeros((rows - x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    return torch.cat([x, pad], 0)


def gather_rows(local, B, group=None):
    """All-gather per-rank row blocks (ragged, contiguous ranges) into (B, ...)."""
    world = dist.get_world_size(group)
    per = -(-B // world)
    buf = torch.empty((per * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(buf, _pad_rows(local, per), group=group)
    parts = []
    for r in range(world):
        lo, hi = shard_range(B, world, r)
        parts.append(buf[r * per: r * per + (hi - lo)])
    return torch.cat(parts, 0)


def _default_forward(seq, cb, T, L, k, V):
    soft, _ = _bcjr.bcjr_soft_forward(seq, cb, T, L, k, V)
    return soft


def _default_backward(seq, cb, T, soft, grad, L, k, V):
    return _bcjr.bcjr_soft_backward(seq, cb, T, soft, grad, L, k, V)


class ShardedBcjr(torch.autograd.Function):
    """soft = BCJR(sequences) with the sequences split across ranks.

    Every rank passes the full (B, N, V) ``sequences`` (replicated latent
    weights, as in data-parallel QAT); each computes its shard, and the full
    soft tensor is all-gathered.  backward: each rank computes d_sequences for
    its shard from its rows of the upstream gradient and the result is
    all-gathered, so every rank ends with the full gradient."""

    @staticmethod
    def forward(ctx, sequences, codebook, T_temp, L, k, V, group, compute):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        B = sequences.shape[0]
        lo, hi = shard_range(B, world, rank)
        fwd = compute[0] if compute else _default_forward
        local = sequences[lo:hi].contiguous()
        soft_local = fwd(local, codebook, T_temp, L, k, V)
        ctx.save_for_backward(local, codebook, soft_local)
        ctx.T = T_temp
        ctx.meta = (L, k, V, group, compute, B, lo, hi)
        return gather_rows(soft_local, B, group)

    @staticmethod
    def backward(ctx, grad_soft):
        local, codebook, soft_local = ctx.saved_tensors
        L, k, V, group, compute, B, lo, hi = ctx.meta
        bwd = compute[1] if compute else _default_backward
        d_local = bwd(local, codebook, ctx.T, soft_local, grad_soft[lo:hi].contiguous(), L, k, V)
        return gather_rows(d_local, B, group), None, None, None, None, None, None, None


def sharded_bcjr(sequences, codebook, T_temp, L=16, k=2, V=1, group=None, compute=None):
    """Sharded soft codewords (B, N, V), identical on every rank."""
    return ShardedBcjr.apply(sequences, codebook, T_temp, L, k, V, group, compute)
