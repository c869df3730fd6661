"""Tile-sharded BCJR across GPUs (one process per GPU, torch.distributed).

Sequences (16x16 weight tiles) are independent in both directions of the
recursion, so they are split across ranks and computed with no
communication.  The reference has no multi-GPU path
(src/bcjr/bcjr_quant.py:85-122 only chunks tiles on one device); its callers
quantize the seven weights of a decoder layer one by one
(src/qat/qat_dense_decoder_layer.py:39-55, src/qat/quantized_linear.py:204-211).

Two ways to split, both in ``LayerShards``:

* tiles (default): rank r owns the contiguous range
  ``[r * B_i // R, (r + 1) * B_i // R)`` of every weight i.  In the
  reference's tile order (src/qat/ste.py:138-149) that range is a slab of
  column blocks of W, so an ``all_gather_into_tensor`` of the per-rank slabs,
  in rank order, is the full soft weight (NCCL over NVLink on B200).
* whole weights (``owners``): each weight lives on one rank, e.g. the
  experts of an MoE layer, a few per GPU; nothing is reassembled.

``layer_forward`` launches one forward per weight on the current stream
(largest weights first) and queues that weight's all-gather on a side stream
behind an event, so the gather of weight i overlaps the kernels of the next
weights; ``GatherHandle.wait()`` orders the current stream after the
gathers, with no host synchronisation.  Measured on 2 to 8 B200s, the
gathers of a Llama-3.2-1B layer finish within its forward, so the backward
is best queued after ``wait()``, on all SMs (as ``ShardedLayerBcjr`` does).
The persistent kernels hold every SM they are given, and an NCCL kernel that
waits for SMs on one GPU stalls its peers, so while gathers are in flight
the kernels leave ``GATHER_RESERVED_SMS`` SMs free (bcjr_set_reserved_sms)
and NCCL is capped to as many CTAs (``nccl_options``).

Gradients.  Every rank's loss depends on every soft weight, so the gradient
of the summed loss with respect to rank r's tiles needs the SUM over ranks
of the upstream gradient rows of those tiles (data parallelism: upstream
gradients differ per rank).  ``reduce_rows`` does that with one
reduce-scatter per weight; the owner then runs the backward kernel on its
tiles.  ``grad_reduce=False`` skips it for callers whose upstream gradient is
the same on every rank (a replicated loss).  DDP-style averaging, where
wanted, is a division by the world size afterwards.

Ragged splits are padded to ceil(B / R) rows for the collectives (equal
sizes on every rank); padded rows are never computed and are dropped on
reassembly.  ``compute`` lets tests substitute a CPU function for the
kernels (gloo ranks on CPU); the default is the sm_100a kernels, with no CPU
fallback.
"""
import contextlib

import torch
import torch.distributed as dist

from . import _lib
from . import bcjr as _bcjr

# SMs left free of the cluster kernels while all-gathers overlap them, and the
# CTA cap of the NCCL communicator that runs the gathers.
GATHER_RESERVED_SMS = 8


def nccl_options(max_ctas=GATHER_RESERVED_SMS):
    """ProcessGroupNCCL options whose collectives use at most ``max_ctas``
    CTAs (also for NVLS), so that they fit the SMs the kernels leave free:
    ``dist.init_process_group("nccl", pg_options=nccl_options(), ...)``."""
    opts = dist.ProcessGroupNCCL.Options()
    opts.config.max_ctas = int(max_ctas)
    opts.config.nvls_ctas = int(max_ctas)
    return opts


def _reserve(n, cuda):
    return _lib.reserved_sms(n) if (cuda and n) else contextlib.nullcontext()


def shard_range(B, world, rank):
    """Contiguous, balanced range of sequences owned by ``rank``."""
    return (rank * B) // world, ((rank + 1) * B) // world


class LayerShards:
    """The sequences of each weight of a layer that one rank owns.

    ``counts[i]``: sequences (16x16 tiles) of weight i.  Without ``owners``
    every weight's tiles are split over all ranks (``shard_range``); with
    ``owners[i]`` = the rank that holds weight i, whole weights are assigned.
    The rank's local sequences are its ranges of every weight, concatenated
    in weight order: ``offsets[i]`` is where weight i's range starts."""

    def __init__(self, counts, world, rank, owners=None):
        self.counts = [int(c) for c in counts]
        self.world, self.rank = int(world), int(rank)
        self.owners = None if owners is None else [int(o) for o in owners]
        if self.owners is not None:
            assert len(self.owners) == len(self.counts)
            assert all(0 <= o < self.world for o in self.owners), "owner rank out of range"
        self.ranges, self.offsets = [], []
        off = 0
        for i, c in enumerate(self.counts):
            if self.owners is None:
                lo, hi = shard_range(c, self.world, self.rank)
            else:
                lo, hi = (0, c) if self.owners[i] == self.rank else (0, 0)
            self.ranges.append((lo, hi))
            self.offsets.append(off)
            off += hi - lo
        self.local = off
        self.total = sum(self.counts)

    @property
    def split(self):
        """True when weights are split over ranks (and reassembled by all-gathers)."""
        return self.owners is None and self.world > 1

    def local_slice(self, i):
        lo, hi = self.ranges[i]
        return slice(self.offsets[i], self.offsets[i] + hi - lo)

    def padded(self, i):
        """Rows per rank of weight i in its collectives."""
        return -(-self.counts[i] // self.world)


def _pad_rows(x, rows):
    if x.shape[0] == rows:
        return x.contiguous()
    pad = torch.zeros((rows - x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    return torch.cat([x, pad], 0)


def _unpad(buf, B, world, per):
    if per * world == B:
        return buf
    parts = []
    for r in range(world):
        lo, hi = shard_range(B, world, r)
        parts.append(buf[r * per: r * per + (hi - lo)])
    return torch.cat(parts, 0)


def gather_rows(local, B, group=None):
    """All-gather per-rank row blocks (ragged, contiguous ranges) into (B, ...)."""
    world = dist.get_world_size(group)
    per = -(-B // world)
    buf = torch.empty((per * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(buf, _pad_rows(local, per), group=group)
    return _unpad(buf, B, world, per)


def reduce_rows(full, B, group=None):
    """Sum of ``full`` (B, ...) over ranks, this rank's rows only
    (``shard_range``), by one reduce-scatter."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    per = -(-B // world)
    if per * world == B:
        src = full.contiguous()
    else:
        src = torch.cat([_pad_rows(full[slice(*shard_range(B, world, r))], per)
                         for r in range(world)], 0)
    out = torch.empty((per,) + tuple(full.shape[1:]), dtype=full.dtype, device=full.device)
    dist.reduce_scatter_tensor(out, src, op=dist.ReduceOp.SUM, group=group)
    lo, hi = shard_range(B, world, rank)
    return out[: hi - lo]


def _default_forward(seq, cb, T, L, k, V):
    soft, _ = _bcjr.bcjr_soft_forward(seq, cb, T, L, k, V)
    return soft


def _default_backward(seq, cb, T, soft, grad, L, k, V):
    return _bcjr.bcjr_soft_backward(seq, cb, T, soft, grad, L, k, V)


_side_streams = {}


def _side_stream(device):
    s = _side_streams.get(device.index)
    if s is None:
        s = _side_streams[device.index] = torch.cuda.Stream(device)
    return s


class GatherHandle:
    """Pending per-weight all-gathers of ``layer_forward``.  ``wait()`` makes
    the current stream wait for them (no host sync); ``gathered[i]`` is the
    full soft weight i after that (None for weights not gathered)."""

    def __init__(self, gathered, side, pads):
        self.gathered = gathered
        self._side = side
        self._pads = pads     # (i, buffer, B, world, per) of ragged gathers to compact

    def wait(self):
        if self._side is not None:
            torch.cuda.current_stream(self._side.device).wait_stream(self._side)
            self._side = None
        for i, buf, B, world, per in self._pads:
            self.gathered[i] = _unpad(buf, B, world, per)
        self._pads = []
        return self.gathered


def layer_forward(local_seqs, shards, codebook, T_temp, L=16, k=2, V=1, group=None,
                  gather=True, compute=None, reserve_sms=None):
    """Soft codewords of this rank's sequences, weight by weight.

    Returns ``(soft_local, handle)``: ``soft_local`` is (shards.local, N, V)
    in the order of ``local_seqs``; ``handle.gathered[i]`` becomes the full
    (counts[i], N, V) soft weight i once ``handle.wait()`` has been called
    (split shards with ``gather``; None otherwise).  One kernel launch per
    weight on the current stream, largest first; on CUDA each weight's
    all-gather runs on a side stream after an event recorded behind its
    launch, with ``reserve_sms`` SMs (default ``GATHER_RESERVED_SMS``) left
    free of the kernels for it."""
    assert local_seqs.dim() == 3 and local_seqs.shape[0] == shards.local, \
        "local_seqs must hold this rank's sequences of every weight"
    fwd = compute[0] if compute else None
    B_local, N, _ = local_seqs.shape
    soft_local = torch.empty((B_local, N, V), dtype=torch.float32, device=local_seqs.device)
    do_gather = gather and shards.split
    cuda = local_seqs.is_cuda
    side = _side_stream(local_seqs.device) if (cuda and do_gather) else None
    cur = torch.cuda.current_stream(local_seqs.device) if cuda else None
    gathered = [None] * len(shards.counts)
    pads = []
    if not do_gather:
        # nothing to overlap: one launch for all local sequences (no
        # per-weight tails)
        if B_local > 0:
            if compute:
                soft_local.copy_(fwd(local_seqs, codebook, T_temp, L, k, V))
            else:
                _bcjr.bcjr_soft_forward(local_seqs, codebook, T_temp, L, k, V, out=soft_local,
                                        want_logZ=False)
        return soft_local, GatherHandle(gathered, None, pads)
    if reserve_sms is None:
        reserve_sms = GATHER_RESERVED_SMS
    # largest weights first: the gathers still running at the end are small
    order = sorted(range(len(shards.counts)), key=lambda i: -shards.counts[i])
    for i in order:
        sl = shards.local_slice(i)
        n = sl.stop - sl.start
        if n > 0:
            if compute:
                soft_local[sl] = fwd(local_seqs[sl], codebook, T_temp, L, k, V)
            else:     # the kernel writes straight into this weight's rows
                with _reserve(reserve_sms, cuda):
                    _bcjr.bcjr_soft_forward(local_seqs[sl], codebook, T_temp, L, k, V,
                                            out=soft_local[sl], want_logZ=False)
        B, per = shards.counts[i], shards.padded(i)
        buf = torch.empty((per * shards.world, N, V), dtype=torch.float32, device=local_seqs.device)
        src = soft_local[sl]
        if cuda:
            ev = torch.cuda.Event()
            ev.record(cur)
            side.wait_event(ev)
            with torch.cuda.stream(side):
                dist.all_gather_into_tensor(buf, _pad_rows(src, per), group=group)
            buf.record_stream(side)
        else:
            dist.all_gather_into_tensor(buf, _pad_rows(src, per), group=group)
        if per * shards.world == B:
            gathered[i] = buf
        else:
            pads.append((i, buf, B, shards.world, per))
    if cuda and do_gather:
        soft_local.record_stream(side)
    return soft_local, GatherHandle(gathered, side, pads)


def layer_backward(local_seqs, soft_local, grad_local, codebook, T_temp, L=16, k=2, V=1,
                   compute=None, reserve_sms=0):
    """Gradient with respect to this rank's sequences (one launch for all of
    them), given the upstream gradient rows of the same sequences.  Pass
    ``reserve_sms`` (e.g. ``GATHER_RESERVED_SMS``) when gathers of a
    ``layer_forward`` are still in flight."""
    bwd = compute[1] if compute else _default_backward
    if local_seqs.shape[0] == 0:
        return torch.zeros_like(local_seqs)
    with _reserve(reserve_sms, local_seqs.is_cuda and not compute):
        return bwd(local_seqs, codebook, T_temp, soft_local, grad_local.contiguous(), L, k, V)


def local_grad_rows(grads, shards, group=None, grad_reduce=True):
    """This rank's upstream gradient rows (shards.local, N, V) from the
    per-weight gradients of the full soft weights: summed over ranks by one
    reduce-scatter per weight (``grad_reduce``), or sliced when every rank
    holds the same upstream gradient.  Whole-weight shards take the owned
    weights' gradients as they are."""
    rows = []
    for i, g in enumerate(grads):
        lo, hi = shards.ranges[i]
        if shards.split and grad_reduce:
            # a collective: every rank takes part, also one with no rows of weight i
            r = reduce_rows(g, shards.counts[i], group)
            if hi > lo:
                rows.append(r)
        elif hi == lo:
            continue
        elif shards.split:
            rows.append(g[lo:hi])
        else:
            rows.append(g)
    return torch.cat(rows, 0) if rows else None


class ShardedLayerBcjr(torch.autograd.Function):
    """Soft codewords of every weight of a layer, computed by tile shards.

    Input: this rank's sequences of every weight (``LayerShards`` order).
    Outputs, one per weight: the full (counts[i], N, V) soft weight when
    shards are split over ranks (all-gathered), else the owned weight's soft
    tensor, or an empty (0, N, V) tensor for a weight this rank does not own.
    Backward: the gradient with respect to this rank's sequences (see the
    module docstring for ``grad_reduce``)."""

    @staticmethod
    def forward(ctx, local_seqs, codebook, T_temp, shards, L, k, V, group, grad_reduce, compute):
        seq = local_seqs.detach().contiguous()
        soft_local, handle = layer_forward(seq, shards, codebook, T_temp, L, k, V, group,
                                           gather=True, compute=compute)
        gathered = handle.wait()
        outs = []
        for i in range(len(shards.counts)):
            if shards.split:
                outs.append(gathered[i])
            else:
                outs.append(soft_local[shards.local_slice(i)].clone())
        ctx.save_for_backward(seq, codebook, soft_local)
        ctx.T = T_temp
        ctx.meta = (shards, L, k, V, group, grad_reduce, compute)
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        seq, codebook, soft_local = ctx.saved_tensors
        shards, L, k, V, group, grad_reduce, compute = ctx.meta
        N = seq.shape[1]
        grads = [g if g is not None else torch.zeros((shards.counts[i] if shards.split else
                                                      shards.ranges[i][1] - shards.ranges[i][0], N, V),
                                                     dtype=torch.float32, device=seq.device)
                 for i, g in enumerate(grads)]
        g_local = local_grad_rows(grads, shards, group, grad_reduce)
        if g_local is None:
            d = torch.zeros_like(seq)
        else:
            d = layer_backward(seq, soft_local, g_local.float(), codebook, ctx.T, L, k, V, compute)
        return d, None, None, None, None, None, None, None, None, None


def sharded_bcjr_layer(local_seqs, codebook, T_temp, shards, L=16, k=2, V=1, group=None,
                       grad_reduce=True, compute=None):
    """Per-weight soft codewords of a layer from this rank's tile shards
    (``ShardedLayerBcjr``); a tuple with one tensor per weight."""
    return ShardedLayerBcjr.apply(local_seqs, codebook, T_temp, shards, L, k, V, group,
                                  grad_reduce, compute)


class ShardedBcjr(torch.autograd.Function):
    """soft = BCJR(sequences) of one weight with the sequences split across ranks.

    Every rank passes the full (B, N, V) ``sequences`` (replicated latent
    weights, as in data-parallel QAT); each computes its shard and the full
    soft tensor is all-gathered.  backward: the upstream gradients of all
    ranks are summed onto each shard by a reduce-scatter (``grad_reduce``;
    the gradient of the summed loss), each rank computes d_sequences for its
    shard, and the shards are all-gathered, so every rank ends with the full
    gradient."""

    @staticmethod
    def forward(ctx, sequences, codebook, T_temp, L, k, V, group, compute, grad_reduce):
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        B = sequences.shape[0]
        lo, hi = shard_range(B, world, rank)
        fwd = compute[0] if compute else _default_forward
        local = sequences[lo:hi].detach().contiguous()
        soft_local = fwd(local, codebook, T_temp, L, k, V)
        ctx.save_for_backward(local, codebook, soft_local)
        ctx.T = T_temp
        ctx.meta = (L, k, V, group, compute, B, lo, hi, grad_reduce)
        return gather_rows(soft_local, B, group)

    @staticmethod
    def backward(ctx, grad_soft):
        local, codebook, soft_local = ctx.saved_tensors
        L, k, V, group, compute, B, lo, hi, grad_reduce = ctx.meta
        bwd = compute[1] if compute else _default_backward
        g = reduce_rows(grad_soft, B, group) if grad_reduce else grad_soft[lo:hi]
        d_local = bwd(local, codebook, ctx.T, soft_local, g.contiguous().float(), L, k, V)
        return gather_rows(d_local, B, group), None, None, None, None, None, None, None, None


def sharded_bcjr(sequences, codebook, T_temp, L=16, k=2, V=1, group=None, compute=None,
                 grad_reduce=True):
    """Sharded soft codewords (B, N, V) of one weight, identical on every rank."""
    return ShardedBcjr.apply(sequences, codebook, T_temp, L, k, V, group, compute, grad_reduce)
