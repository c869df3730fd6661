"""Benchmark: BCJR forward+backward state-transitions/sec on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c3|c5|v2|layer|viterbi|viterbi1] [--temperature T] [--weights gauss|t3]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU, NCCL)

Workload (synthetic, seeded): L=16, k=2, V=1, N=256 steps, T=0.5, codebook
randn(65536) (seed 0), weights randn drawn after the codebook.
* c3 (default): the Llama-3.2-1B-shaped decoder layer, q/o 2048x2048, k/v
  512x2048, gate/up 8192x2048, down 2048x8192 (237,568 sequences, per-row
  scale U[0.5,2]), tile-sharded across the N ranks (strong scaling) through
  quant_2bit_b200.distributed: one forward launch per weight, each weight's
  soft matrix all-gathered over NCCL on a side stream while the next
  weight's kernels run.
* c2: one 1024x1024 weight = 4,096 sequences per GPU (weak scaling: one
  weight of 4,096 N tiles split over the ranks and all-gathered).
* c5: the OLMoE-shaped MoE layer (64 experts x gate/up 1024x2048, down
  2048x1024; 1,572,864 sequences, per-expert scale U[0.5,2]), whole experts
  per GPU (64 / N each, strong scaling; nothing to reassemble).
* v2: the shape the reference's QAT layers use, k=2, V=2 (b = 4, 16
  predecessors per state), N=128: one 1024x1024 weight = 4,096 sequences of
  128 two-dimensional steps per GPU, codebook randn(65536, 2).
* layer: the reference's QAT caller path on one Llama-3.2-1B decoder layer:
  each of its 7 weights (per-row scale U[0.5, 2]) through
  bcjr_quantize_weight (RHT, RMS scale, tile, BCJR at V=2, untile, inverse
  RHT), forward and backward; 237,568 sequences of N=128.  Reports the time
  of the RHT / tiling kernels as well.
* viterbi: hard (min-sum) Viterbi encoding of config v2's sequences (one
  1024x1024 weight per GPU at L=16, k=2, V=2), the reference's
  viterbi_encode_v_batched_cuda; its own metric (min-sum transitions/s).
* viterbi1: the same at V=1 (config c2's 4096 sequences of N=256), the
  reference's viterbi_encode (src/viterbi/encode.py:47-90).

One step = forward (soft) + backward (d_seq for an upstream gradient of ones)
of every local sequence (+ the per-weight all-gathers when N > 1; the
backward runs on each rank's own tiles, whose latent weights it owns, with
that rank's rows of the upstream gradient).  One transition = one trellis
edge: B * N * 2^L * 2^kV per step.

--impl reference: the reference's own eager torch BCJR
(src.bcjr.forward_backward.bcjr_forward_backward, imported unmodified from
baseline/_ref when that install is present, else its restatement
oracle/torch_port.py) on the host's CPU cores, on a bounded sample of the
same workload per step.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "BCJR fwd+bwd state-transitions/sec (L=16,k=2) at 1/2/4/8 B200; % MUFU roofline"
UNIT = "transitions/s"
L, K_BITS, TEMP = 16, 2, 0.5
# (V, N) per config
SHAPES = {"c2": (1, 256), "c3": (1, 256), "c5": (1, 256), "v2": (2, 128), "layer": (2, 128),
          "viterbi": (2, 128), "viterbi1": (1, 256)}
VITERBI_CONFIGS = ("viterbi", "viterbi1")


def viterbi_metric(V):
    return f"Viterbi (min-sum) state-transitions/sec (L=16,k=2,V={V}), 1 B200"
# Algorithmic MUFU (ex2/lg2/rcp) per state-step, forward call and backward
# call: alpha LSE (2^b+1)/2^b + beta LSE (2^b+1)/2^b + marginal exp 1 for the
# forward; the same recompute plus 2/2^b softmax normalisers for the
# backward.  b = 2: 3.5 + 4.0 = 7.5; b = 4: 3.125 + 3.25 = 6.375.
MUFU = {1: (3.5, 4.0), 2: (3.125, 3.25)}
MUFU_PER_SM_CLK = 16
# dram__bytes_read.sum + dram__bytes_write.sum per sequence of the cluster
# kernels, from one ncu capture of a small launch of each (profiles/);
# traffic grows in proportion to sequences.  V=1: L=16, N=256, 296 sequences
# (2-CTA clusters); V=2: L=16, N=128, 297 sequences (part of the history rows
# stays in L2).
DRAM_BYTES_PER_SEQ = {1: {"forward": (4.812766e9 + 4.970556e9) / 296,
                          "backward": (9.551417e9 + 9.918947e9) / 296},
                      2: {"forward": (0.364880e9 + 0.627745e9) / 297,
                          "backward": (0.998954e9 + 1.249169e9) / 297}}
L2_BYTES = 126 * 1024 * 1024


def llama_layer_shapes():
    # q, k, v, o, gate, up, down (out x in), Llama-3.2-1B
    return [(2048, 2048), (512, 2048), (512, 2048), (2048, 2048),
            (8192, 2048), (8192, 2048), (2048, 8192)]


def olmoe_layer_shapes():
    # gate, up, down of each of the 64 experts
    return [(1024, 2048), (1024, 2048), (2048, 1024)] * 64


def layer_shapes(config):
    return llama_layer_shapes() if config in ("c3", "layer") else olmoe_layer_shapes()


def layer_matrix(config, idx):
    """Weight `idx` of a layer workload and its scale, on CPU.

    c3 / layer: the Llama-3.2-1B layer, randn(m, n) times a per-row scale
    U[0.5, 2] (scale drawn first from the matrix's generator, then W).
    c5: the OLMoE layer, randn(m, n) times one scale U[0.5, 2] per expert,
    shared by the expert's gate, up and down weights (matrices 3e .. 3e+2)."""
    m, n = layer_shapes(config)[idx]
    gm = torch.Generator().manual_seed(100 + idx)
    if config in ("c3", "layer"):
        scale = torch.empty(m, 1).uniform_(0.5, 2.0, generator=gm)
    else:
        ge = torch.Generator().manual_seed(5000 + idx // 3)
        scale = torch.empty(1, 1).uniform_(0.5, 2.0, generator=ge)
    return torch.randn(m, n, generator=gm) * scale, scale


def tile(W, Tx=16, Ty=16):
    """Reference tile order (src/qat/ste.py:138-149): sequence j*(m/16)+i holds
    the row-major 16x16 block at rows 16i.., cols 16j.."""
    m, n = W.shape
    return W.view(m, n // Ty, Ty).permute(1, 0, 2).reshape((m // Tx) * (n // Ty), Tx * Ty)


def layer_plan(config, world, rank):
    """How a layer workload is split over the ranks (quant_2bit_b200.distributed.LayerShards):
    c3 splits every weight's tiles evenly; c5 keeps each expert's three
    weights on one rank (64 / world experts per rank)."""
    from quant_2bit_b200.distributed import LayerShards
    counts = [(m // 16) * (n // 16) for m, n in layer_shapes(config)]
    if config == "c5":
        return LayerShards(counts, world, rank, owners=[(i // 3) * world // 64 for i in range(len(counts))])
    return LayerShards(counts, world, rank)


def make_inputs(config, rank, world, weights="gauss"):
    """Codebook (65536, V) and this rank's sequences (B_local, N, V), on CPU,
    and the total sequence count of the job.  For the layer workloads the
    local sequences are this rank's share of every weight (layer_plan), in
    weight order.  weights="t3": config 4's heavy-tailed variant,
    Student-t(3)/sqrt(3) drawn with numpy.random.default_rng(seed) in place of
    the N(0,1) draws."""
    V, NSTEP = SHAPES[config]
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g)
    if config in ("c2", "v2") + VITERBI_CONFIGS:
        gw = torch.Generator().manual_seed(1000 + rank) if rank else g
        w = torch.randn(4096, NSTEP, V, generator=gw)
        if weights == "t3":
            w = torch.tensor(np.random.default_rng(rank).standard_t(3, size=(4096, NSTEP, V))
                             / math.sqrt(3.0), dtype=torch.float32)
        return cb, w, 4096 * world
    plan = layer_plan(config, world, rank)
    seqs = []
    for idx, (lo, hi) in enumerate(plan.ranges):
        if hi > lo:
            W, _ = layer_matrix(config, idx)
            seqs.append(tile(W)[lo:hi])
    w = torch.cat(seqs).view(-1, NSTEP, V).contiguous()
    return cb, w, plan.total


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for nm, val in zip(names, r[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_fb():
    """(fn(seq, cb, T, V) -> None running forward + backward with an
    upstream gradient of ones, kind).  The reference's own eager
    bcjr_forward_backward (src/bcjr/forward_backward.py:190-232), imported
    unmodified from its install in baseline/_ref; without that install, its
    restatement oracle/torch_port.py (bitwise equal on CPU)."""
    if os.path.isdir(os.path.join(REF_DIR, "src", "bcjr")):
        sys.path.insert(0, REF_DIR)
        try:
            from src.bcjr.forward_backward import bcjr_forward_backward as ref
        finally:
            sys.path.remove(REF_DIR)

        def run(seq, cb, T, V):
            x = seq.detach().clone().requires_grad_(True)
            soft, _ = ref(x, cb, float(T), L=L, k=K_BITS, V=V)
            soft.sum().backward()
        return run, "reference"
    from oracle import torch_port

    def run(seq, cb, T, V):
        torch_port.fwd_bwd(seq, cb, T, L, K_BITS, V, chunk=8)
    return run, "port"


def cpu_sample(config, nseq, weights="gauss"):
    """The first `nseq` sequences of the workload (per-sequence cost does not
    depend on the data) and the codebook, on CPU."""
    V, NSTEP = SHAPES[config]
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g)
    if config in ("c3", "c5", "layer"):
        w = tile(layer_matrix(config, 0)[0])[:nseq].reshape(nseq, NSTEP, V).contiguous()
    else:
        w = make_inputs(config, 0, 1, weights)[1][:nseq].contiguous()
    return cb, w


def cpu_reference(args, nseq, steps, warmup):
    """The reference's eager torch BCJR on all the host's CPU cores, in
    chunks of 8 sequences (the reference default BCJR_CHUNK=8,
    src/bcjr/bcjr_quant.py:60): `warmup` untimed steps, then `steps` timed
    steps, each one forward + backward (upstream gradient of ones) of the
    same `nseq`-sequence sample of the workload."""
    if args.config in VITERBI_CONFIGS:
        return cpu_viterbi(args)
    V, NSTEP = SHAPES[args.config]
    edges_per_seq = NSTEP * (1 << L) * (1 << (K_BITS * V))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    run, kind = reference_fb()
    cb, sample = cpu_sample(args.config, nseq, args.weights)

    def one_step(x):
        for i in range(0, x.shape[0], 8):
            run(x[i:i + 8], cb, args.temperature, V)

    warm = sample[:1] if steps == 1 else sample     # a single timed step: a 1-sequence warm-up
    for _ in range(warmup):
        one_step(warm)
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step(sample)
    dt = (time.perf_counter() - t0) / steps
    value = nseq * edges_per_seq / dt
    what = ("the reference's src.bcjr.forward_backward.bcjr_forward_backward (unmodified, "
            "baseline/_ref)" if kind == "reference" else
            "oracle/torch_port.py (the reference's eager ops restated; baseline/_ref absent)")
    return {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "cpu": cpu_model(),
            "sample_sequences": nseq,
            "sample": f"{nseq} sequence(s) of {args.config} (L=16, k=2, V={V}, N={NSTEP}, "
                      f"T={args.temperature:g}), fwd + bwd with grad=ones, chunks of 8, {what}, "
                      f"torch {torch.__version__} CPU, {threads} threads, {warmup} warm-up "
                      f"step(s), {dt:.2f} s per timed step"}


def hbm_peak_gbs():
    """Measured copy bandwidth of this pool's B200s (MEASURED_PEAKS.json),
    else the earlier measurement on this pool (6650 GB/s)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def run_layer(args, rank, world, local_rank):
    """--config layer: bcjr_quantize_weight (RHT, RMS scale, tile, BCJR at V=2,
    untile, inverse RHT), forward and backward, over the 7 weights of one
    Llama-3.2-1B decoder layer; weights assigned round-robin to the ranks."""
    from quant_2bit_b200 import quant
    V, NSTEP = SHAPES["layer"]
    edges_per_seq = NSTEP * (1 << L) * (1 << (K_BITS * V))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=600))
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g).to(dev)
    T = torch.tensor(args.temperature, dtype=torch.float32, device=dev)
    mats = []
    for idx, (m, n) in enumerate(llama_layer_shapes()):
        if idx % world != rank:
            continue
        gm = torch.Generator().manual_seed(100 + idx)
        scale = torch.empty(m, 1).uniform_(0.5, 2.0, generator=gm)
        W = (torch.randn(m, n, generator=gm) * scale).to(dev)
        sl = torch.tensor(quant.make_sign_vector(m, 2 * idx), device=dev)
        sr = torch.tensor(quant.make_sign_vector(n, 2 * idx + 1), device=dev)
        mats.append((W, sl, sr, torch.ones(m, n, device=dev)))
    seqs_local = sum(W.numel() // 256 for W, _, _, _ in mats)
    seqs_total = sum(m * n // 256 for m, n in llama_layer_shapes())
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        # the whole layer: one BCJR launch per direction for all weights' tiles
        xs = [W.detach().requires_grad_(True) for W, _, _, _ in mats]
        outs = quant.bcjr_quantize_layer(xs, [m[1] for m in mats], [m[2] for m in mats], cb, T)
        torch.autograd.backward(outs, [m[3] for m in mats])

    def step_per_weight():
        for W, sl, sr, ones in mats:
            x = W.detach().requires_grad_(True)
            quant.bcjr_quantize_weight(x, sl, sr, cb, T).backward(ones)

    def wrapper_only():
        for W, sl, sr, ones in mats:
            x = W.detach().requires_grad_(True)
            seqs, r = quant._RhtTile.apply(x, sl, sr)
            quant._UntileIrht.apply(seqs, sl, sr, r, *W.shape).backward(ones)

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for e0, e1 in ev:
            flush.zero_()
            e0.record(stream)
            fn()
            e1.record(stream)
        torch.cuda.synchronize()
        return sum(e0.elapsed_time(e1) for e0, e1 in ev)

    for _ in range(args.warmup):
        step()
        wrapper_only()
    torch.cuda.synchronize()
    props = torch.cuda.get_device_properties(dev)
    uuid = getattr(props, "uuid", None)
    clocks = ClockSampler(f"GPU-{uuid}" if uuid is not None else local_rank)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    t_step = timed(step, args.steps)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    t_wrap = timed(wrapper_only, args.steps)
    t_pw = timed(step_per_weight, args.steps)
    tt = torch.tensor([t_step, t_wrap, t_pw], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
    t_step, t_wrap, t_pw = float(tt[0]), float(tt[1]), float(tt[2])
    if rank != 0:
        return
    value = seqs_total * edges_per_seq * args.steps / (t_step / 1e3)
    sms = props.multi_processor_count
    clk_mhz = clk.get("sm_max_mhz") or 1965.0
    from quant_2bit_b200 import _lib
    peak = _lib.measure_mufu_gops(dev)          # measured ex2 throughput of this GPU
    mufu_ops = sum(MUFU[V]) * seqs_total * NSTEP * (1 << L) / world
    bcjr_ms = (t_step - t_wrap) / args.steps
    elems = sum(W.numel() for W, _, _, _ in mats)
    hbm, hbm_kind = hbm_peak_gbs()
    wrap_bytes = 32.0 * elems          # read + write of every weight, 2 ops, fwd + bwd
    wrap_gbs = wrap_bytes / (t_wrap / args.steps / 1e3) / 1e9
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded randn weights with per-row scale U[0.5, 2], randn codebook)",
        "config": {"workload": "layer: bcjr_quantize_layer fwd+bwd over the 7 weights of one "
                               f"Llama-3.2-1B layer (L=16, k=2, V=2, N=128, T={args.temperature:g}), "
                               "one BCJR launch per direction",
                   "sequences_total": seqs_total, "sequences_per_gpu": seqs_local,
                   "l2": "flushed between timed steps (256 MB write, outside the events)",
                   "collective": "none (weights round-robin over ranks)"},
        "clocks": clk,
        # per weight: RHT+tile 5, untile+inverse RHT 5; backward: tile 4,
        # untile+inverse RHT 5; plus one BCJR forward and one backward
        "gpu_launches": (19 * len(mats) + 2) * args.steps,
        "wrapper_ms": {"rht_tile_untile_irht_fwd_bwd": t_wrap / args.steps,
                       "share_of_step": t_wrap / t_step},
        "per_weight_ms_per_step": t_pw / args.steps,
        "roofline": {"bound": "mufu", "kernel": "b4 forward + backward (step minus wrapper)",
                     "achieved": mufu_ops / (bcjr_ms / 1e3) / 1e9, "peak": peak, "unit": "Gop/s",
                     "frac": mufu_ops / (bcjr_ms / 1e3) / 1e9 / peak, "traffic": None},
        "roofline_wrapper": {"bound": "hbm", "achieved": wrap_gbs, "peak": hbm, "unit": "GB/s",
                             "frac": wrap_gbs / hbm, "peak_kind": hbm_kind,
                             "note": "algorithmic bytes: each weight read and written once per op"},
        "e2e": {"value": None, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)


def viterbi_reference():
    """(fn(seqs (B, N V) float32, cb (2^L, V), V) -> None, kind): the
    reference's fastest host encoder, viterbi_encode_v_batched
    (src/viterbi/encode.py:425-470: numpy, local costs by a BLAS matmul),
    imported unmodified from its install in baseline/_ref; without that
    install, the exact-arithmetic restatement oracle/viterbi.py."""
    if os.path.isdir(os.path.join(REF_DIR, "src", "viterbi")):
        sys.path.insert(0, REF_DIR)
        try:
            from src.viterbi.encode import viterbi_encode_v_batched as ref
        finally:
            sys.path.remove(REF_DIR)

        def run(seqs, cb, V):
            ref(seqs, L, K_BITS, V, lambda st: cb[st])
        return run, "reference"
    from oracle import viterbi as ov

    def run(seqs, cb, V):
        ov.viterbi(seqs, cb, L, K_BITS, V)
    return run, "port"


def cpu_viterbi(args):
    """The reference's host Viterbi encoder (viterbi_reference) on a bounded
    sample of the Viterbi config's sequences, on the host cores."""
    V, NSTEP = SHAPES[args.config]
    cb, w, _ = make_inputs(args.config, 0, 1)
    nseq = max(args.cpu_sample_seqs, 4)
    sample = w[:nseq].reshape(nseq, NSTEP * V).numpy()
    cbn = cb.numpy()
    run, kind = viterbi_reference()
    for _ in range(args.warmup if args.impl == "reference" else 1):
        run(sample, cbn, V)
    steps = args.steps if args.impl == "reference" else 1
    t0 = time.perf_counter()
    for _ in range(steps):
        run(sample, cbn, V)
    dt = (time.perf_counter() - t0) / steps
    value = nseq * NSTEP * (1 << L) * (1 << (K_BITS * V)) / dt
    what = ("viterbi_encode_v_batched, unmodified (numpy " + np.__version__ +
            ", BLAS matmul threads up to all host cores)" if kind == "reference"
            else "oracle/viterbi.py (numpy " + np.__version__ + ", one thread)")
    return {"value": value, "unit": UNIT, "cores": (os.cpu_count() or 1) if kind == "reference" else 1,
            "kind": kind, "sample_sequences": nseq, "cpu_model": cpu_model(),
            "sample": f"{nseq} sequences of config {args.config} (L=16, V={V}, N={NSTEP}), "
                      f"{what}, {dt:.2f} s per step"}


def run_viterbi(args, rank, world, local_rank):
    """--config viterbi / viterbi1: one 1024x1024 weight per GPU as 4096
    sequences of 128 two-dimensional steps (V=2) or 256 scalar steps (V=1),
    hard Viterbi encoded (bitstreams, start states, reconstructions, MSEs)."""
    from quant_2bit_b200.viterbi import viterbi_encode_batched
    V, NSTEP = SHAPES[args.config]
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    cb_cpu, w_cpu, _ = make_inputs(args.config, rank, world)
    if args.sequences:
        w_cpu = w_cpu[:args.sequences]
    Bl = w_cpu.shape[0]
    seqs_cpu = w_cpu.reshape(Bl, NSTEP * V).contiguous()
    cb = cb_cpu.to(dev)
    seqs = seqs_cpu.to(dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        viterbi_encode_batched(seqs, cb, L, K_BITS, V)
    torch.cuda.synchronize()
    props = torch.cuda.get_device_properties(dev)
    uuid = getattr(props, "uuid", None)
    clocks = ClockSampler(f"GPU-{uuid}" if uuid is not None else local_rank)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record(stream)
        viterbi_encode_batched(seqs, cb, L, K_BITS, V)
        e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    t_ms = sum(e0.elapsed_time(e1) for e0, e1 in ev)
    from quant_2bit_b200 import _lib
    launches_per_call = _lib.load().bcjr_viterbi_launches(Bl, NSTEP, L, K_BITS, V)
    # e2e: pinned host sequences in, bitstreams and reconstructions out
    host_in = seqs_cpu.pin_memory()
    bits_h = torch.empty((Bl, NSTEP), dtype=torch.int32).pin_memory()
    rec_h = torch.empty((Bl, NSTEP * V)).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        b, st, rec, mse = viterbi_encode_batched(host_in.to(dev, non_blocking=True), cb, L, K_BITS, V)
        bits_h.copy_(b, non_blocking=True)
        rec_h.copy_(rec, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    t_e2e = e0.elapsed_time(e1)
    tt = torch.tensor([t_ms, t_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    t_ms, t_e2e = float(tt[0]), float(tt[1])
    per_seq = NSTEP * (1 << L) * (1 << (K_BITS * V))
    value = Bl * world * per_seq * args.steps / (t_ms / 1e3)
    # issue roofline: per state-step the exact min-sum needs d = c - w and its
    # square per dimension, their sum at V=2, the add of the group minimum
    # (f32x2 instructions: 3 per state at V=2, 1.5 at V=1) and a compare /
    # select for the minimum and its index (2 per state): 5 (V=2) or 3.5
    # (V=1) thread instructions; peak 128 thread instructions per clock per SM
    sms = props.multi_processor_count
    clk_mhz = clk.get("sm_max_mhz") or 1965.0
    inst = 5.0 if V == 2 else 3.5
    ops = inst * Bl * NSTEP * (1 << L) * args.steps
    achieved = ops / (t_ms / 1e3) / 1e9
    peak = sms * 128 * clk_mhz * 1e6 / 1e9
    result = {
        "metric": viterbi_metric(V), "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded randn codebook (65536, {V}) and weights)",
        "config": {"workload": f"{args.config}: one 1024x1024 weight per GPU, {Bl} sequences of "
                               f"N={NSTEP} at L=16, k=2, V={V} (bitstreams, starts, recons, MSEs)",
                   "sequences_per_gpu": Bl, "sequences_total": Bl * world,
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "clocks": clk,
        "gpu_launches": args.steps * launches_per_call,
        "roofline": {"bound": "issue",
                     "kernel": f"vit_b{2 * V}_kernel + walk-back",
                     "achieved": achieved, "peak": peak, "unit": "Ginst/s", "frac": achieved / peak,
                     "traffic": float(Bl * NSTEP * 4096),   # one byte per 4 (V=1) or 16 groups
                     "traffic_unit": "backpointer bytes written per launch",
                     "note": f"{inst:g} algorithmic thread instructions per state-step; "
                             f"peak {sms} SMs x 128/clk x {clk_mhz:.0f} MHz"},
        "e2e": {"value": Bl * world * per_seq * args.steps / (t_e2e / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": host_in.numel() * 4,
                "d2h_bytes_per_step": (bits_h.numel() + rec_h.numel()) * 4},
    }
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_viterbi(args)
    print(json.dumps(result), flush=True)


# FMA-pipe busy cycles per state-step (SM-cycles) of the cluster kernels,
# measured by ncu (sm__pipe_fma_cycles_active.sum over one launch / the
# launch's state-steps; profiles/): the basis of the FP32-issue fraction in
# the bench line, next to the MUFU fraction.
FMA_CYCLES_PER_STATE_STEP = {1: {"forward": 0.0963, "backward": 0.1944},
                             2: {"forward": 0.1349, "backward": 0.2337}}


def run_bcjr(args, rank, world, local_rank):
    """Configs c2 / c3 / c5 / v2: forward + backward of every sequence
    through quant_2bit_b200.distributed (the product's sharding API)."""
    import quant_2bit_b200 as q
    from quant_2bit_b200 import _lib
    from quant_2bit_b200 import distributed as qd

    V, NSTEP = SHAPES[args.config]
    EDGES_PER_SEQ = NSTEP * (1 << L) * (1 << (K_BITS * V))
    STATE_STEPS_PER_SEQ = NSTEP * (1 << L)
    MUFU_FWD, MUFU_BWD = MUFU[V]
    if args.gather_sms is not None:
        qd.GATHER_RESERVED_SMS = args.gather_sms
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        # NCCL capped to the SMs the kernels leave free while gathers overlap them
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300),
                                pg_options=qd.nccl_options(qd.GATHER_RESERVED_SMS))

    cb_cpu, w_cpu, total_seqs = make_inputs(args.config, rank, world, args.weights)
    if args.config in ("c3", "c5") and not args.sequences:
        shards = layer_plan(args.config, world, rank)
    else:
        if args.sequences:
            w_cpu = w_cpu[:args.sequences].contiguous()
        # one weight of (local sequences x world) tiles, split evenly
        shards = qd.LayerShards([w_cpu.shape[0] * world], world, rank)
        total_seqs = shards.total
    assert shards.local == w_cpu.shape[0]
    cb = cb_cpu.to(dev)
    w = w_cpu.to(dev)
    Bl = w.shape[0]
    T = torch.tensor(args.temperature, dtype=torch.float32, device=dev)
    grad = torch.ones((Bl, NSTEP, V), device=dev)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    lib = _lib.load()
    gather = world > 1 and shards.split
    last = {}

    def step(ev=None, do_gather=gather):
        # forward launches (each weight's gather overlapping the next weights'
        # kernels), then the wait for the gathers, then the backward on all SMs
        if ev:
            ev[0].record(stream)
        soft, handle = qd.layer_forward(w, shards, cb, T, L, K_BITS, V, gather=do_gather)
        if ev:
            ev[1].record(stream)
        handle.wait()
        if ev:
            ev[2].record(stream)
        d = qd.layer_backward(w, soft, grad, cb, T, L, K_BITS, V)
        if ev:
            ev[3].record(stream)
        last["soft"], last["d"] = soft, d

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    props = torch.cuda.get_device_properties(dev)
    uuid = getattr(props, "uuid", None)
    clocks = ClockSampler(f"GPU-{uuid}" if uuid is not None else local_rank)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()                     # L2 flush between timed steps (outside the events)
        step(events[i])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    # a failed bounded wait turns the outputs of the call into NaN: a number
    # timed over failed calls is not reported
    bad = (~torch.isfinite(last["soft"])).any() | (~torch.isfinite(last["d"])).any()
    nbad = torch.tensor([float(bad)], dtype=torch.float64, device=dev)

    step_ms = [e[0].elapsed_time(e[3]) for e in events]
    fwd_ms = [e[0].elapsed_time(e[1]) for e in events]
    tail_ms = [e[1].elapsed_time(e[2]) for e in events]     # gathers still running after the forward
    bwd_ms = [e[2].elapsed_time(e[3]) for e in events]
    t = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(nbad, op=dist.ReduceOp.MAX)
    t_max_ms = float(t.item())
    edges_total = total_seqs * EDGES_PER_SEQ
    value = edges_total * args.steps / (t_max_ms / 1e3)

    # the same step without the all-gathers: what the collectives cost
    t_nogather = None
    if gather:
        nsteps = min(args.steps, 3)
        ev2 = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(nsteps)]
        dist.barrier()
        for i in range(nsteps):
            flush.zero_()
            step(ev2[i], do_gather=False)
        torch.cuda.synchronize()
        tn = torch.tensor([sum(e[0].elapsed_time(e[3]) for e in ev2) / nsteps],
                          dtype=torch.float64, device=dev)
        dist.all_reduce(tn, op=dist.ReduceOp.MAX)
        t_nogather = float(tn.item())

    # e2e: the public autograd API (quant_2bit_b200.distributed.sharded_bcjr_layer)
    # with this rank's weights in pinned host memory: H2D of the weights, the
    # per-weight soft matrices (all-gathered), backward with an upstream
    # gradient of ones, D2H of this rank's soft rows and gradient.
    w_host = w_cpu.pin_memory()
    soft_host = torch.empty((Bl, NSTEP, V)).pin_memory()
    dseq_host = torch.empty((Bl, NSTEP, V)).pin_memory()
    e2e_steps = min(args.steps, 3)

    def e2e_step():
        x = w_host.to(dev, non_blocking=True).requires_grad_(True)
        outs = qd.sharded_bcjr_layer(x, cb, T, shards, L, K_BITS, V, grad_reduce=False)
        torch.autograd.backward([o for o in outs if o.shape[0]],
                                [torch.ones_like(o) for o in outs if o.shape[0]])
        rows = [o[lo:hi] if shards.split else o for o, (lo, hi) in zip(outs, shards.ranges)
                if hi > lo]
        soft_host.copy_(torch.cat(rows) if len(rows) > 1 else rows[0], non_blocking=True)
        dseq_host.copy_(x.grad, non_blocking=True)

    e2e_value = None
    if not args.no_e2e:
        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
            dist.barrier()
        e2e_value = edges_total * e2e_steps / (float(te.item()) / 1e3)

    # roofline of the dominant kernel (MUFU-bound; algorithmic ops per launch)
    fwd_avg = sum(fwd_ms) / len(fwd_ms)
    bwd_avg = sum(bwd_ms) / len(bwd_ms)
    sstep = Bl * STATE_STEPS_PER_SEQ
    dom, dom_ms, ops = (("backward", bwd_avg, MUFU_BWD * sstep) if bwd_avg >= fwd_avg
                        else ("forward", fwd_avg, MUFU_FWD * sstep))
    sms = props.multi_processor_count
    clk_mhz = clk.get("sm_max_mhz") or 1965.0
    spec_peak = sms * MUFU_PER_SM_CLK * clk_mhz * 1e6 / 1e9     # Gop/s at max SM clock
    # measured MUFU throughput of this GPU (ex2 probe kernel), the roofline's denominator
    peak = _lib.measure_mufu_gops(dev)
    achieved = ops / (dom_ms / 1e3) / 1e9
    fma = FMA_CYCLES_PER_STATE_STEP[V][dom]
    fp32 = None
    if fma is not None:
        fp32 = {"frac": fma * sstep / (dom_ms / 1e3 * clk_mhz * 1e6 * sms),
                "basis": f"{fma} FMA-pipe busy SM-cycles per state-step (ncu "
                         "sm__pipe_fma_cycles_active, profiles/) x state-steps / "
                         f"(kernel time x {clk_mhz:.0f} MHz x {sms} SMs)"}
    # our kernels per step: one forward call per weight when gathering (else
    # one), one backward call; a call's grids from bcjr_kernel_launches
    n_fwd = len([1 for lo, hi in shards.ranges if hi > lo]) if gather else 1
    launches_per_step = (n_fwd * lib.bcjr_kernel_launches(Bl, NSTEP, L, K_BITS, V, _lib.WS_FORWARD)
                         + lib.bcjr_kernel_launches(Bl, NSTEP, L, K_BITS, V, _lib.WS_BACKWARD))
    names = {"c2": "config 2: one 1024x1024 weight per GPU",
             "c3": "config 3: Llama-3.2-1B decoder layer (q,k,v,o,gate,up,down), tile-sharded",
             "c5": "config 5: OLMoE MoE layer (64 experts), whole experts per GPU",
             "v2": "b=4 (k=2, V=2): one 1024x1024 weight per GPU"}
    result = None
    if rank == 0:
        if gather:
            collective = ("NCCL all_gather_into_tensor per weight on a side stream, each behind "
                          "its weight's forward launch and overlapped with the next weights' "
                          f"kernels, which leave {qd.GATHER_RESERVED_SMS} SMs free (NCCL capped "
                          f"to {qd.GATHER_RESERVED_SMS} CTAs); the backward follows the gathers "
                          "on all SMs")
        else:
            collective = "none"
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max_ms / args.steps,
            "higher_is_better": True, "scaling": "weak" if args.config in ("c2", "v2") else "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded randn codebook and weights of the workload's shapes)",
            "config": {"workload": names[args.config]
                       + f" (L=16, k=2, V={V}, N={NSTEP}, T={args.temperature:g}, {args.weights} weights,"
                         " fwd+bwd, grad=ones)",
                       "sequences_per_gpu": Bl, "sequences_total": total_seqs,
                       "l2": "flushed between timed steps (256 MB write, outside the events); "
                             "inputs larger than L2",
                       "collective": collective},
            "clocks": clk,
            "gpu_launches": launches_per_step * args.steps,
            "kernel_ms": {"forward": fwd_avg, "backward": bwd_avg},
            "roofline": {"bound": "mufu", "kernel": dom, "achieved": achieved, "peak": peak,
                         "unit": "Gop/s", "frac": achieved / peak,
                         "peak_kind": "measured: best of 3 launches of bcjr_probe_mufu (ex2.approx "
                                      "throughput, 8 chains x 1024 threads per SM) on this GPU",
                         "spec_peak": spec_peak, "frac_of_spec": achieved / spec_peak,
                         "traffic": DRAM_BYTES_PER_SEQ[V][dom] * Bl,
                         "traffic_unit": "bytes per launch (ncu capture of a small launch "
                                         "scaled by sequences; see profiles/)",
                         "note": f"algorithmic MUFU ops: {MUFU_FWD}/{MUFU_BWD} per state-step "
                                 f"(fwd/bwd call); spec_peak = {sms} SMs x 16/clk x {clk_mhz:.0f} MHz"},
            "fp32_issue": fp32,
            "e2e": {"value": e2e_value, "unit": UNIT, "steps": e2e_steps,
                    "h2d_bytes_per_step": w_host.numel() * 4,
                    "d2h_bytes_per_step": (soft_host.numel() + dseq_host.numel()) * 4,
                    "api": "quant_2bit_b200.distributed.sharded_bcjr_layer (autograd)"},
        }
        if gather:
            result["gather"] = {"exposed_ms_per_step": sum(tail_ms) / len(tail_ms),
                                "step_ms_without_gathers": t_nogather,
                                "cost_share": 1.0 - t_nogather / (t_max_ms / args.steps),
                                "bytes_received_per_rank": sum(
                                    c - (hi - lo) for c, (lo, hi) in zip(shards.counts, shards.ranges))
                                * NSTEP * V * 4}
        if world > 1:
            result["e2e"]["note"] = "per rank: H2D of its shard, D2H of its soft rows and d_seq"
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if float(nbad.item()) != 0.0:
        print("bench: non-finite outputs after the timed region (a device-side wait gave up or "
              "the inputs are not finite); no number reported", file=sys.stderr, flush=True)
        raise SystemExit(1)
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_reference(args, args.cpu_sample_seqs, 1, 1)
        print(json.dumps(result), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c3",
                    choices=["c2", "c3", "c5", "v2", "layer", "viterbi", "viterbi1"])
    ap.add_argument("--temperature", type=float, default=TEMP,
                    help="T (config 4 sweeps 4, 2, 1, 0.5, 0.25, 0.1, 0.05)")
    ap.add_argument("--weights", default="gauss", choices=["gauss", "t3"],
                    help="config 4's Student-t(3) weights with --config c2")
    ap.add_argument("--cpu-sample-seqs", type=int, default=8,
                    help="sequences of the CPU baseline leg (one reference chunk)")
    ap.add_argument("--ref-sample-seqs", type=int, default=2,
                    help="sequences per step of --impl reference")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sequences", type=int, default=0,
                    help="use only this many sequences per GPU (small cases for ncu)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gather-sms", type=int, default=None,
                    help="SMs left free for the all-gathers at N > 1 (default: "
                         "quant_2bit_b200.distributed.GATHER_RESERVED_SMS)")
    args = ap.parse_args()

    V, NSTEP = SHAPES[args.config]
    EDGES_PER_SEQ = NSTEP * (1 << L) * (1 << (K_BITS * V))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        nsample = args.ref_sample_seqs
        ref = cpu_reference(args, nsample, args.steps, args.warmup)
        nsample = ref.get("sample_sequences", nsample)
        line = {"metric": viterbi_metric(V) if args.config in VITERBI_CONFIGS else METRIC,
                "value": ref["value"], "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": nsample * EDGES_PER_SEQ / ref["value"] * 1e3,
                "higher_is_better": True,
                "scaling": "weak" if args.config in ("c2", "v2") + VITERBI_CONFIGS else "strong",
                "vs_baseline": None,
                "dtype": "f32", "data": "synthetic (seeded randn codebook and weights of the workload's shapes)",
                "impl": "reference",
                "config": {"workload": f"{args.config}: L=16 k=2 V={V} N={NSTEP} "
                                       + ("" if args.config in VITERBI_CONFIGS else f"T={args.temperature:g} ")
                                       + f"{args.weights} weights, CPU sample of {nsample} sequence(s) per step",
                           "sample_sequences": nsample},
                "cpu_baseline": ref,
                "e2e": {"value": ref["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if args.config == "layer":
        run_layer(args, rank, world, local_rank)
    elif args.config in VITERBI_CONFIGS:
        run_viterbi(args, rank, world, local_rank)
    else:
        run_bcjr(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
