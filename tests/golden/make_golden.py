"""Generate the golden fixtures in this directory from the reference itself.

Runs only where the reference checkout is importable (pass its root with
--ref; it is not needed by the tests, which read the committed .npz files).
Each fixture holds the inputs and the outputs of the reference's eager
``bcjr_forward_backward`` (src/bcjr/forward_backward.py:190-232) with
autograd backward, run on CPU in float32 (the parity target) and in float64
(the same reference code with float64 tensors, for error attribution).

Input generation follows the benchmark configs: torch.Generator seeded with
``seed``; the codebook is drawn first, then the weights; Student-t weights use
numpy.random.default_rng(seed).standard_t(3) / sqrt(3).

    python tests/golden/make_golden.py --ref <reference root> [--only c1|small|l16|v2|v2sweep|rht|viterbi|c3|c5|dropin]
"""
import argparse
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
T_SWEEP = (4.0, 2.0, 1.0, 0.5, 0.25, 0.1, 0.05)


def run_ref(ref_fb, w, cb, T, L, k, V, grad):
    out = {}
    for tag, dt in (("32", torch.float32), ("64", torch.float64)):
        x = torch.from_numpy(w).to(dt).clone().requires_grad_(True)
        soft, lz = ref_fb(x, torch.from_numpy(cb).to(dt), float(T), L=L, k=k, V=V)
        (soft * torch.from_numpy(grad).to(dt)).sum().backward()
        out["soft" + tag] = soft.detach().numpy()
        out["logZ" + tag] = lz.detach().numpy()
        out["dseq" + tag] = x.grad.numpy()
    return out


def save(name, **arrs):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrs)
    print("wrote", path, flush=True)


def gen_c1(ref_fb):
    # Config 1: L=8, k=2, V=1, N=256, 64 sequences, T=1, grad = ones.
    L, k, V, N, B, T = 8, 2, 1, 256, 64, 1.0
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g).numpy()
    w = torch.randn(B, N, V, generator=g).numpy()
    for tag, grad in (("ones", np.ones_like(w)),
                      ("randgrad", torch.randn(B, N, V, generator=torch.Generator().manual_seed(1)).numpy())):
        out = run_ref(ref_fb, w, cb, T, L, k, V, grad)
        save(f"c1_{tag}.npz", cb=cb, w=w, grad=grad, T=np.float64(T),
             L=L, k=k, V=V, **out)


def gen_small(ref_fb):
    cases = [  # (L, k, V, N, B, T)
        (4, 2, 1, 8, 3, 1.0), (6, 2, 1, 32, 4, 0.5), (6, 1, 1, 20, 3, 0.8),
        (10, 2, 1, 64, 4, 0.5), (8, 2, 2, 32, 4, 1.0), (12, 2, 2, 16, 2, 0.5),
        (9, 3, 1, 24, 3, 0.7), (12, 2, 1, 96, 2, 0.25),
    ]
    for (L, k, V, N, B, T) in cases:
        g = torch.Generator().manual_seed(7 + L + 10 * V + 100 * k)
        cb = torch.randn(1 << L, V, generator=g).numpy()
        w = (1.3 * torch.randn(B, N, V, generator=g)).numpy()
        grad = torch.randn(B, N, V, generator=g).numpy()
        out = run_ref(ref_fb, w, cb, T, L, k, V, grad)
        save(f"small_L{L}_k{k}_V{V}.npz", cb=cb, w=w, grad=grad, T=np.float64(T),
             L=L, k=k, V=V, **out)


def gen_l16(ref_fb, nseq=2):
    # Config 2/4 inputs: codebook randn(65536,1), weights randn(4096,256,1)
    # (first nseq sequences kept), T sweep; plus Student-t(3)/sqrt(3) weights.
    L, k, V, N = 16, 2, 1, 256
    g = torch.Generator().manual_seed(0)
    cb = torch.randn(1 << L, V, generator=g).numpy()
    w_all = torch.randn(4096, N, V, generator=g)
    w_gauss = w_all[:nseq].numpy().copy()
    w_t3 = (np.random.default_rng(0).standard_t(3, size=(nseq, N, V)) / math.sqrt(3.0)).astype(np.float32)
    grad = torch.randn(nseq, N, V, generator=torch.Generator().manual_seed(1)).numpy()
    np.save(os.path.join(HERE, "l16_cb.npy"), cb)
    for dist, w in (("gauss", w_gauss), ("t3", w_t3)):
        for T in T_SWEEP:
            t0 = time.time()
            out = run_ref(ref_fb, w, cb, T, L, k, V, grad)
            save(f"l16_{dist}_T{T:g}.npz", w=w, grad=grad, T=np.float64(T),
                 L=L, k=k, V=V, **out)
            print(f"  {dist} T={T}: {time.time() - t0:.0f}s", flush=True)


def _pick_tiles(scale_rows, m, n, count):
    """Indices (reference tile order, column block 0) of the `count` tiles
    whose 16 rows have the largest mean scale."""
    per_tile = scale_rows.view(m // 16, 16).mean(1)
    return [int(i) for i in torch.argsort(per_tile, descending=True)[:count]]


def gen_layer(ref_fb, config):
    # Configs 3 and 5 as bench.py builds them (bench.layer_matrix): weights
    # scaled by U[0.5, 2] per row (config 3) or per expert (config 5), so
    # |w| reaches ~8 at T = 0.5.  A few tiles with the largest scales, T=0.5,
    # random upstream gradient; `rows` = their indices among all the layer's
    # sequences (weights concatenated in order).
    root = os.path.dirname(os.path.dirname(HERE))
    sys.path.insert(0, root)
    import bench
    L, k, V, N, T = 16, 2, 1, 256, 0.5
    shapes = bench.layer_shapes(config)
    counts = [(m // 16) * (n // 16) for m, n in shapes]
    starts = np.cumsum([0] + counts)
    picks = []   # (weight index, tile index)
    if config == "c3":
        for idx, cnt in ((4, 2), (6, 1)):          # gate (8192 x 2048), down (2048 x 8192)
            m, n = shapes[idx]
            _, scale = bench.layer_matrix(config, idx)
            picks += [(idx, i) for i in _pick_tiles(scale[:, 0], m, n, cnt)]
    else:
        scales = [float(bench.layer_matrix(config, 3 * e)[1]) for e in range(64)]
        e = int(np.argmax(scales))
        picks = [(3 * e, 0), (3 * e + 2, 5)]       # the largest-scale expert's gate and down
    w = np.stack([bench.tile(bench.layer_matrix(config, idx)[0])[i].numpy() for idx, i in picks])
    w = w.reshape(len(picks), N, V).astype(np.float32)
    rows = np.array([starts[idx] + i for idx, i in picks], np.int64)
    g = torch.Generator().manual_seed(31 if config == "c3" else 53)
    cb = torch.randn(1 << L, V, generator=torch.Generator().manual_seed(0)).numpy()
    assert np.array_equal(cb, np.load(os.path.join(HERE, "l16_cb.npy")))
    grad = torch.randn(len(picks), N, V, generator=g).numpy()
    t0 = time.time()
    out = run_ref(ref_fb, w, cb, T, L, k, V, grad)
    save(f"{config}_scaled_T0.5.npz", w=w, grad=grad, T=np.float64(T), L=L, k=k, V=V, rows=rows,
         **out)
    print(f"  {config}: {len(picks)} sequences, max |w| {np.abs(w).max():.2f}, "
          f"{time.time() - t0:.0f}s", flush=True)


def gen_dropin(ref_root):
    # The reference's own QuantizedLinear(quant_mode="bcjr") pipeline
    # (src/qat/quantized_linear.py:204-211 -> src/bcjr/bcjr_quant.py:159-178)
    # on CPU for a 32x64 weight with a HYB codebook at T = 0.5: the RHT as
    # torch matmuls with Sylvester-Hadamard matrices (checked here against the
    # reference's numpy apply_rht / apply_inverse_rht, src/rht/transform.py),
    # the reference's bcjr_quantize_weight_rotated (eager BCJR, chunks of 8
    # with checkpointing), a linear forward with bias, and an upstream
    # gradient; W_q, y and W_latent.grad in fp32 and fp64.
    from src.rht.transform import apply_rht, apply_inverse_rht, make_sign_vector
    from src.bcjr.bcjr_quant import bcjr_quantize_weight_rotated
    from src.bcjr.forward_backward import build_pred_succ_tables
    from src.codes.ref import decode_hyb_batch
    m, n, seed, T = 32, 64, 7, 0.5
    lut = np.random.default_rng(21).standard_normal((512, 2)).astype(np.float32)
    cb = decode_hyb_batch(np.arange(1 << 16, dtype=np.uint32), lut, Q=9).astype(np.float32)
    sl = make_sign_vector(m, seed=seed)          # as QuantizedLinear(seed=7) makes them
    sr = make_sign_vector(n, seed=seed + 1)
    rng = np.random.default_rng(22)
    W = (0.05 * rng.standard_normal((m, n))).astype(np.float32)
    bias = (0.1 * rng.standard_normal(m)).astype(np.float32)
    x = rng.standard_normal((4, n)).astype(np.float32)
    gy = rng.standard_normal((4, m)).astype(np.float32)

    def sylvester(k):
        H = np.ones((1, 1))
        while H.shape[0] < k:
            H = np.block([[H, H], [H, -H]])
        return H

    preds, succs = build_pred_succ_tables(device="cpu")
    out = {}
    for tag, dt in (("32", torch.float32), ("64", torch.float64)):
        Hm, Hn = torch.tensor(sylvester(m), dtype=dt), torch.tensor(sylvester(n), dtype=dt)
        slt, srt = torch.tensor(sl, dtype=dt), torch.tensor(sr, dtype=dt)
        scale = math.sqrt(m * n)
        Wt = torch.tensor(W, dtype=dt, requires_grad=True)
        W_tilde = (Hm @ (slt[:, None] * Wt * srt[None, :]) @ Hn) / scale
        assert np.allclose(W_tilde.detach().numpy(), apply_rht(W.astype(np.float64), sl, sr),
                           rtol=1e-5, atol=1e-6)
        Wq_tilde = bcjr_quantize_weight_rotated(W_tilde, torch.tensor(cb, dtype=dt), float(T),
                                                preds, succs)
        Wq = slt[:, None] * (Hm @ Wq_tilde @ Hn) * srt[None, :] / scale
        assert np.allclose(Wq.detach().numpy(),
                           apply_inverse_rht(Wq_tilde.detach().numpy().astype(np.float64), sl, sr),
                           rtol=1e-5, atol=1e-6)
        y = torch.tensor(x, dtype=dt) @ Wq.T + torch.tensor(bias, dtype=dt)
        (y * torch.tensor(gy, dtype=dt)).sum().backward()
        out["Wq" + tag] = Wq.detach().numpy()
        out["y" + tag] = y.detach().numpy()
        out["grad" + tag] = Wt.grad.numpy()
    save("dropin_qlinear_T0.5.npz", W=W, bias=bias, x=x, gy=gy, lut=lut, sign_l=sl, sign_r=sr,
         seed=seed, T=np.float64(T), m=m, n=n, **out)


def gen_v2(ref_fb):
    # The production drop-in shape: L=16, k=2, V=2 (16 predecessors), N=128.
    L, k, V, N, B, T = 16, 2, 2, 128, 1, 0.5
    g = torch.Generator().manual_seed(3)
    cb = torch.randn(1 << L, V, generator=g).numpy()
    w = torch.randn(B, N, V, generator=g).numpy()
    grad = torch.randn(B, N, V, generator=g).numpy()
    out = run_ref(ref_fb, w, cb, T, L, k, V, grad)
    save("l16_v2.npz", cb=cb, w=w, grad=grad, T=np.float64(T), L=L, k=k, V=V, **out)


def gen_v2sweep(ref_fb, ref_root):
    # b = 4 cluster-kernel cases: L=16, k=2, V=2, N=128, two sequences each;
    # Gaussian codebook (shared file) at three temperatures, Student-t weights,
    # and a HYB codebook built by the reference's decoder from a random LUT.
    from src.codes.ref import decode_hyb_batch
    L, k, V, N, B = 16, 2, 2, 128, 2
    g = torch.Generator().manual_seed(5)
    cb = torch.randn(1 << L, V, generator=g).numpy()
    np.save(os.path.join(HERE, "l16v2_cb.npy"), cb)
    w = torch.randn(B, N, V, generator=g).numpy()
    grad = torch.randn(B, N, V, generator=g).numpy()
    for T in (0.05, 0.25, 2.0):
        out = run_ref(ref_fb, w, cb, T, L, k, V, grad)
        save(f"l16v2_gauss_T{T:g}.npz", w=w, grad=grad, T=np.float64(T), L=L, k=k, V=V, **out)
    w3 = (np.random.default_rng(5).standard_t(3, size=(B, N, V)) / math.sqrt(3.0)).astype(np.float32)
    out = run_ref(ref_fb, w3, cb, 0.5, L, k, V, grad)
    save("l16v2_t3_T0.5.npz", w=w3, grad=grad, T=np.float64(0.5), L=L, k=k, V=V, **out)
    lut = np.random.default_rng(6).standard_normal((512, 2)).astype(np.float32)
    cb_hyb = decode_hyb_batch(np.arange(1 << L, dtype=np.uint32), lut, Q=9)
    rows = np.random.default_rng(7).integers(0, 1 << L, size=256)
    out = run_ref(ref_fb, w, cb_hyb, 0.3, L, k, V, grad)
    save("l16v2_hyb_T0.3.npz", w=w, grad=grad, T=np.float64(0.3), L=L, k=k, V=V, lut=lut,
         cb_rows=rows, cb_at_rows=cb_hyb[rows], **out)


def gen_viterbi(ref_root):
    # Hard Viterbi encodes of the reference's exact-arithmetic encoders
    # (src/viterbi/encode.py:47-90 viterbi_encode, :258-310 viterbi_encode_v),
    # one fixture per trellis: (L, k, V, sequences, steps, codebook kind).
    from src.viterbi.encode import viterbi_encode, viterbi_encode_v
    from src.codes.ref import decode_hyb_batch
    cases = [(16, 2, 2, 4, 128, "hyb"), (16, 2, 2, 3, 128, "gauss"), (16, 2, 1, 3, 256, "gauss"),
             (8, 2, 1, 4, 64, "gauss"), (10, 2, 2, 4, 32, "gauss"), (9, 3, 1, 3, 40, "gauss"),
             (6, 1, 1, 4, 50, "gauss")]
    for (L, k, V, B, N, kind) in cases:
        rng = np.random.default_rng(1000 + 10 * L + V)
        if kind == "hyb":
            lut = rng.standard_normal((512, 2)).astype(np.float32)
            cb = decode_hyb_batch(np.arange(1 << L, dtype=np.uint32), lut, Q=9).astype(np.float32)
        else:
            cb = rng.standard_normal((1 << L, V)).astype(np.float32)
        seqs = rng.standard_normal((B, N * V)).astype(np.float32)
        out = {"bits": [], "starts": [], "recons": [], "mses": []}
        for i in range(B):
            if V == 1:
                bs, ss, rec, mse = viterbi_encode(seqs[i], L=L, k=k, decode_fn=lambda st: cb[st, 0])
            else:
                bs, ss, rec, mse = viterbi_encode_v(seqs[i], L=L, k=k, V=V, decode_fn=lambda st: cb[st])
            out["bits"].append(bs); out["starts"].append(ss)
            out["recons"].append(rec); out["mses"].append(mse)
        extra = {"lut": lut} if kind == "hyb" else {"cb": cb}
        save(f"viterbi_L{L}_k{k}_V{V}_{kind}.npz", seqs=seqs, L=L, k=k, V=V,
             bits=np.array(out["bits"], np.int32), starts=np.array(out["starts"], np.int32),
             recons=np.array(out["recons"], np.float32), mses=np.array(out["mses"], np.float32),
             **extra)


def gen_rht(ref_root):
    # RHT, sign vectors and tile order of the reference's quantizer wrapper
    # (src/rht/transform.py:59-126, src/qat/ste.py:76-110).
    from src.rht.transform import apply_rht, apply_inverse_rht, make_sign_vector
    from src.qat.ste import _tile_for_viterbi
    rng = np.random.default_rng(11)
    W = rng.standard_normal((32, 64)).astype(np.float32)
    sl, sr = make_sign_vector(32, 5), make_sign_vector(64, 6)
    Wt = apply_rht(W, sl, sr)
    Wi = apply_inverse_rht(Wt, sl, sr)
    seqs, info = _tile_for_viterbi(Wt)
    save("rht.npz", W=W, sign_l=sl, sign_r=sr, W_rht=Wt, W_inv=Wi, tiles=seqs,
         info=np.array(info))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference checkout")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from src.bcjr.forward_backward import bcjr_forward_backward as ref_fb
    torch.set_num_threads(os.cpu_count() or 1)
    todo = [args.only] if args.only else ["small", "c1", "v2", "l16", "v2sweep", "rht", "viterbi"]
    for what in todo:
        if what == "rht":
            gen_rht(args.ref)
        elif what == "viterbi":
            gen_viterbi(args.ref)
        elif what == "v2sweep":
            gen_v2sweep(ref_fb, args.ref)
        elif what in ("c3", "c5"):
            gen_layer(ref_fb, what)
        elif what == "dropin":
            gen_dropin(args.ref)
        else:
            {"c1": gen_c1, "small": gen_small, "l16": gen_l16, "v2": gen_v2}[what](ref_fb)


if __name__ == "__main__":
    main()
