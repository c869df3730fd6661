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

    python tests/golden/make_golden.py --ref <reference root> [--only c1|small|l16|v2|v2sweep|rht|viterbi]
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
        else:
            {"c1": gen_c1, "small": gen_small, "l16": gen_l16, "v2": gen_v2}[what](ref_fb)


if __name__ == "__main__":
    main()
