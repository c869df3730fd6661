"""Hard-quantizer side of the reference's QAT (src/qat/ste.py), on the native
kernels: the Viterbi encode of the tiles (bcjr_vit_b4.cu / bcjr_viterbi.cu)
between the native RHT + RMS scale + tiling and its inverse (bcjr_rht.cu).

Same names, arguments and results as the reference:
* viterbi_encode_chunked (src/qat/ste.py:58-73): one launch for all tiles
  (the chunk argument is accepted and ignored: the kernel bounds its own
  memory);
* quantize_forward_gpu_no_rht / quantize_forward_gpu (:160-210);
* TrellisQuantSTE / TrellisQuantSTE_IP (:286-356): hard quantization forward,
  straight-through backward;
* make_hyb_codebook_gpu (:376-392), on the native expansion kernel.
The reference needs the fast_hadamard_transform extension on this path and
falls back to numpy on the CPU; here everything runs on the GPU and CPU
tensors raise.
"""
import numpy as np
import torch

from . import _lib
from . import quant as _q
from .viterbi import viterbi_encode_v_batched_cuda

TX = _q.TX
TY = _q.TY
VITERBI_CHUNK = 128
L_BITS = 16


def viterbi_encode_chunked(sequences, codebook, chunk=VITERBI_CHUNK):
    """(bitstreams, start_states, recons, mses) of every sequence (B, T)."""
    return viterbi_encode_v_batched_cuda(sequences, codebook)


def quantize_forward_gpu_no_rht(W_rotated, codebook_gpu, Tx=TX, Ty=TY):
    """Hard-quantize a weight already in the rotated basis: RMS scale, tile,
    Viterbi, untile, rescale (src/qat/ste.py:160-179)."""
    m, n = W_rotated.shape
    W_scale = W_rotated.pow(2).mean().sqrt().clamp(min=1e-30)
    seqs, info = _q._tile_for_viterbi_gpu(W_rotated / W_scale, Tx=Tx, Ty=Ty)
    _, _, recons, _ = viterbi_encode_chunked(seqs, codebook_gpu)
    return _q._untile_from_viterbi_gpu(recons, info, (m, n), Tx, Ty) * W_scale


def quantize_forward_gpu(W_latent, sign_l_gpu, sign_r_gpu, codebook_gpu, Tx=TX, Ty=TY):
    """RHT, RMS scale, tile, Viterbi, untile, rescale, inverse RHT
    (src/qat/ste.py:182-210); with 16x16 tiles the rotation, scale and tiling
    are one native call on each side of the encode."""
    if Tx != TX or Ty != TY:
        W_tilde = _q.apply_rht_gpu(W_latent, sign_l_gpu, sign_r_gpu)
        return _q.apply_inverse_rht_gpu(quantize_forward_gpu_no_rht(W_tilde, codebook_gpu, Tx, Ty),
                                        sign_l_gpu, sign_r_gpu)
    W, sl, sr, m, n = _q._rht_args(W_latent, sign_l_gpu, sign_r_gpu)
    seqs, rms = _q._tile_call(W, sl, sr, m, n)
    _, _, recons, _ = viterbi_encode_chunked(seqs, codebook_gpu)
    return _q._untile_call(recons.contiguous(), sl, sr, m, n, rms)


def _to_cuda_float32(x, device):
    if isinstance(x, torch.Tensor):
        return x.detach().to(device=device, dtype=torch.float32)
    return torch.as_tensor(np.asarray(x, dtype=np.float32), device=device)


class TrellisQuantSTE(torch.autograd.Function):
    """W_q = TrellisQuantSTE.apply(W_latent, sign_l, sign_r, codebook_gpu):
    hard trellis quantization in the forward, straight-through backward
    (src/qat/ste.py:286-333)."""

    @staticmethod
    def forward(ctx, W_latent, sign_l, sign_r, codebook_gpu):
        if not W_latent.is_cuda:
            raise RuntimeError("TrellisQuantSTE needs a CUDA W_latent (there is no CPU path)")
        dev = W_latent.device
        W_q = quantize_forward_gpu(W_latent.detach().float(), _to_cuda_float32(sign_l, dev),
                                   _to_cuda_float32(sign_r, dev), codebook_gpu)
        return W_q.to(dtype=W_latent.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output, None, None, None


class TrellisQuantSTE_IP(torch.autograd.Function):
    """Full-IP variant: W_latent already rotated (src/qat/ste.py:336-356)."""

    @staticmethod
    def forward(ctx, W_latent_rotated, codebook_gpu):
        assert W_latent_rotated.is_cuda, "IP mode requires CUDA"
        W_q = quantize_forward_gpu_no_rht(W_latent_rotated.detach().float(), codebook_gpu)
        return W_q.to(device=W_latent_rotated.device, dtype=W_latent_rotated.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output, None


def make_hyb_codebook_gpu(lut_np, Q=9, L_bits=L_BITS, device="cuda"):
    """(2^L, 2) HYB codebook from a (2^Q, 2) LUT (src/qat/ste.py:376-392) by
    the native expansion kernel (bcjr_hyb_codebook): hash x = s*s + s mod
    2^32, row (x >> (15 - Q)) & (2^Q - 1), second component negated when bit
    15 of x is set."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("make_hyb_codebook_gpu builds the codebook on a CUDA device (there is no CPU path)")
    lut = torch.as_tensor(np.asarray(lut_np, dtype=np.float32)).to(dev).contiguous()
    assert lut.shape == (1 << Q, 2), f"LUT shape mismatch: {tuple(lut.shape)}"
    cb = torch.empty((1 << L_bits, 2), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().bcjr_hyb_codebook(_lib.ptr(lut), Q, L_bits, _lib.ptr(cb),
                                                 _lib.stream_ptr(dev)), "bcjr_hyb_codebook")
    return cb


__all__ = ["VITERBI_CHUNK", "viterbi_encode_chunked", "quantize_forward_gpu_no_rht",
           "quantize_forward_gpu", "TrellisQuantSTE", "TrellisQuantSTE_IP",
           "make_hyb_codebook_gpu"]
