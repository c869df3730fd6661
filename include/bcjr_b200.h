/*
 * bcjr_b200 -- C ABI of the B200 (sm_100a) BCJR forward-backward library.
 *
 * The library computes sum-product message passing at temperature T over the
 * QTIP bitshift trellis (2^L states, next state ((s << kV) | c) & (2^L - 1))
 * with a per-state codebook c(s) in R^V, for B independent sequences of N
 * steps.  It returns the soft codeword E[c(s_t)] per step and, in the
 * backward entry point, the gradient of <grad_soft, soft> with respect to the
 * input sequence.
 *
 * All pointers are device pointers (fp32, C-contiguous) unless stated
 * otherwise.  Every call is asynchronous and ordered on `stream`; no call
 * synchronises the host or reads T on the host.  The caller owns every
 * buffer, including the workspace, whose size comes from
 * bcjr_workspace_bytes().  Calls on the same workspace must not overlap.
 *
 * Failures on the device are never silent: when a bounded device-side wait
 * gives up (BCJR_ERR_TIMEOUT in the workspace status word, read by
 * bcjr_ws_status), every output written after the failure was recorded --
 * always including those of the sequences whose wait expired -- is NaN, and
 * so is every output of a call whose device temperature T is not positive
 * and finite.  NaN and infinite inputs propagate to the outputs of their
 * sequences, as in the reference.
 *
 * Reference interfaces replaced (Venugopalan2610/quant-2bit):
 *   src/bcjr/bcjr_monolithic.py:157-243  BcjrForwardBackwardMonolithic
 *   src/bcjr/forward_backward.py:190-232  bcjr_forward_backward
 *   src/bcjr/bcjr_triton.py:32-119        the per-step Triton kernels
 */
#ifndef BCJR_B200_H
#define BCJR_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define BCJR_API __attribute__((visibility("default")))
#else
#define BCJR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; declared here so that the header needs no
 * CUDA include.  Pass 0 for the legacy default stream. */
typedef struct CUstream_st *bcjr_stream_t;

/* Status codes.  0 is success.  The reference raises AssertionError for shape
 * and dtype problems (forward_backward.py:206-207, bcjr_monolithic.py:162-163);
 * the Python layer maps BCJR_ERR_BAD_SHAPE back to AssertionError. */
enum {
    BCJR_OK = 0,
    BCJR_ERR_BAD_SHAPE = 1,      /* B, N, L, k, V inconsistent or out of range */
    BCJR_ERR_UNSUPPORTED = 2,    /* (L, k, V) combination not built           */
    BCJR_ERR_NULL_POINTER = 3,   /* a required pointer is NULL                */
    BCJR_ERR_ALIGNMENT = 4,      /* pointer not aligned to its element size   */
    BCJR_ERR_WORKSPACE = 5,      /* workspace missing or too small            */
    BCJR_ERR_LAUNCH = 6,         /* CUDA launch or device query failed        */
    BCJR_ERR_DEVICE = 7,         /* device is not sm_100 or not usable        */
    BCJR_ERR_TIMEOUT = 8         /* a bounded device-side wait gave up        */
};

/* Workspace flags for bcjr_workspace_bytes(). */
enum {
    BCJR_WS_FORWARD = 1,
    BCJR_WS_BACKWARD = 2,
    BCJR_WS_INTERNALS = 4
};

/* Library version (major * 10000 + minor * 100 + patch). */
BCJR_API int bcjr_version(void);

/* Test and diagnostic switches, process-wide, all 0 by default.  Nothing in
 * the library reads the environment.  No counterpart in the reference.
 *   BCJR_OPT_TEST_DROP_SENDS      1: CTA 1 of every cluster kernel withholds
 *                                 its messages, so bounded waits expire
 *                                 (tests of the timeout path only)
 *   BCJR_OPT_FORCE_GENERIC        1: one-block-per-sequence kernels for all
 *                                 shapes (cross-checks of the cluster kernels)
 *   BCJR_OPT_L16_FORWARD_CLUSTER  2 or 4: cluster size of the L=16, k=2, V=1
 *   BCJR_OPT_L16_BACKWARD_CLUSTER   forward / backward (0: automatic)
 * Returns the previous value, or -1 for an unknown option. */
enum {
    BCJR_OPT_TEST_DROP_SENDS = 1,
    BCJR_OPT_FORCE_GENERIC = 2,
    BCJR_OPT_L16_FORWARD_CLUSTER = 3,
    BCJR_OPT_L16_BACKWARD_CLUSTER = 4
};
BCJR_API int bcjr_set_test_option(int option, int value);

/* SMs that the persistent cluster kernels leave free, process-wide, 0 by
 * default (0..64).  A persistent kernel holds every SM it is given until it
 * ends; a collective kernel queued beside it (an NCCL all-gather of a soft
 * weight while the next weight is quantized) then waits for SMs, and one
 * that started on one GPU spins until its peers' copies start.  Reserving a
 * few SMs, and capping the collective's CTAs to them (NCCL_MAX_CTAS), lets
 * both run at once.  Workspace sizes depend on it: set it before
 * bcjr_workspace_bytes and keep it until the call is launched.  Returns the
 * previous value, or -1 when out of range.  No counterpart in the reference
 * (it has no multi-GPU path). */
BCJR_API int bcjr_set_reserved_sms(int sms);

/* Static string for a status code. */
BCJR_API const char *bcjr_status_string(int status);

/* Bytes of device workspace needed by the entry points named in `flags` for
 * this problem on the current device.  Returns 0 for an invalid or
 * unsupported shape (bcjr_check_shape() gives the reason).
 * Replaces the reference's per-call (B,N,S) allocations
 * (bcjr_monolithic.py:49-56, :83-87, :109-112) with an O(grid) buffer. */
BCJR_API size_t bcjr_workspace_bytes(int B, int N, int L, int k, int V, int flags);

/* Shape validation without launching anything: BCJR_OK or the error code. */
BCJR_API int bcjr_check_shape(int B, int N, int L, int k, int V);

/* Kernel launches one call of the entry point named by `flags`
 * (BCJR_WS_FORWARD, BCJR_WS_BACKWARD or BCJR_WS_INTERNALS, one of them)
 * makes for this problem on the current device, with a 16-byte aligned
 * codebook; 0 for an invalid shape.  For profiling and launch accounting. */
BCJR_API int bcjr_kernel_launches(int B, int N, int L, int k, int V, int flags);

/*
 * Forward: soft[b,t,:] = sum_s P_t(s) c(s)  and  logZ[b] (natural log).
 *   seq   (B, N, V)   input sequences (the 16x16 weight tiles)
 *   cb    (2^L, V)    codebook
 *   T_dev scalar      temperature, device memory (read on the device)
 *   soft  (B, N, V)   output
 *   logZ  (B,)        output, may be NULL
 * Replaces BcjrForwardBackwardMonolithic.forward (bcjr_monolithic.py:160-189)
 * and the value part of bcjr_forward_backward (forward_backward.py:190-232).
 */
BCJR_API int bcjr_fb_forward(const float *seq, const float *cb, const float *T_dev,
                    int B, int N, int L, int k, int V,
                    float *soft, float *logZ,
                    void *ws, size_t ws_bytes, bcjr_stream_t stream);

/*
 * Backward: d_seq = d <grad_soft, soft> / d seq, the gradient the reference's
 * analytic backward defines (bcjr_monolithic.py:191-243):
 *   d_seq[b,u,:] = (2/T) sum_s dl_u(s) (c(s) - seq[b,u,:]),
 *   dl_u(s) = P_u(s) (E[G | s_u = s] - E[G]),  G = sum_t <grad_soft_t, c(s_t)>.
 *   soft       (B, N, V)  the forward's output (used to centre G)
 *   grad_soft  (B, N, V)  upstream gradient
 *   d_seq      (B, N, V)  output
 * Replaces BcjrForwardBackwardMonolithic.backward and the Triton
 * _alpha_step_bwd_kernel scatter (bcjr_triton.py:75-119).
 */
BCJR_API int bcjr_fb_backward(const float *seq, const float *cb, const float *T_dev,
                     const float *soft, const float *grad_soft,
                     int B, int N, int L, int k, int V,
                     float *d_seq,
                     void *ws, size_t ws_bytes, bcjr_stream_t stream);

/*
 * Full internals for return_internals=True (forward_backward.py:202-204,
 * :230-231): P, log_alpha, log_beta, each (B, N, 2^L) fp32, natural log.
 * Any of the three may be NULL.  O(B N 2^L) output: for diagnostics only
 * (src/bcjr/anneal.py:143-184).
 */
BCJR_API int bcjr_fb_internals(const float *seq, const float *cb, const float *T_dev,
                      int B, int N, int L, int k, int V,
                      float *P, float *log_alpha, float *log_beta,
                      void *ws, size_t ws_bytes, bcjr_stream_t stream);

/* Device-side status of the last call that used `ws` (synchronises
 * `stream`): BCJR_OK, or BCJR_ERR_TIMEOUT if a bounded wait gave up. */
BCJR_API int bcjr_ws_status(const void *ws, bcjr_stream_t stream);

/*
 * Forward without a workspace, for callers that cannot allocate device
 * memory: a host binding this ABI from another language with no device
 * allocator of its own, or a loop that must not call cudaMalloc between
 * steps (cudaMalloc synchronises the device).  No counterpart in the
 * reference (it has no C ABI); same inputs, outputs and meaning as
 * bcjr_fb_forward.
 *
 * Scratch is a fixed 64 MiB array inside this library's device image, held
 * by every GPU that loads the library until the process exits.  One
 * sequence slot takes (N + 3) 2^(L - kV) + 2N floats (+1 when that is odd);
 * a shape whose single slot does not fit is rejected with
 * BCJR_ERR_WORKSPACE (at L=16, k=2, V=1: N > 1020).  Smaller shapes run on
 * as many slots as fit, one block per slot, each block taking the next
 * sequence when it finishes one; that is slower than bcjr_fb_forward for
 * large batches.  The first call on each device (and the first after the
 * device's context was reset and re-created) looks up the array's device
 * address with cudaGetSymbolAddress; make it before any stream capture.
 * All calls share the array and it keeps the last call's contents (the
 * kernel writes every element before reading it): calls that overlap on the
 * GPU race and must be serialised by the caller.  Allocates nothing, on the
 * host or the device.
 */
BCJR_API int bcjr_fb_forward_noalloc(const float *seq, const float *cb, const float *T_dev,
                                     int B, int N, int L, int k, int V,
                                     float *soft, float *logZ, bcjr_stream_t stream);

/*
 * MUFU throughput probe, a diagnostic: launches 4 x (SM count) blocks of 256
 * threads, each thread running 8 independent chains of `iters`
 * ex2.approx.f32 operations, and writes the number of ex2 operations launched
 * to *ops (host pointer).  Timed with events on `stream`, ops / time is the
 * MUFU pipe's measured throughput: the roofline denominator of the BCJR
 * kernels, which are bound by that pipe.  `out` is one device float that
 * the kernel never writes in practice.  No counterpart in the reference.
 */
BCJR_API int bcjr_probe_mufu(float *out, int iters, double *ops, bcjr_stream_t stream);

/*
 * Randomized Hadamard transform and tiling around the op: the caller side
 * of the reference's quantizer wrapper.  m, n are powers of two in
 * [16, 32768]; fp32 matrices row-major; sign vectors of +-1 (length m for
 * sign_l, n for sign_r); workspace of bcjr_rht_workspace_bytes(m, n) bytes,
 * 256-byte aligned.  Stream-ordered, no host synchronisation.
 *
 * bcjr_rht: out = H_m diag(sign_l) W diag(sign_r) H_n / sqrt(m n) (inverse
 * = 0), or its inverse diag(sign_l) H_m W H_n diag(sign_r) / sqrt(m n)
 * (inverse = 1), H the unnormalised Walsh-Hadamard matrix.  Replaces
 * apply_rht_gpu / apply_inverse_rht_gpu (src/qat/ste.py:113-135, which need
 * the fast_hadamard_transform extension) and apply_rht / apply_inverse_rht
 * (src/rht/transform.py:65-126).
 */
BCJR_API size_t bcjr_rht_workspace_bytes(int m, int n);
BCJR_API int bcjr_rht(const float *W, const float *sign_l, const float *sign_r, int m, int n,
                      int inverse, float *out, void *ws, size_t ws_bytes, bcjr_stream_t stream);

/*
 * seqs (m n / 256 sequences of 256) = tile(RHT(W)) * mu, in the 16 x 16 tile
 * order of _tile_for_viterbi_gpu (src/qat/ste.py:138-149): sequence
 * j (m/16) + i holds rows 16i.., cols 16j.., row-major.  mu_dev NULL: mu =
 * 1 / max(RMS(RHT(W)), 1e-30), the detached RMS scale of
 * bcjr_quantize_weight_rotated (src/bcjr/bcjr_quant.py:125-141); the RMS is
 * written to rms_out when it is not NULL (device float).  Otherwise mu is
 * read from mu_dev (device float) and rms_out is ignored.
 */
BCJR_API int bcjr_rht_tile(const float *W, const float *sign_l, const float *sign_r, int m, int n,
                           const float *mu_dev, float *seqs, float *rms_out, void *ws,
                           size_t ws_bytes, bcjr_stream_t stream);

/*
 * out (m x n) = RHT^-1(untile(seqs) * s), s read from s_dev (device float):
 * the untile, rescale and inverse RHT that follow the op in
 * bcjr_quantize_weight_rotated / bcjr_quantize_weight
 * (src/bcjr/bcjr_quant.py:149-178, src/qat/ste.py:152-159).  It is also the
 * adjoint of bcjr_rht_tile with mu = s, and bcjr_rht_tile with mu = s is its
 * adjoint (gradients of the pair).
 */
BCJR_API int bcjr_untile_irht(const float *seqs, const float *sign_l, const float *sign_r, int m,
                              int n, const float *s_dev, float *out, void *ws, size_t ws_bytes,
                              bcjr_stream_t stream);

/*
 * Hard (min-sum) Viterbi encoding of B sequences of N steps (seq: B x N x V
 * fp32, i.e. the reference's (B, T) with T = N V) over the same trellis and
 * codebook.  Outputs: bitstreams (B x N int32, the low kV bits of each state
 * of the best walk), start_states (B int32, the state before step 0),
 * recons (B x N x V fp32, the walk's codewords) and mses (B fp32, mean
 * squared error of recons).  Replaces viterbi_encode_v_batched_cuda
 * (src/viterbi/cuda_kernel.py:147-220, L=16, k=2, V=2 only) and the numpy
 * encoders viterbi_encode_v / viterbi_encode_v_batched
 * (src/viterbi/encode.py:258-310, :425-497): costs accumulate as in
 * viterbi_encode_v (fp32, d = c - w, d*d summed over V, no fused
 * multiply-add), ties go to the lowest predecessor index and the lowest
 * final state, so walks are bit-identical to it.  Shapes as for the BCJR
 * op; workspace of bcjr_viterbi_workspace_bytes bytes, 256-byte aligned
 * (L=16, k=2 runs on 4-CTA clusters for N <= 512 and needs N * 4096 bytes
 * per sequence, for up to 2048 sequences at a time at V=2 and up to
 * 2^18 / N at V=1; other shapes run fewer sequences at a time when given
 * fewer bytes).  bcjr_ws_status reports a device-side wait timeout.
 * bcjr_viterbi_launches: the number of kernels one bcjr_viterbi call with
 * these shapes launches on the current device given a workspace of
 * bcjr_viterbi_workspace_bytes (one per chunk of sequences and its
 * walk-back on the cluster paths, one otherwise; 0 for B = 0, a negative
 * error code for an unsupported shape).  No counterpart in the reference:
 * launch accounting for benchmarks.
 */
BCJR_API size_t bcjr_viterbi_workspace_bytes(int B, int N, int L, int k, int V);
BCJR_API int bcjr_viterbi_launches(int B, int N, int L, int k, int V);
BCJR_API int bcjr_viterbi(const float *seq, const float *cb, int B, int N, int L, int k, int V,
                          int *bitstreams, int *start_states, float *recons, float *mses,
                          void *ws, size_t ws_bytes, bcjr_stream_t stream);

/* HYB codebook: cb_out (2^L x 2 fp32, device) from lut (2^Q x 2 fp32,
 * device): for each state s, x = (s*s + s) mod 2^32, row = (x >> (15 - Q))
 * mod 2^Q, cb_out[s] = (lut[row][0], +-lut[row][1]) with the sign flipped
 * when bit 15 of x is set.  1 <= Q <= 15, 1 <= L <= 24; both pointers 8-byte
 * aligned.  Replaces make_hyb_codebook_gpu (src/qat/ste.py:376-392) and
 * decode_hyb_batch (src/codes/ref.py:116-128); bit-identical to both. */
BCJR_API int bcjr_hyb_codebook(const float *lut, int Q, int L, float *cb_out, bcjr_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BCJR_B200_H */
