// Randomized Hadamard transform (RHT), RMS scale and 16x16 tiling around the
// BCJR op: the caller side of the reference's quantizer wrapper
// (src/bcjr/bcjr_quant.py:125-178, src/qat/ste.py:113-159,
// src/rht/transform.py:26-126), as native kernels.
//
//   RHT(W)      = H_m diag(s_l) W diag(s_r) H_n / sqrt(m n)     (H unnormalised)
//   RHT^-1(Z)   = diag(s_l) H_m Z H_n diag(s_r) / sqrt(m n)
//   A(W, mu)    = tile(RHT(W)) * mu          (mu = 1 / RMS(RHT(W)) by default)
//   B(S, s)     = RHT^-1(untile(S) * s)
//
// RHT is orthogonal and tiling is a permutation, so the adjoint of A(., mu)
// is B(., mu) and the adjoint of B(., s) is A(., s): each op's backward is
// the other op.
//
// Passes (all HBM-bound; m, n powers of two, 16 <= m, n <= 32768):
//   row pass     one CTA per row: load (times a sign vector), Walsh-Hadamard
//                butterflies in shared memory, store (times a sign vector and
//                a scale); optionally the row's sum of squares (in double)
//   transpose    32 x 32 tiles through shared memory
//   tile/untile  a transpose that writes (reads) the 16 x 16 tile order:
//                sequence b = j (m / 16) + i holds rows 16 i.., cols 16 j..,
//                row-major (src/qat/ste.py:138-159)
//   rms          one block adds the row sums in a fixed order: deterministic
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/bcjr_b200.h"
#include "bcjr_kernels.h"

namespace bcjr {
namespace rht {

constexpr int kRowThreads = 512;
constexpr int kMaxLen = 32768;        // 128 KB of shared memory per row

// One row of length `len` (power of two): y = H (x * pre) * scale * post.
__global__ void __launch_bounds__(kRowThreads)
fwht_rows(const float *in, float *out, int len, const float *__restrict__ pre,
          const float *__restrict__ post, const float *__restrict__ scale_dev, float scale,
          double *__restrict__ row_sumsq) {
    extern __shared__ float x[];
    __shared__ double red[kRowThreads / 32];
    const long row = blockIdx.x;
    const float *src = in + row * (long)len;
    for (int k = threadIdx.x; k < len; k += blockDim.x) {
        float v = src[k];
        if (pre) v *= __ldg(pre + k);
        x[k] = v;
    }
    __syncthreads();
    const int half = len >> 1;
    for (int h = 1; h < len; h <<= 1) {
        for (int b = threadIdx.x; b < half; b += blockDim.x) {
            const int i = ((b & ~(h - 1)) << 1) | (b & (h - 1));
            const float a = x[i], c = x[i + h];
            x[i] = a + c;
            x[i + h] = a - c;
        }
        __syncthreads();
    }
    const float sc = scale * (scale_dev ? *scale_dev : 1.f);
    double ss = 0.0;
    float *dst = out + row * (long)len;
    for (int k = threadIdx.x; k < len; k += blockDim.x) {
        float v = x[k] * sc;
        if (post) v *= __ldg(post + k);
        dst[k] = v;
        ss += (double)v * (double)v;
    }
    if (row_sumsq) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
            row_sumsq[row] = t;
        }
    }
}

// out (C x R) = in (R x C) transposed; block (32, 8), 32 x 32 tiles.
__global__ void transpose(const float *__restrict__ in, float *__restrict__ out, int R, int C) {
    __shared__ float t[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x;
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int r = r0 + k, c = c0 + tx;
        if (r < R && c < C) t[k][tx] = in[(long)r * C + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int c = c0 + k, r = r0 + tx;
        if (r < R && c < C) out[(long)c * R + r] = t[tx][k];
    }
}

// seqs[b][16 (r % 16) + c % 16] = Z(r, c) * mu,  b = (c / 16) (m / 16) + r / 16,
// reading Z transposed: zt (n x m), zt[c][r] = Z(r, c).
__global__ void transpose_tile(const float *__restrict__ zt, float *__restrict__ seqs, int m, int n,
                               const float *__restrict__ mu_dev) {
    __shared__ float t[32][33];
    const int r0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const int tx = threadIdx.x;
    const float mu = *mu_dev;
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int c = c0 + k, r = r0 + tx;
        if (r < m && c < n) t[k][tx] = zt[(long)c * m + r];
    }
    __syncthreads();
    const long rb = m >> 4;
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int r = r0 + k, c = c0 + tx;
        if (r < m && c < n)
            seqs[((long)(c >> 4) * rb + (r >> 4)) * 256 + (r & 15) * 16 + (c & 15)] = t[tx][k] * mu;
    }
}

// X(r, c) = seqs[b][16 (r % 16) + c % 16] * s, X (m x n) row-major.
__global__ void untile(const float *__restrict__ seqs, float *__restrict__ x, int m, int n,
                       const float *__restrict__ s_dev) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)m * n) return;
    const int r = (int)(i / n), c = (int)(i % n);
    const long rb = m >> 4;
    x[i] = seqs[((long)(c >> 4) * rb + (r >> 4)) * 256 + (r & 15) * 16 + (c & 15)] * *s_dev;
}

// rms = max(sqrt(sum / count), 1e-30) over the row sums (fixed order);
// mu = 1 / rms.  One block.
__global__ void rms_from_rows(const double *__restrict__ row_sumsq, int rows, double count,
                              float *__restrict__ rms_out, float *__restrict__ mu_out) {
    __shared__ double red[1024];
    double t = 0.0;
    for (int i = threadIdx.x; i < rows; i += blockDim.x) t += row_sumsq[i];
    red[threadIdx.x] = t;
    __syncthreads();
    for (int w = blockDim.x >> 1; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float rms = (float)sqrt(red[0] / count);
        if (!(rms >= 1e-30f)) rms = rms != rms ? rms : 1e-30f;   // clamp(min=1e-30), NaN kept
        if (rms_out) *rms_out = rms;
        *mu_out = 1.f / rms;
    }
}

}  // namespace rht
}  // namespace bcjr

// ---------------------------------------------------------------------------
// Host side: C ABI (include/bcjr_b200.h).

namespace {

using bcjr::rht::kMaxLen;
using bcjr::rht::kRowThreads;

constexpr size_t kRhtHeader = 256;

bool pow2_in_range(int v) { return v >= 16 && v <= kMaxLen && (v & (v - 1)) == 0; }

struct RhtWs {
    float *buf1, *buf2;
    double *rows;
    float *mu, *rms;
};

size_t rht_bytes(int m, int n) {
    const size_t mn = (size_t)m * n;
    const size_t mx = (size_t)(m > n ? m : n);
    return kRhtHeader + 2 * mn * 4 + mx * 8 + 256;
}

int rht_check(const void *a, const void *sl, const void *sr, int m, int n, const void *out,
              void *ws, size_t ws_bytes, RhtWs &w) {
    if (!pow2_in_range(m) || !pow2_in_range(n)) return BCJR_ERR_BAD_SHAPE;
    if (!a || !sl || !sr || !out) return BCJR_ERR_NULL_POINTER;
    if (!ws) return BCJR_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(sl) |
         reinterpret_cast<uintptr_t>(sr) | reinterpret_cast<uintptr_t>(out)) & 3u)
        return BCJR_ERR_ALIGNMENT;
    if (reinterpret_cast<uintptr_t>(ws) & 255u) return BCJR_ERR_ALIGNMENT;
    if (ws_bytes < rht_bytes(m, n)) return BCJR_ERR_WORKSPACE;
    char *p = static_cast<char *>(ws) + kRhtHeader;
    const size_t mn = (size_t)m * n;
    w.buf1 = reinterpret_cast<float *>(p); p += mn * 4;
    w.buf2 = reinterpret_cast<float *>(p); p += mn * 4;
    w.rows = reinterpret_cast<double *>(p); p += (size_t)(m > n ? m : n) * 8;
    w.mu = reinterpret_cast<float *>(p);
    w.rms = w.mu + 1;
    return BCJR_OK;
}

cudaError_t rows_pass(const float *in, float *out, int nrows, int len, const float *pre,
                      const float *post, float scale, double *sums, cudaStream_t st) {
    // rows up to kMaxLen floats of dynamic shared memory (set on the current device)
    const cudaError_t ea = cudaFuncSetAttribute(bcjr::rht::fwht_rows,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kMaxLen * 4);
    if (ea != cudaSuccess) return ea;
    int threads = len / 2;
    if (threads > kRowThreads) threads = kRowThreads;
    if (threads < 32) threads = 32;
    bcjr::rht::fwht_rows<<<nrows, threads, (size_t)len * 4, st>>>(in, out, len, pre, post, nullptr,
                                                                  scale, sums);
    return cudaGetLastError();
}

cudaError_t transpose_pass(const float *in, float *out, int R, int C, cudaStream_t st) {
    const dim3 grid((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32)), block(32, 8);
    bcjr::rht::transpose<<<grid, block, 0, st>>>(in, out, R, C);
    return cudaGetLastError();
}

int done(cudaError_t e) { return e == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH; }

}  // namespace

extern "C" {

BCJR_API size_t bcjr_rht_workspace_bytes(int m, int n) {
    if (!pow2_in_range(m) || !pow2_in_range(n)) return 0;
    return rht_bytes(m, n);
}

BCJR_API int bcjr_rht(const float *W, const float *sign_l, const float *sign_r, int m, int n,
                      int inverse, float *out, void *ws, size_t ws_bytes, bcjr_stream_t stream) {
    RhtWs w;
    const int st = rht_check(W, sign_l, sign_r, m, n, out, ws, ws_bytes, w);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const float inv = (float)(1.0 / sqrt((double)m * (double)n));
    cudaError_t e;
    if (!inverse) {
        // rows: W diag(s_r) H_n; columns: H_m diag(s_l) (.)
        if ((e = rows_pass(W, w.buf1, m, n, sign_r, nullptr, 1.f, nullptr, s))) return done(e);
        if ((e = transpose_pass(w.buf1, w.buf2, m, n, s))) return done(e);
        if ((e = rows_pass(w.buf2, w.buf2, n, m, sign_l, nullptr, inv, nullptr, s))) return done(e);
    } else {
        // rows: Z H_n diag(s_r); columns: diag(s_l) H_m (.)
        if ((e = rows_pass(W, w.buf1, m, n, nullptr, sign_r, 1.f, nullptr, s))) return done(e);
        if ((e = transpose_pass(w.buf1, w.buf2, m, n, s))) return done(e);
        if ((e = rows_pass(w.buf2, w.buf2, n, m, nullptr, sign_l, inv, nullptr, s))) return done(e);
    }
    return done(transpose_pass(w.buf2, out, n, m, s));
}

BCJR_API int bcjr_rht_tile(const float *W, const float *sign_l, const float *sign_r, int m, int n,
                           const float *mu_dev, float *seqs, float *rms_out, void *ws,
                           size_t ws_bytes, bcjr_stream_t stream) {
    RhtWs w;
    const int st = rht_check(W, sign_l, sign_r, m, n, seqs, ws, ws_bytes, w);
    if (st) return st;
    if ((mu_dev && (reinterpret_cast<uintptr_t>(mu_dev) & 3u)) ||
        (rms_out && (reinterpret_cast<uintptr_t>(rms_out) & 3u)))
        return BCJR_ERR_ALIGNMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const float inv = (float)(1.0 / sqrt((double)m * (double)n));
    cudaError_t e;
    if ((e = rows_pass(W, w.buf1, m, n, sign_r, nullptr, 1.f, nullptr, s))) return done(e);
    if ((e = transpose_pass(w.buf1, w.buf2, m, n, s))) return done(e);
    if ((e = rows_pass(w.buf2, w.buf2, n, m, sign_l, nullptr, inv, mu_dev ? nullptr : w.rows, s)))
        return done(e);
    const float *mu = mu_dev;
    if (!mu) {
        bcjr::rht::rms_from_rows<<<1, 1024, 0, s>>>(w.rows, n, (double)m * (double)n,
                                                    rms_out ? rms_out : w.rms, w.mu);
        if ((e = cudaGetLastError())) return done(e);
        mu = w.mu;
    }
    const dim3 grid((unsigned)((m + 31) / 32), (unsigned)((n + 31) / 32)), block(32, 8);
    bcjr::rht::transpose_tile<<<grid, block, 0, s>>>(w.buf2, seqs, m, n, mu);
    return done(cudaGetLastError());
}

BCJR_API int bcjr_untile_irht(const float *seqs, const float *sign_l, const float *sign_r, int m,
                              int n, const float *s_dev, float *out, void *ws, size_t ws_bytes,
                              bcjr_stream_t stream) {
    RhtWs w;
    const int st = rht_check(seqs, sign_l, sign_r, m, n, out, ws, ws_bytes, w);
    if (st) return st;
    if (!s_dev) return BCJR_ERR_NULL_POINTER;
    if (reinterpret_cast<uintptr_t>(s_dev) & 3u) return BCJR_ERR_ALIGNMENT;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const float inv = (float)(1.0 / sqrt((double)m * (double)n));
    const long mn = (long)m * n;
    bcjr::rht::untile<<<(unsigned)((mn + 255) / 256), 256, 0, s>>>(seqs, w.buf1, m, n, s_dev);
    cudaError_t e;
    if ((e = cudaGetLastError())) return done(e);
    if ((e = rows_pass(w.buf1, w.buf1, m, n, nullptr, sign_r, 1.f, nullptr, s))) return done(e);
    if ((e = transpose_pass(w.buf1, w.buf2, m, n, s))) return done(e);
    if ((e = rows_pass(w.buf2, w.buf2, n, m, nullptr, sign_l, inv, nullptr, s))) return done(e);
    return done(transpose_pass(w.buf2, out, n, m, s));
}

}  // extern "C"
