// Hard (min-sum) Viterbi over the same bitshift trellis: the T -> 0 limit of
// the forward recursion, as the reference's encoders compute it
// (src/viterbi/encode.py:258-310 viterbi_encode_v, :47-90 viterbi_encode;
// src/viterbi/cuda_kernel.py:17-93 for L=16, k=2, V=2).
//
//   cum_{-1}(s) = 0
//   cum_t(s)    = min_p cum_{t-1}(pred_p(s)) + |c(s) - w_t|^2
//   best_t(s)   = the lowest p attaining that minimum
//   final state = the lowest s minimising cum_{N-1}; walk back through best.
//
// pred_p(s) = (p << M) | (s >> b) depends on s only through its group
// h = s >> b, so the minimum and its index are computed once per group
// (one byte per group and step: 4096 bytes at L=16, b=4) and shared by the
// group's 2^b states.  Costs are accumulated exactly as the reference does
// (fp32, no renormalisation, d = c - w, d*d summed over V without fused
// multiply-add), so the walk, bitstream and start state are bit-identical
// to viterbi_encode_v on the same inputs.
//
// One block per sequence (persistent); the cost rows ping-pong in a global
// workspace slot (L2-resident), the per-group backpointers of all steps go
// to the same slot, and thread 0 walks back at the end.
#include <cfloat>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include "../../include/bcjr_b200.h"
#include "bcjr_kernels.h"

namespace bcjr {
namespace vit {

constexpr int kNT = 512;

// Workspace of one block: two cost rows (2^L floats each), N * G backpointer
// bytes, then the walk (N ints).
__host__ __device__ inline size_t slot_bytes(int N, int L, int BB) {
    const size_t S = (size_t)1 << L, G = S >> BB;
    size_t b = 2 * S * 4 + (size_t)N * G;
    b = (b + 15) & ~(size_t)15;
    b += (size_t)N * 4;
    return (b + 255) & ~(size_t)255;
}

template <int BB, int V>
__global__ void __launch_bounds__(kNT)
viterbi_kernel(const float *__restrict__ seq, const float *__restrict__ cb, int B, int N, int L,
               unsigned char *__restrict__ ws, size_t slot, int *__restrict__ bits,
               int *__restrict__ starts, float *__restrict__ recon, float *__restrict__ mse) {
    constexpr int NP = 1 << BB;
    const int S = 1 << L, M = L - BB, G = S >> BB;
    unsigned char *base = ws + (size_t)blockIdx.x * slot;
    float *cum[2] = {reinterpret_cast<float *>(base), reinterpret_cast<float *>(base) + S};
    unsigned char *bp = base + 2 * (size_t)S * 4;
    int *walk = reinterpret_cast<int *>(base + (((2 * (size_t)S * 4 + (size_t)N * G) + 15) & ~(size_t)15));
    __shared__ float rv[kNT / 32];
    __shared__ int ri[kNT / 32];
    __shared__ double rm[kNT / 32];

    for (long b = blockIdx.x; b < B; b += gridDim.x) {
        const float *w = seq + b * (long)N * V;
        int cur = 0;
        for (int t = 0; t < N; ++t) {
            float wv[V];
#pragma unroll
            for (int v = 0; v < V; ++v) wv[v] = __ldg(w + t * V + v);
            const float *prev = cum[cur];
            float *next = cum[cur ^ 1];
            unsigned char *bpt = bp + (size_t)t * G;
            for (int h = threadIdx.x; h < G; h += kNT) {
                float best = 0.f;
                int bi = 0;
                if (t > 0) {
                    best = prev[h];
#pragma unroll
                    for (int p = 1; p < NP; ++p) {
                        const float x = prev[(p << M) | h];
                        if (x < best) { best = x; bi = p; }
                    }
                }
                bpt[h] = (unsigned char)bi;
#pragma unroll
                for (int c = 0; c < NP; ++c) {
                    const int s = (h << BB) | c;
                    float local = 0.f;
#pragma unroll
                    for (int v = 0; v < V; ++v) {
                        const float d = __fsub_rn(__ldg(cb + (size_t)s * V + v), wv[v]);
                        local = v == 0 ? __fmul_rn(d, d) : __fadd_rn(local, __fmul_rn(d, d));
                    }
                    next[s] = __fadd_rn(best, local);
                }
            }
            cur ^= 1;
            __syncthreads();
        }
        // lowest s minimising the last cost row
        const float *last = cum[cur];
        float bv = FLT_MAX;
        int bs = S;
        for (int s = threadIdx.x; s < S; s += kNT) {
            const float x = last[s];
            if (x < bv || (x == bv && s < bs)) { bv = x; bs = s; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            const int s2 = __shfl_xor_sync(0xffffffffu, bs, o);
            if (v2 < bv || (v2 == bv && s2 < bs)) { bv = v2; bs = s2; }
        }
        if ((threadIdx.x & 31) == 0) { rv[threadIdx.x >> 5] = bv; ri[threadIdx.x >> 5] = bs; }
        __syncthreads();
        if (threadIdx.x == 0) {
            bv = rv[0];
            bs = ri[0];
            for (int i = 1; i < kNT / 32; ++i)
                if (rv[i] < bv || (rv[i] == bv && ri[i] < bs)) { bv = rv[i]; bs = ri[i]; }
            if (bs >= S) bs = 0;   // no finite cost (NaN inputs): walk from state 0
            // walk back: state at t-1 = (best_t(s >> b) << M) | (s >> b)
            int s = bs;
            walk[N - 1] = s;
            for (int t = N - 1; t > 0; --t) {
                const int h = s >> BB;
                s = ((int)bp[(size_t)t * G + h] << M) | h;
                walk[t - 1] = s;
            }
            const int h0 = s >> BB;
            starts[b] = ((int)bp[h0] << M) | h0;
        }
        __syncthreads();
        // bitstream, reconstruction and MSE of the walk
        double e2 = 0.0;
        for (int t = threadIdx.x; t < N; t += kNT) {
            const int s = walk[t];
            bits[b * (long)N + t] = s & (NP - 1);
#pragma unroll
            for (int v = 0; v < V; ++v) {
                const float r = __ldg(cb + (size_t)s * V + v);
                recon[(b * (long)N + t) * V + v] = r;
                const double d = (double)r - (double)__ldg(w + t * V + v);
                e2 += d * d;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) e2 += __shfl_xor_sync(0xffffffffu, e2, o);
        if ((threadIdx.x & 31) == 0) rm[threadIdx.x >> 5] = e2;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t2 = 0.0;
            for (int i = 0; i < kNT / 32; ++i) t2 += rm[i];
            mse[b] = (float)(t2 / ((double)N * V));
        }
        __syncthreads();
    }
}

}  // namespace vit
}  // namespace bcjr

// ---------------------------------------------------------------------------
// Host side: C ABI (include/bcjr_b200.h).

namespace {

int vit_check(int B, int N, int L, int k, int V) {
    if (B < 0 || N < 1 || N > (1 << 20) || L < 1 || k < 1 || V < 1) return BCJR_ERR_BAD_SHAPE;
    const int b = k * V;
    if (V > 2 || b > 4 || L < b || L > 16) return BCJR_ERR_UNSUPPORTED;
    switch (b * 10 + V) {
        case 11: case 21: case 31: case 41: case 22: case 42: return BCJR_OK;
        default: return BCJR_ERR_UNSUPPORTED;
    }
}

int vit_grid_cap() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return 2 * sms;
}

template <int BB, int V>
cudaError_t vit_launch(const float *seq, const float *cb, int B, int N, int L, unsigned char *ws,
                       size_t slot, int grid, int *bits, int *starts, float *recon, float *mse,
                       cudaStream_t st) {
    bcjr::vit::viterbi_kernel<BB, V><<<grid, bcjr::vit::kNT, 0, st>>>(seq, cb, B, N, L, ws, slot,
                                                                      bits, starts, recon, mse);
    return cudaGetLastError();
}

}  // namespace

extern "C" {

// Workspace: a 256-byte header (device status word, read by bcjr_ws_status)
// then the kernel's data: the cluster kernel's backpointers for L=16, k=2,
// V=2 (bcjr_vit_b4.cu) or L=16, k=2, V=1 (bcjr_vit_b2.cu), else sequence
// slots of the generic kernel.
constexpr size_t kVitHeader = 256;

// The cluster kernel for this shape: 4 (b = 4), 2 (b = 2) or 0 (none).
int vit_cluster(int N, int L, int k, int V, const void *cb) {
    if (bcjr::test_option(bcjr::kOptForceGeneric)) return 0;
    if (bcjr::vit_b4_applicable(N, L, k, V, cb)) return 4;
    if (bcjr::vit_b2_applicable(N, L, k, V, cb)) return 2;
    return 0;
}

size_t vit_cluster_bytes(int which, int B, int N) {
    return which == 4 ? bcjr::vit_b4_workspace_bytes(B, N)
                      : which == 2 ? bcjr::vit_b2_workspace_bytes(B, N) : 0;
}

BCJR_API size_t bcjr_viterbi_workspace_bytes(int B, int N, int L, int k, int V) {
    if (vit_check(B, N, L, k, V)) return 0;
    const int cap = vit_grid_cap();
    if (cap <= 0) return 0;
    const long grid = B < cap ? (B > 0 ? B : 1) : cap;
    size_t need = (size_t)grid * bcjr::vit::slot_bytes(N, L, k * V);
    const int which = vit_cluster(N, L, k, V, nullptr);
    if (which) {
        const size_t c = vit_cluster_bytes(which, B, N);
        if (c > need) need = c;
    }
    return kVitHeader + need;
}

BCJR_API int bcjr_viterbi_launches(int B, int N, int L, int k, int V) {
    const int st = vit_check(B, N, L, k, V);
    if (st) return -st;
    if (B == 0) return 0;
    const int which = vit_cluster(N, L, k, V, nullptr);
    return which == 4 ? bcjr::vit_b4_launches(B) : which == 2 ? bcjr::vit_b2_launches(B, N) : 1;
}

BCJR_API int bcjr_viterbi(const float *seq, const float *cb, int B, int N, int L, int k, int V,
                          int *bitstreams, int *start_states, float *recons, float *mses,
                          void *ws, size_t ws_bytes, bcjr_stream_t stream) {
    int st = vit_check(B, N, L, k, V);
    if (st) return st;
    if (B == 0) return BCJR_OK;
    if (!seq || !cb || !bitstreams || !start_states || !recons || !mses) return BCJR_ERR_NULL_POINTER;
    if (!ws) return BCJR_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(seq) | reinterpret_cast<uintptr_t>(cb) |
         reinterpret_cast<uintptr_t>(bitstreams) | reinterpret_cast<uintptr_t>(start_states) |
         reinterpret_cast<uintptr_t>(recons) | reinterpret_cast<uintptr_t>(mses)) & 3u)
        return BCJR_ERR_ALIGNMENT;
    if (reinterpret_cast<uintptr_t>(ws) & 255u) return BCJR_ERR_ALIGNMENT;
    if (ws_bytes <= kVitHeader) return BCJR_ERR_WORKSPACE;
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10)
        return BCJR_ERR_DEVICE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int *status = static_cast<int *>(ws);
    void *data = static_cast<char *>(ws) + kVitHeader;
    const size_t data_bytes = ws_bytes - kVitHeader;
    if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return BCJR_ERR_LAUNCH;
    const int which = vit_cluster(N, L, k, V, cb);
    if (which && data_bytes >= vit_cluster_bytes(which, B, N)) {
        // Test-only (BCJR_OPT_TEST_DROP_SENDS): the cluster kernel's CTA 1
        // withholds its outputs so that the bounded waits time out.
        const int drop = bcjr::test_option(bcjr::kOptDropSends) ? 1 : 0;
        const cudaError_t e =
            which == 4 ? bcjr::launch_vit_b4(seq, cb, B, N, bitstreams, start_states, recons, mses,
                                             data, data_bytes, status, drop, s)
                       : bcjr::launch_vit_b2(seq, cb, B, N, bitstreams, start_states, recons, mses,
                                             data, data_bytes, status, drop, s);
        return e == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH;
    }
    const size_t slot = bcjr::vit::slot_bytes(N, L, k * V);
    long grid = (long)(data_bytes / slot);
    if (grid > B) grid = B;
    const int cap = vit_grid_cap();
    if (cap > 0 && grid > cap) grid = cap;
    if (grid < 1) return BCJR_ERR_WORKSPACE;
    unsigned char *w = static_cast<unsigned char *>(data);
    cudaError_t e;
    switch (k * V * 10 + V) {
        case 11: e = vit_launch<1, 1>(seq, cb, B, N, L, w, slot, (int)grid, bitstreams, start_states, recons, mses, s); break;
        case 21: e = vit_launch<2, 1>(seq, cb, B, N, L, w, slot, (int)grid, bitstreams, start_states, recons, mses, s); break;
        case 31: e = vit_launch<3, 1>(seq, cb, B, N, L, w, slot, (int)grid, bitstreams, start_states, recons, mses, s); break;
        case 41: e = vit_launch<4, 1>(seq, cb, B, N, L, w, slot, (int)grid, bitstreams, start_states, recons, mses, s); break;
        case 22: e = vit_launch<2, 2>(seq, cb, B, N, L, w, slot, (int)grid, bitstreams, start_states, recons, mses, s); break;
        default: e = vit_launch<4, 2>(seq, cb, B, N, L, w, slot, (int)grid, bitstreams, start_states, recons, mses, s); break;
    }
    return e == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH;
}

}  // extern "C"
