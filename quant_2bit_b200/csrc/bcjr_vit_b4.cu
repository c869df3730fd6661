// Hard (min-sum) Viterbi for the trellis of the reference's QAT layers,
// L=16, k=2, V=2 (src/viterbi/cuda_kernel.py:17-93, src/viterbi/encode.py
// :258-310): the forward recursion of bcjr_b4.cu with the soft-min replaced
// by an exact minimum and its lowest-index argmin.
//
//   cum_t(s) = min_p cum_{t-1}(p 2^12 + (s >> 4)) + |c(s) - w_t|^2,  cum_{-1} = 0
//
// Butterfly r (0..255) of the b = 4 layout reads the 16 group minima
// m_t(p 2^8 + r) and writes m_{t+1}(16 r + c) = min_p cum_t(p 2^12 + 16 r + c)
// with the winning p (one backpointer byte per group and step, to HBM).  The
// arithmetic is the reference's: fp32, d = c - w, d0*d0 + d1*d1 without fused
// multiply-add, cum = min + local, no renormalisation, lowest index on ties,
// so walks are bit-identical to viterbi_encode_v.
//
// Layout and exchange as in bcjr_b4.cu (4-CTA cluster, 512 threads, one c and
// all 16 p of two butterflies per thread, codebook in registers, alpha ring
// [p/2][64][p%2] filled by st.async ... complete_tx, bounded waits).  Each
// warp also sends one token per consumer CTA after its step, so a producer
// that has a complete consumption u knows every warp has finished reading
// consumption u-1 (the ring buffer it is about to overwrite).  The last
// step's 65536 state costs give the final state (lowest index on ties,
// reduced over the cluster).  A second kernel walks back, one thread per
// sequence, writing bitstream, start state, reconstruction and MSE.
#include <cfloat>
#include <cstdint>
#include <cstring>

#include "../../include/bcjr_b200.h"
#include "bcjr_cluster.cuh"
#include "bcjr_kernels.h"

namespace bcjr {
namespace vb4 {

using namespace clu;

constexpr int kL = 16;
constexpr int kB = 4;
constexpr int kV = 2;
constexpr int kG = 1 << (kL - kB);    // 4096 groups
constexpr int kCL = 4;
constexpr int kRPC = 64;              // butterflies per CTA
constexpr int kIn = kRPC * 16;        // 1024 inputs per CTA per step
constexpr int kNT = 512;
constexpr int kWarps = kNT / 32;
// Four sequences in flight per cluster: measured on B200 (4096 x 128)
// 3.68e13 transitions/s with 2, 3.98e13 with 3, 4.28e13 with 4, 4.07e13
// with 8 (shared memory ~13 KB per slot), with the costs' sums still fused
// by the compiler; with the separately rounded sums (add2_sep) 3.66e13 at 4
// (128 registers, an 8-byte spill).
#ifndef BCJR_VIT_SLOTS
#define BCJR_VIT_SLOTS 4
#endif
constexpr int kSlots = BCJR_VIT_SLOTS;   // sequences in flight per cluster
constexpr int kNMax = 512;

struct alignas(128) Smem {
    float buf[kSlots][2][kIn];            // input ring: group minima of the previous step
    float zero[kIn];                      // inputs of step 0 (cum_{-1} = 0)
    float tok[kSlots][2][kCL * kWarps];   // per-warp tokens riding with the data
    float2 w[kSlots][kNMax];
    float wv[kSlots][kWarps];             // per-warp best final cost
    int wi[kSlots][kWarps];               // and its state
    float cv[kSlots][kCL];                // per-CTA best final cost (cluster exchange)
    int ci[kSlots][kCL];
    unsigned long long full[kSlots][2];
};

// (value, index) with the lower value, the lower index on ties.
__device__ __forceinline__ void arg_better(float &v, int &i, float v2, int i2) {
    if (v2 < v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __cluster_dims__(kCL, 1, 1) __launch_bounds__(kNT, 1)
vit_b4_kernel(const float *__restrict__ seq, const float *__restrict__ cb, int B, int N,
              unsigned char *__restrict__ bp_all, int *__restrict__ final_states, int *status,
              int drop_sends) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem &sm = *reinterpret_cast<Smem *>(smem_raw);
    constexpr uint32_t kBytes = kIn * 4 + kCL * kWarps * 4;

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t rank = cluster_rank();
    const uint32_t cid = cluster_id();
    const uint32_t ncl = num_clusters();
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem_raw);
    auto soff = [&](const void *p) -> uint32_t {
        return (uint32_t)__cvta_generic_to_shared(p) - sbase;
    };

    // one c, all 16 p of butterflies arl and arl + 16 (local)
    const int ac = lane & 15;
    const int aq = 2 * warp + (lane >> 4);
    const int arl = (aq & 15) + 32 * (aq >> 4);
    const uint32_t a_base = mapa(sbase, (uint32_t)((aq & 15) >> 2));
    const uint32_t a_off = 2u * ((uint32_t)(2 * (int)rank + (aq >> 4)) * kRPC +
                                 (uint32_t)(16 * (aq & 3) + ac));
    int hg[2];                            // my two output groups 16 r + c
    F2 C0[2][8], C1[2][8];
    const float2 *cb2 = reinterpret_cast<const float2 *>(cb);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int r = (int)rank * kRPC + arl + 16 * rr;
        hg[rr] = 16 * r + ac;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float *u = reinterpret_cast<const float *>(cb2 + (2 * i) * kG + 16 * r + ac);
            const float *v = reinterpret_cast<const float *>(cb2 + (2 * i + 1) * kG + 16 * r + ac);
            C0[rr][i] = ldg_pair(u, v);
            C1[rr][i] = ldg_pair(u + 1, v + 1);
        }
    }

    for (int i = tid; i < kIn; i += kNT) sm.zero[i] = 0.f;
    if (tid == 0) {
        for (int z = 0; z < kSlots; ++z)
            for (int x = 0; x < 2; ++x) mbar_init(sbase + soff(&sm.full[z][x]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster_sync();

    bool failed = false;
    // Test-only fault injection (BCJR_OPT_TEST_DROP_SENDS): CTA rank 1 never
    // sends its group minima or tokens, so every consumer's bounded wait expires.
    const bool drop = drop_sends != 0 && rank == 1;
    uint32_t use[kSlots];
#pragma unroll
    for (int z = 0; z < kSlots; ++z) use[z] = 0;

    for (long pair = cid; pair * kSlots < B; pair += ncl) {
        bool active[kSlots];
        long sidx[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            sidx[z] = pair * kSlots + z;
            active[z] = sidx[z] < B;
        }
        __syncthreads();
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            for (int t = tid; t < N; t += kNT) {
                const long e = (sidx[z] * N + t) * kV;
                sm.w[z][t] = make_float2(__ldg(seq + e), __ldg(seq + e + 1));
            }
        }
        __syncthreads();
        float fv[kSlots];
        int fi[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) { fv[z] = FLT_MAX; fi[z] = 1 << 30; }

        for (int t = 0; t < N; ++t) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                const float *in = sm.zero;
                if (t > 0) {
                    const int x = use[z] & 1;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_bar(bar, (use[z] >> 1) & 1, status, failed);
                    // lanes give up independently: the warp sends (and
                    // syncs) only if none of them has
                    failed = __any_sync(0xffffffffu, failed);
                    in = sm.buf[z][x];
                    ++use[z];
                }
                const int nb = use[z] & 1;
                const bool last = (t == N - 1);
                const float2 wv = sm.w[z][t];
                const F2 W0 = bc(wv.x), W1 = bc(wv.y);
                // backpointers of the groups at step t + 1 (step 0's are all 0)
                unsigned char *bpt = bp_all + ((size_t)sidx[z] * N + t + 1) * kG;
                float o[2];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int rl = arl + 16 * rr;
                    F2 x[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const F2 A = *reinterpret_cast<const F2 *>(in + 2 * (i * kRPC + rl));
                        const F2 d0 = sub2(C0[rr][i], W0), d1 = sub2(C1[rr][i], W1);
                        // cum_t of 16 states; separately rounded sums (add2_sep)
                        x[i] = add2_sep(A, add2_sep(mul2(d0, d0), mul2(d1, d1)));
                    }
                    float m = x[0].x;
                    int bi = 0;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        if (x[i].x < m) { m = x[i].x; bi = 2 * i; }
                        if (x[i].y < m) { m = x[i].y; bi = 2 * i + 1; }
                    }
                    o[rr] = m;
                    if (!last) {
                        bpt[hg[rr]] = (unsigned char)bi;
                    } else {
                        // final state: lowest-index minimum over my 32 states
                        // s = p 2^12 + 16 r + c
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            arg_better(fv[z], fi[z], x[i].x, ((2 * i) << 12) | hg[rr]);
                            arg_better(fv[z], fi[z], x[i].y, ((2 * i + 1) << 12) | hg[rr]);
                        }
                    }
                }
                if (!last && !failed && !drop) {
                    const uint32_t bar = a_base + soff(&sm.full[z][nb]);
                    st_async2(a_base + soff(&sm.buf[z][nb][0]) + 4u * a_off, o[0], o[1], bar);
                    __syncwarp();
                    if (lane < kCL) {   // token: this warp is done with consumption t
                        const uint32_t peer = mapa(sbase, (uint32_t)lane);
                        st_async1(peer + soff(&sm.tok[z][nb][rank * kWarps + warp]), 0.f,
                                  peer + soff(&sm.full[z][nb]));
                    }
                }
            }
        }
        // final state per slot: warp, CTA, cluster (lowest index on ties)
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            float v = fv[z];
            int i = fi[z];
#pragma unroll
            for (int sh = 16; sh > 0; sh >>= 1)
                arg_better(v, i, __shfl_xor_sync(0xffffffffu, v, sh),
                           __shfl_xor_sync(0xffffffffu, i, sh));
            if (lane == 0) { sm.wv[z][warp] = v; sm.wi[z][warp] = i; }
        }
        __syncthreads();
        if (tid == 0) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                float v = sm.wv[z][0];
                int i = sm.wi[z][0];
                for (int q = 1; q < kWarps; ++q) arg_better(v, i, sm.wv[z][q], sm.wi[z][q]);
                for (int r = 0; r < kCL; ++r) {
                    const uint32_t peer = mapa(sbase, (uint32_t)r);
                    st_cluster(peer + soff(&sm.cv[z][rank]), v);
                    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(peer + soff(&sm.ci[z][rank])),
                                 "r"(i) : "memory");
                }
            }
        }
        cluster_sync();
        if (rank == 0 && tid == 0) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                float v = sm.cv[z][0];
                int i = sm.ci[z][0];
                for (int r = 1; r < kCL; ++r) arg_better(v, i, sm.cv[z][r], sm.ci[z][r]);
                final_states[sidx[z]] = (i >= 0 && i < (1 << kL)) ? i : 0;
            }
        }
        // rank 0 has read cv / ci before any CTA writes the next group's
        // (with N = 1 nothing else orders the two)
        cluster_sync();
    }
}

// Walk back, one thread per sequence: state at t-1 = (bp_t(s >> 4) << 12) | (s >> 4).
__global__ void vit_b4_backtrace(const unsigned char *__restrict__ bp_all,
                                 const int *__restrict__ final_states,
                                 const float *__restrict__ seq, const float *__restrict__ cb, int B,
                                 int N, int *__restrict__ bits, int *__restrict__ starts,
                                 float *__restrict__ recon, float *__restrict__ mse,
                                 const int *__restrict__ status) {
    const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    // After a failed wait the walk is not the optimum: NaN reconstructions
    // and MSEs (the bitstreams stay in range, see below).  Selected, not
    // added, so that reconstructions stay bit-exact codebook values.
    const bool failed = poison_value(false, status) != 0.f;
    const float nanv = __int_as_float(0x7fffffff);
    // The masks keep every index in range whatever the arrays hold: after a
    // wait timeout (BCJR_ERR_TIMEOUT) the forward kernel leaves backpointers
    // and final states unwritten, and this walk must still read in bounds.
    int s = final_states[b] & ((1 << kL) - 1);
    double e2 = 0.0;
    for (int t = N - 1; t >= 0; --t) {
        const long i = b * N + t;
        bits[i] = s & 15;
        const float r0 = __ldg(cb + 2 * (size_t)s), r1 = __ldg(cb + 2 * (size_t)s + 1);
        recon[2 * i] = failed ? nanv : r0;
        recon[2 * i + 1] = failed ? nanv : r1;
        const double d0 = (double)r0 - (double)__ldg(seq + 2 * i);
        const double d1 = (double)r1 - (double)__ldg(seq + 2 * i + 1);
        e2 += d0 * d0 + d1 * d1;
        const int h = s >> 4;
        if (t > 0) s = (((int)bp_all[((size_t)b * N + t) * kG + h] & 15) << 12) | h;
        else s = h;   // step 0's backpointers are all 0
    }
    starts[b] = s;
    mse[b] = failed ? nanv : (float)(e2 / (2.0 * N));
}

}  // namespace vb4

// ---------------------------------------------------------------------------
// Host side (called by bcjr_viterbi in bcjr_viterbi.cu).

namespace {

int vit_b4_max_clusters() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev] > 0) return cached[dev];
    if (cudaFuncSetAttribute(vb4::vit_b4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(vb4::Smem)) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(sms / vb4::kCL * vb4::kCL), 1, 1);
    cfg.blockDim = dim3(vb4::kNT, 1, 1);
    cfg.dynamicSmemBytes = sizeof(vb4::Smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = vb4::kCL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, vb4::vit_b4_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cached[dev] = n;
    return n;
}

}  // namespace

constexpr long kVitChunk = 2048;   // sequences per forward + backtrace launch pair

bool vit_b4_applicable(int N, int L, int k, int V, const void *cb) {
    return L == vb4::kL && k * V == vb4::kB && V == vb4::kV && N >= 1 && N <= vb4::kNMax &&
           (reinterpret_cast<uintptr_t>(cb) & 7u) == 0 && vit_b4_max_clusters() > 0;
}

int vit_b4_launches(int B) {
    return B <= 0 ? 0 : (int)(2 * ((B + kVitChunk - 1) / kVitChunk));
}

size_t vit_b4_workspace_bytes(int B, int N) {
    const long c = B < kVitChunk ? (B > 0 ? B : 1) : kVitChunk;
    return 256 + (size_t)c * N * vb4::kG + (size_t)c * 4;
}

cudaError_t launch_vit_b4(const float *seq, const float *cb, int B, int N, int *bits,
                          int *starts, float *recon, float *mse, void *ws, size_t ws_bytes,
                          int *status, int drop_sends, cudaStream_t st) {
    const long c = B < kVitChunk ? B : kVitChunk;
    unsigned char *bp = static_cast<unsigned char *>(ws) + 256;
    int *finals = reinterpret_cast<int *>(bp + (size_t)c * N * vb4::kG);
    if (ws_bytes < vit_b4_workspace_bytes(B, N)) return cudaErrorInvalidValue;
    const int maxc = vit_b4_max_clusters();
    if (maxc <= 0) return cudaErrorInvalidConfiguration;
    for (long b0 = 0; b0 < B; b0 += c) {
        const int nb = (int)((B - b0) < c ? (B - b0) : c);
        long ncl = (nb + vb4::kSlots - 1) / vb4::kSlots;
        if (ncl > maxc) ncl = maxc;
        vb4::vit_b4_kernel<<<(unsigned)(ncl * vb4::kCL), vb4::kNT, sizeof(vb4::Smem), st>>>(
            seq + b0 * N * 2, cb, nb, N, bp, finals, status, drop_sends);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        vb4::vit_b4_backtrace<<<(nb + 127) / 128, 128, 0, st>>>(
            bp, finals, seq + b0 * N * 2, cb, nb, N, bits + b0 * N, starts + b0, recon + b0 * N * 2,
            mse + b0, status);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace bcjr
