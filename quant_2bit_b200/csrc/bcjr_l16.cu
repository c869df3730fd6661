// Production kernel for the QTIP trellis L=16, k=2, V=1 (b = 2): one
// 4-CTA thread-block cluster per pair of sequences, one CTA per SM.
//
// Work decomposition
// ------------------
// With M = 14, the 2^16 states split into 4096 "butterflies"
//     j in [0, 4096):  states q = p * 2^14 + 4 j + c,   p, c in 0..3.
// In the forward (alpha) direction butterfly j reads the four group values
// A_t(p 2^12 + j) (one per p) and writes A_{t+1}(4 j + c) (one per c); in the
// backward (beta) direction it reads Bt_{t+1}(4 j + c) and writes
// Bt_t(p 2^12 + j).  Every step touches the same 16 states per butterfly, so
// each thread owns two butterflies for the whole kernel and keeps their 32
// codebook values in registers: no codebook traffic at all after the first
// load.  CTA r of the cluster owns butterflies [1024 r, 1024 r + 1024).
//
// Exchange between steps
// ----------------------
// The outputs of a step are the inputs of butterflies spread over the whole
// cluster (a perfect shuffle).  Producers push them straight into the
// consumer CTA's shared memory with st.async ... mbarrier::complete_tx, into
// a 3-deep ring of input buffers; each buffer has an mbarrier that the
// consumer arms with the expected byte count.  The ring depth plus one
// __syncthreads per step guarantee a buffer is never overwritten before
// every thread of its CTA has read it (a producer writing buffer u+1 during
// consumption u proves all CTAs finished consumption u-2).  Every wait is
// bounded (about 1 s); on timeout the kernel records BCJR_ERR_TIMEOUT in the
// workspace status word, stops waiting and sending, and runs to completion.
//
// Renormalisation: each CTA's maximum output travels with the data (one
// st.async per destination), so every consumer subtracts the exact global
// maximum of the previous step; shifts accumulate in double.
//
// Two sequences are interleaved step by step ("slots") so that one slot's
// exchange latency hides behind the other's arithmetic.  Alpha/H rows go to
// a global history (float4 stores, read back with L1-bypassing loads in the
// backward-time sweep).  Per-step partial sums of soft / d_seq are written
// per CTA and added in a fixed order by CTA 0: results are deterministic.
//
// The recursions are documented in bcjr_common.cuh.
#include <cstdint>

#include "bcjr_common.cuh"
#include "bcjr_kernels.h"

namespace bcjr {
namespace l16 {

constexpr int kL = 16;
constexpr int kB = 2;                 // branch bits b = kV
constexpr int kG = 1 << (kL - kB);    // 16384 groups
constexpr int kNJ = kG >> kB;         // 4096 butterflies
constexpr int kCL = 4;                // CTAs per cluster
constexpr int kJPC = kNJ / kCL;       // 1024 butterflies per CTA
constexpr int kNT = 512;              // threads per CTA
constexpr int kJPT = kJPC / kNT;      // 2 butterflies per thread
constexpr int kSlots = 2;             // sequences in flight per cluster
constexpr int kNMax = 512;            // longest sequence staged in shared memory
constexpr int kRing = 3;              // input ring depth
constexpr int kWarps = kNT / 32;

template <bool GRAD>
struct alignas(16) Smem {
    float buf[kSlots][kRing][GRAD ? 2 : 1][kNJ];  // 16 KB per plane
    float maxslot[kSlots][kRing][kCL];
    float w[kSlots][kNMax];
    float g[kSlots][GRAD ? kNMax : 4];
    float sf[kSlots][GRAD ? kNMax : 4];
    float wmax[kSlots][kWarps];
    float wacc[kSlots][kWarps];
    float lz[kSlots][kCL][2];
    unsigned long long full[kSlots][kRing];
};

// ---------------------------------------------------------------------------
// PTX wrappers.

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t num_clusters() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arm(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;"
        " selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void st_async4(uint32_t addr, float a, float b, float c, float d,
                                          uint32_t bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1,%2,%3,%4}, [%5];"
        ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void st_async1(uint32_t addr, float a, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                 ::"r"(addr), "r"(__float_as_uint(a)), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void st_cluster(uint32_t addr, float a) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(a) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: ~1 s, then BCJR_ERR_TIMEOUT in the status word.  Once any
// thread of the grid has failed, every later wait returns at once.
__device__ __forceinline__ void wait_full(uint32_t bar, uint32_t parity, int *status,
                                          bool &failed) {
    if (failed) return;
    if (mbar_try(bar, parity)) return;
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try(bar, parity)) return;
        if ((i & 63) == 0) {
            if (*reinterpret_cast<volatile int *>(status) != 0) {
                failed = true;
                return;
            }
            if (global_ns() - t0 > 1000000000ull) {
                atomicExch(status, 8 /* BCJR_ERR_TIMEOUT */);
                failed = true;
                return;
            }
        }
    }
}

__device__ __forceinline__ float max4(float a, float b, float c, float d) {
    return fmaxf(fmaxf(a, b), fmaxf(c, d));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Workspace of one (cluster, slot): float offsets.
struct SlotLayout {
    long hist;      // A rows: N x kG  (row t holds S_t, t >= 1)
    long hhist;     // H rows: N x kG  (backward only)
    long part;      // N x kCL per-step per-CTA partial sums
    long off;       // kCL x N doubles (alpha shifts O_t, one copy per CTA)
    long total;
};

__host__ __device__ inline SlotLayout slot_layout(int N, bool grad) {
    SlotLayout s;
    long p = 0;
    s.hist = p; p += (long)N * kG;
    s.hhist = p; if (grad) p += (long)N * kG;
    s.part = p; p += (long)N * kCL;
    p = (p + 3) & ~3L;
    s.off = p; p += 2L * kCL * N;
    s.total = (p + 63) & ~63L;   // 256-byte aligned slots
    return s;
}

template <bool GRAD>
__global__ void __cluster_dims__(kCL, 1, 1) __launch_bounds__(kNT, 1)
l16_kernel(const float *__restrict__ seq, const float *__restrict__ cb,
           const float *__restrict__ T_dev, const float *__restrict__ soft_in,
           const float *__restrict__ grad, int B, int N,
           float *__restrict__ out, float *__restrict__ logZ_out,
           float *__restrict__ ws, int *status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem<GRAD> &sm = *reinterpret_cast<Smem<GRAD> *>(smem_raw);
    constexpr int kPlanes = GRAD ? 2 : 1;
    constexpr uint32_t kBytes = kPlanes * kNJ * 4 + kCL * 4;

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t rank = cluster_rank();
    const uint32_t cid = cluster_id();
    const uint32_t ncl = num_clusters();
    const SlotLayout lay = slot_layout(N, GRAD);

    const float T = __ldg(T_dev);
    const float nk = -kLog2e / T;        // -kappa
    const float two_over_T = 2.f / T;

    // Codebook of my two butterflies: cbr[jj][p][c] = c(p 2^14 + 4 j + c).
    int jg[kJPT];
    float cbr[kJPT][4][4];
#pragma unroll
    for (int jj = 0; jj < kJPT; ++jj) {
        jg[jj] = (int)rank * kJPC + tid + kNT * jj;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(cb + p * kG + 4 * jg[jj]));
            cbr[jj][p][0] = v.x; cbr[jj][p][1] = v.y; cbr[jj][p][2] = v.z; cbr[jj][p][3] = v.w;
        }
    }

    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem_raw);
    uint32_t cbase[kCL];
#pragma unroll
    for (int r = 0; r < kCL; ++r) cbase[r] = mapa(sbase, r);
    auto soff = [&](const void *p) -> uint32_t {
        return (uint32_t)__cvta_generic_to_shared(p) - sbase;
    };

    if (tid == 0) {
        for (int z = 0; z < kSlots; ++z)
            for (int x = 0; x < kRing; ++x) mbar_init(sbase + soff(&sm.full[z][x]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster_sync();

    bool failed = false;
    uint32_t use[kSlots] = {0, 0};   // consumptions per slot (ring position, parity)

    for (long pair = cid; pair * kSlots < B; pair += ncl) {
        bool active[kSlots];
        long sidx[kSlots];
        float *slot_ws[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            sidx[z] = pair * kSlots + z;
            active[z] = sidx[z] < B;
            slot_ws[z] = ws + ((long)cid * kSlots + z) * lay.total;
        }
        __syncthreads();
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            for (int t = tid; t < N; t += kNT) {
                sm.w[z][t] = __ldg(seq + sidx[z] * N + t);
                if (GRAD) {
                    sm.g[z][t] = __ldg(grad + sidx[z] * N + t);
                    sm.sf[z][t] = __ldg(soft_in + sidx[z] * N + t);
                }
            }
        }
        __syncthreads();

        // ------------------------------------------------------------ alpha
        double O[kSlots] = {0.0, 0.0};
        float lzm[kSlots] = {kNegInf, kNegInf}, lzs[kSlots] = {0.f, 0.f};
        for (int t = 0; t < N; ++t) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                float *hist = slot_ws[z] + lay.hist;
                float *hhist = slot_ws[z] + lay.hhist;
                double *offs = reinterpret_cast<double *>(slot_ws[z] + lay.off) + (long)rank * N;
                float shift;
                float ain[kJPT][4], hin[kJPT][4];
                if (t == 0) {
                    shift = (float)kB;            // S_0 = A_0 = b
#pragma unroll
                    for (int jj = 0; jj < kJPT; ++jj)
#pragma unroll
                        for (int p = 0; p < 4; ++p) { ain[jj][p] = 0.f; hin[jj][p] = 0.f; }
                } else {
                    const int x = use[z] % kRing;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_full(bar, (use[z] / kRing) & 1, status, failed);
                    const float4 mx = *reinterpret_cast<const float4 *>(sm.maxslot[z][x]);
                    shift = max4(mx.x, mx.y, mx.z, mx.w);
#pragma unroll
                    for (int jj = 0; jj < kJPT; ++jj) {
                        const int jl = tid + kNT * jj;
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            ain[jj][p] = sm.buf[z][x][0][p * kJPC + jl] - shift;
                            hin[jj][p] = GRAD ? sm.buf[z][x][kPlanes - 1][p * kJPC + jl] : 0.f;
                        }
                    }
                    ++use[z];
                }
                O[z] += (double)shift;
                if (tid == 0) offs[t] = O[z];
                const int nb = use[z] % kRing;       // ring slot of the next consumption
                const float w = sm.w[z][t];
                float gt = 0.f, gs = 0.f;
                if (GRAD) {
                    gt = sm.g[z][t];
                    gs = gt * sm.sf[z][t];
                }
                const bool last = (t == N - 1);
                float lmax = kNegInf;
#pragma unroll
                for (int jj = 0; jj < kJPT; ++jj) {
                    float o4[4], h4[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float xv[4];
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            const float d = cbr[jj][p][c] - w;
                            xv[p] = fmaf(d, d * nk, ain[jj][p]);
                        }
                        const float m = max4(xv[0], xv[1], xv[2], xv[3]);
                        float e[4], s = 0.f;
#pragma unroll
                        for (int p = 0; p < 4; ++p) { e[p] = ex2(xv[p] - m); s += e[p]; }
                        o4[c] = m + lg2(s);
                        if (GRAD) {
                            float hf = 0.f;
#pragma unroll
                            for (int p = 0; p < 4; ++p)
                                hf = fmaf(e[p], fmaf(gt, cbr[jj][p][c], -gs) + hin[jj][p], hf);
                            h4[c] = hf * rcp(s);
                        }
                    }
                    lmax = fmaxf(lmax, max4(o4[0], o4[1], o4[2], o4[3]));
                    const int j = jg[jj];
                    if (!last) {
                        const uint32_t dst = (uint32_t)(j >> 8) & 3u;
                        const uint32_t o0 = soff(&sm.buf[z][nb][0][rank * kJPC + 4 * (j & 255)]);
                        const uint32_t bar = cbase[dst] + soff(&sm.full[z][nb]);
                        if (!failed) {
                            st_async4(cbase[dst] + o0, o4[0], o4[1], o4[2], o4[3], bar);
                            if (GRAD) {
                                const uint32_t o1 = soff(&sm.buf[z][nb][kPlanes - 1][rank * kJPC + 4 * (j & 255)]);
                                st_async4(cbase[dst] + o1, h4[0], h4[1], h4[2], h4[3], bar);
                            }
                        }
                        *reinterpret_cast<float4 *>(hist + (long)(t + 1) * kG + 4 * j) =
                            make_float4(o4[0], o4[1], o4[2], o4[3]);
                        if (GRAD)
                            *reinterpret_cast<float4 *>(hhist + (long)(t + 1) * kG + 4 * j) =
                                make_float4(h4[0], h4[1], h4[2], h4[3]);
                    } else {
#pragma unroll
                        for (int c = 0; c < 4; ++c) lse_merge(lzm[z], lzs[z], o4[c], 1.f);
                    }
                }
                if (!last) {
                    lmax = warp_max(lmax);
                    if (lane == 0) sm.wmax[z][warp] = lmax;
                }
                __syncthreads();
                if (!last && tid == 0) {
                    float cm = kNegInf;
                    for (int i = 0; i < kWarps; ++i) cm = fmaxf(cm, sm.wmax[z][i]);
                    const uint32_t om = soff(&sm.maxslot[z][nb][rank]);
                    if (!failed)
#pragma unroll
                        for (int r = 0; r < kCL; ++r)
                            st_async1(cbase[r] + om, cm, cbase[r] + soff(&sm.full[z][nb]));
                }
            }
        }

        // log2 Z = O_{N-1} + LSE over all 16384 values of S_N (four CTAs).
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            float m = lzm[z], s = lzs[z];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
                const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
                lse_merge(m, s, m2, s2);
            }
            if (lane == 0) { sm.wmax[z][warp] = m; sm.wacc[z][warp] = s; }
        }
        __syncthreads();
        if (tid == 0) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                float m = kNegInf, s = 0.f;
                for (int i = 0; i < kWarps; ++i) lse_merge(m, s, sm.wmax[z][i], sm.wacc[z][i]);
#pragma unroll
                for (int r = 0; r < kCL; ++r) {
                    st_cluster(cbase[r] + soff(&sm.lz[z][rank][0]), m);
                    st_cluster(cbase[r] + soff(&sm.lz[z][rank][1]), s);
                }
            }
        }
        cluster_sync();
        double logZ2[kSlots] = {0.0, 0.0};
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            float m = kNegInf, s = 0.f;
#pragma unroll
            for (int r = 0; r < kCL; ++r) lse_merge(m, s, sm.lz[z][r][0], sm.lz[z][r][1]);
            logZ2[z] = O[z] + (double)m + (double)log2f(s);
            if (!GRAD && rank == 0 && tid == 0 && logZ_out)
                logZ_out[sidx[z]] = (float)(logZ2[z] * (double)kLn2);
        }

        // ------------------------------------------------------------- beta
        double U[kSlots] = {0.0, 0.0};
        for (int t = N - 2; t >= -1; --t) {
            const int tn = t + 1;
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                const float *hist = slot_ws[z] + lay.hist;
                const float *hhist = slot_ws[z] + lay.hhist;
                const double *offs = reinterpret_cast<const double *>(slot_ws[z] + lay.off) + (long)rank * N;
                float *part = slot_ws[z] + lay.part;
                float sigma;
                float bin[kJPT][4], bbin[kJPT][4];
                if (t == N - 2) {
                    sigma = 0.f;
#pragma unroll
                    for (int jj = 0; jj < kJPT; ++jj)
#pragma unroll
                        for (int c = 0; c < 4; ++c) { bin[jj][c] = 0.f; bbin[jj][c] = 0.f; }
                } else {
                    const int x = use[z] % kRing;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_full(bar, (use[z] / kRing) & 1, status, failed);
                    const float4 mx = *reinterpret_cast<const float4 *>(sm.maxslot[z][x]);
                    sigma = max4(mx.x, mx.y, mx.z, mx.w);
#pragma unroll
                    for (int jj = 0; jj < kJPT; ++jj) {
                        const int jl = tid + kNT * jj;
                        const float4 v = *reinterpret_cast<const float4 *>(&sm.buf[z][x][0][4 * jl]);
                        bin[jj][0] = v.x - sigma; bin[jj][1] = v.y - sigma;
                        bin[jj][2] = v.z - sigma; bin[jj][3] = v.w - sigma;
                        if (GRAD) {
                            const float4 u = *reinterpret_cast<const float4 *>(&sm.buf[z][x][kPlanes - 1][4 * jl]);
                            bbin[jj][0] = u.x; bbin[jj][1] = u.y; bbin[jj][2] = u.z; bbin[jj][3] = u.w;
                        } else {
#pragma unroll
                            for (int c = 0; c < 4; ++c) bbin[jj][c] = 0.f;
                        }
                    }
                    ++use[z];
                }
                U[z] += (double)sigma;
                const double Oa = tn > 0 ? offs[tn - 1] : 0.0;
                const float C = (float)(logZ2[z] - Oa - U[z]);
                const int nb = use[z] % kRing;
                const float w = sm.w[z][tn];
                float gt = 0.f, st = 0.f, gs = 0.f;
                if (GRAD) {
                    gt = sm.g[z][tn];
                    st = sm.sf[z][tn];
                    gs = gt * st;
                }
                float acc = 0.f, lmax = kNegInf;
#pragma unroll
                for (int jj = 0; jj < kJPT; ++jj) {
                    const int j = jg[jj];
                    float a4[4], h4[4];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        a4[p] = tn > 0 ? __ldcg(hist + (long)tn * kG + p * kNJ + j) : (float)kB;
                        h4[p] = (GRAD && tn > 0) ? __ldcg(hhist + (long)tn * kG + p * kNJ + j) : 0.f;
                    }
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        float xv[4], yv[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const float d = cbr[jj][p][c] - w;
                            xv[c] = fmaf(d, d * nk, bin[jj][c]);
                            if (GRAD) yv[c] = fmaf(gt, cbr[jj][p][c], -gs) + bbin[jj][c];
                        }
                        const float m = max4(xv[0], xv[1], xv[2], xv[3]);
                        float e[4], s = 0.f;
#pragma unroll
                        for (int c = 0; c < 4; ++c) { e[c] = ex2(xv[c] - m); s += e[c]; }
                        const float f = ex2(m + a4[p] - C);
                        float ob = 0.f, bbo = 0.f;
                        if (t >= 0) ob = m + lg2(s);
                        if (!GRAD) {
                            float ec = 0.f;
#pragma unroll
                            for (int c = 0; c < 4; ++c) ec = fmaf(e[c], cbr[jj][p][c], ec);
                            acc = fmaf(f, ec, acc);
                        } else {
                            float ey = 0.f, dl = 0.f;
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                ey = fmaf(e[c], yv[c], ey);
                                dl = fmaf(e[c] * (yv[c] + h4[p]), cbr[jj][p][c] - st, dl);
                            }
                            bbo = ey * rcp(s);
                            acc = fmaf(f, dl, acc);
                        }
                        if (t >= 0) {
                            lmax = fmaxf(lmax, ob);
                            if (!failed) {
                                const uint32_t bar = cbase[p] + soff(&sm.full[z][nb]);
                                st_async1(cbase[p] + soff(&sm.buf[z][nb][0][j]), ob, bar);
                                if (GRAD) st_async1(cbase[p] + soff(&sm.buf[z][nb][kPlanes - 1][j]), bbo, bar);
                            }
                        }
                    }
                }
                acc = warp_sum(acc);
                if (t >= 0) lmax = warp_max(lmax);
                if (lane == 0) {
                    sm.wacc[z][warp] = acc;
                    sm.wmax[z][warp] = lmax;
                }
                __syncthreads();
                if (tid == 0) {
                    if (t >= 0) {
                        float cm = kNegInf;
                        for (int i = 0; i < kWarps; ++i) cm = fmaxf(cm, sm.wmax[z][i]);
                        const uint32_t om = soff(&sm.maxslot[z][nb][rank]);
                        if (!failed)
#pragma unroll
                            for (int r = 0; r < kCL; ++r)
                                st_async1(cbase[r] + om, cm, cbase[r] + soff(&sm.full[z][nb]));
                    }
                    float sacc = 0.f;
                    for (int i = 0; i < kWarps; ++i) sacc += sm.wacc[z][i];
                    part[(long)tn * kCL + rank] = sacc;
                }
            }
        }

        // Per-step partials of the four CTAs, added in a fixed order.
        cluster_sync();
        if (rank == 0) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                const float *part = slot_ws[z] + lay.part;
                for (int tn = tid; tn < N; tn += kNT) {
                    const float4 v = __ldcg(reinterpret_cast<const float4 *>(part + (long)tn * kCL));
                    const float sum = ((v.x + v.y) + v.z) + v.w;
                    out[sidx[z] * N + tn] = GRAD ? two_over_T * sum : sum;
                }
            }
        }
    }
    cluster_sync();
}

}  // namespace l16

// ---------------------------------------------------------------------------
// Host side.

namespace {

template <bool GRAD>
int l16_max_clusters() {
    static int cached[2][64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    int &c = cached[GRAD ? 1 : 0][dev];
    if (c > 0) return c;
    const size_t smem = sizeof(l16::Smem<GRAD>);
    if (cudaFuncSetAttribute(l16::l16_kernel<GRAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(sms / l16::kCL * l16::kCL), 1, 1);
    cfg.blockDim = dim3(l16::kNT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = l16::kCL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, l16::l16_kernel<GRAD>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    c = n;
    return n;
}

}  // namespace

bool l16_applicable(int B, int N, int L, int BB, int V) {
    (void)B;
    return L == l16::kL && BB == l16::kB && V == 1 && N >= 2 && N <= l16::kNMax;
}

int l16_clusters(int B, int mode) {
    const int maxc = (mode == kModeBackward) ? l16_max_clusters<true>() : l16_max_clusters<false>();
    const long pairs = ((long)B + l16::kSlots - 1) / l16::kSlots;
    long n = maxc;
    if (n > pairs) n = pairs;
    return (int)n;
}

size_t l16_workspace_bytes(int B, int N, int mode) {
    const int ncl = l16_clusters(B, mode);
    if (ncl <= 0) return 0;
    const long slot = l16::slot_layout(N, mode == kModeBackward).total;
    return (size_t)ncl * l16::kSlots * slot * 4;
}

cudaError_t launch_l16(const LaunchArgs &a) {
    const bool grad = (a.mode == kModeBackward);
    const int ncl = l16_clusters(a.B, a.mode);
    if (ncl <= 0) return cudaErrorInvalidConfiguration;
    const long slot = l16::slot_layout(a.N, grad).total;
    if ((size_t)ncl * l16::kSlots * slot * 4 > a.ws_data_bytes) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)(ncl * l16::kCL)), block(l16::kNT);
    float *ws = reinterpret_cast<float *>(a.ws_data);
    if (grad) {
        l16::l16_kernel<true><<<grid, block, sizeof(l16::Smem<true>), a.stream>>>(
            a.seq, a.cb, a.T_dev, a.soft_in, a.grad, a.B, a.N, a.dseq, nullptr, ws, a.status);
    } else {
        l16::l16_kernel<false><<<grid, block, sizeof(l16::Smem<false>), a.stream>>>(
            a.seq, a.cb, a.T_dev, nullptr, nullptr, a.B, a.N, a.soft, a.logZ, ws, a.status);
    }
    return cudaGetLastError();
}

}  // namespace bcjr
