// Hard (min-sum) Viterbi for the V=1 trellis L=16, k=2 (b = 2, four
// predecessors per state): src/viterbi/encode.py:47-90 (viterbi_encode) and
// :258-310 (viterbi_encode_v at V=1).  Same recursion and arithmetic as the
// one-block kernel of bcjr_viterbi.cu:
//
//   cum_t(s) = m_t(s >> 2) + (c(s) - w_t)^2,   m_t(h) = min_p cum_{t-1}(p 2^14 + h),   m_0 = 0
//
// in fp32 with d = c - w, d * d and min + local each rounded (no fused
// multiply-add: the sums are scalar __fadd_rn, add2_sep of bcjr_cluster.cuh,
// which the compiler does not merge with the f32x2 products), no
// renormalisation, the lowest p and the lowest final state on ties, so walks
// are bit-identical to the reference encoder's.
//
// Work decomposition.  With M = 14 the 2^16 states split into 4096
// butterflies r: states s = p 2^14 + 4 r + c, p, c in 0..3.  Butterfly r
// reads the group minima m_t(p 2^12 + r) of its four predecessor groups and
// writes m_{t+1}(4 r + c) for its four successor groups, with the winning p
// of each.  CTA k of a 4-CTA cluster owns butterflies [1024 k, 1024 k + 1024);
// a thread owns two whole butterflies (32 states, codebook values in
// registers as f32x2 pairs along c).
//
// Exchange.  Output group 4 r + c is input p' = r >> 10 (the producer's CTA
// rank) of butterfly (4 r + c) mod 4096, which CTA (r >> 8) mod 4 owns.  The
// consumer's input ring is laid out [p'][1024 butterflies], so a
// butterfly's four outputs are contiguous there: one 16-byte st.async ...
// complete_tx per butterfly, a warp's 32 butterflies one 512-byte block to
// one consumer.  Consumers read their four inputs per butterfly with
// conflict-free 4-byte loads.  As in bcjr_vit_b4.cu, every warp also sends
// one token per consumer CTA after its step (part of the consumption's byte
// count), so a producer that has a complete consumption u knows that every
// warp has finished reading consumption u-1, the ring buffer it writes next.
// Waits are bounded (about 1 s, then BCJR_ERR_TIMEOUT in the status word).
//
// Backpointers: the four 2-bit winners of a butterfly pack into one byte
// (bits 2c, 2c+1 for output group 4 r + c), 4096 bytes per step and
// sequence, written to HBM; a second kernel walks back, one thread per
// sequence, writing bitstream, start state, reconstruction and MSE.
#include <cfloat>
#include <cstdint>

#include "../../include/bcjr_b200.h"
#include "bcjr_cluster.cuh"
#include "bcjr_kernels.h"

namespace bcjr {
namespace vb2 {

using namespace clu;

constexpr int kL = 16;
constexpr int kB = 2;
constexpr int kM = kL - kB;           // 14
constexpr int kG = 1 << kM;           // 16384 groups
constexpr int kNR = kG >> kB;         // 4096 butterflies
constexpr int kCL = 4;
constexpr int kRPC = kNR / kCL;       // 1024 butterflies per CTA
constexpr int kIn = 4 * kRPC;         // 4096 inputs per CTA per step, [p][butterfly]
#ifndef BCJR_VIT2_NT
#define BCJR_VIT2_NT 512
#endif
// 512 threads, two butterflies each: measured on B200 (4096 x 256) 24.8 ms
// against 33.8 ms for 256 threads with four (fewer warps to hide latency).
constexpr int kNT = BCJR_VIT2_NT;     // threads per CTA (256 or 512)
constexpr int kWarps = kNT / 32;
constexpr int kBPT = kRPC / kNT;      // butterflies per thread
static_assert(kNT == 256 || kNT == 512, "a warp's butterflies must go to one consumer CTA");
#ifndef BCJR_VIT2_SLOTS
#define BCJR_VIT2_SLOTS 4
#endif
constexpr int kSlots = BCJR_VIT2_SLOTS;   // sequences in flight per cluster
constexpr int kNMax = 512;

struct alignas(128) Smem {
    float buf[kSlots][2][kIn];            // input ring: group minima of the previous step
    float tok[kSlots][2][kCL * kWarps];   // per-warp tokens riding with the data
    float zero[kIn];                      // inputs of step 0 (m_0 = 0): plain loads, no selects
    float w[kSlots][kNMax];
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
vit_b2_kernel(const float *__restrict__ seq, const float *__restrict__ cb, int B, int N,
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

    // my butterflies: local rl = tid + kNT j, global r = 1024 rank + rl
    int rg[kBPT];
    uint32_t o_cta[kBPT], o_off[kBPT];    // consumer CTA (shared::cluster base) and byte offset
    F2 C[kBPT][4][2];                     // c(p 2^14 + 4 r + c), pairs (c, c + 1)
#pragma unroll
    for (int j = 0; j < kBPT; ++j) {
        const int rl = tid + kNT * j;
        rg[j] = (int)rank * kRPC + rl;
        o_cta[j] = mapa(sbase, (uint32_t)(rl >> 8));
        o_off[j] = 4u * (rank * (uint32_t)kRPC + 4u * (uint32_t)(rl & 255));
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(cb + ((size_t)p << kM)) + rg[j]);
            C[j][p][0] = mk(v.x, v.y);
            C[j][p][1] = mk(v.z, v.w);
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

    for (long grp = cid; grp * kSlots < B; grp += ncl) {
        bool active[kSlots];
        long sidx[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            sidx[z] = grp * kSlots + z;
            active[z] = sidx[z] < B;
        }
        __syncthreads();
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            for (int t = tid; t < N; t += kNT) sm.w[z][t] = __ldg(seq + sidx[z] * N + t);
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
                const float *in = sm.zero;    // m_0 = 0
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
                const F2 W = bc(sm.w[z][t]);
                // backpointers of the groups at step t + 1 (step 0's are all 0)
                unsigned char *bpt = bp_all + ((size_t)sidx[z] * N + t + 1) * kNR;
                const bool send = !last && !failed && !drop;
#pragma unroll
                for (int j = 0; j < kBPT; ++j) {
                    const int rl = tid + kNT * j;
                    F2 x[4][2];                       // cum_t of my 16 states
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const F2 A = bc(in[p * kRPC + rl]);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const F2 d = sub2(C[j][p][h], W);
                            x[p][h] = add2_sep(A, mul2(d, d));
                        }
                    }
                    float o[4];
                    uint32_t packed = 0;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float m = (c & 1) ? x[0][c >> 1].y : x[0][c >> 1].x;
                        uint32_t bi = 0;
#pragma unroll
                        for (int p = 1; p < 4; ++p) {
                            const float v = (c & 1) ? x[p][c >> 1].y : x[p][c >> 1].x;
                            if (v < m) { m = v; bi = (uint32_t)p << (2 * c); }
                        }
                        o[c] = m;
                        packed |= bi;
                    }
                    if (!last) {
                        bpt[rg[j]] = (unsigned char)packed;
                        if (send)
                            st_async4(o_cta[j] + soff(&sm.buf[z][nb][0]) + o_off[j], o[0], o[1], o[2],
                                      o[3], o_cta[j] + soff(&sm.full[z][nb]));
                    } else {
                        // final state: lowest-index minimum over my states
                        // s = p 2^14 + 4 r + c
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int s = (p << kM) | (4 * rg[j] + 2 * h);
                                arg_better(fv[z], fi[z], x[p][h].x, s);
                                arg_better(fv[z], fi[z], x[p][h].y, s + 1);
                            }
                        }
                    }
                }
                if (send) {
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
                const uint32_t peer = mapa(sbase, 0u);
                st_cluster(peer + soff(&sm.cv[z][rank]), v);
                st_cluster_u32(peer + soff(&sm.ci[z][rank]), (uint32_t)i);
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

// Walk back, one thread per sequence: state at t-1 = (bp_t(s >> 2) << 14) | (s >> 2).
__global__ void vit_b2_backtrace(const unsigned char *__restrict__ bp_all,
                                 const int *__restrict__ final_states,
                                 const float *__restrict__ seq, const float *__restrict__ cb, int B,
                                 int N, int *__restrict__ bits, int *__restrict__ starts,
                                 float *__restrict__ recon, float *__restrict__ mse,
                                 const int *__restrict__ status) {
    const long b = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    // After a failed wait the walk is not the optimum: NaN reconstructions
    // and MSEs (selected, not added, so that reconstructions stay exact
    // codebook values otherwise).  The masks keep every index in range
    // whatever the arrays hold (unwritten after a timeout).
    const bool failed = poison_value(false, status) != 0.f;
    const float nanv = __int_as_float(0x7fffffff);
    int s = final_states[b] & ((1 << kL) - 1);
    double e2 = 0.0;
    for (int t = N - 1; t >= 0; --t) {
        const long i = b * N + t;
        bits[i] = s & 3;
        const float r = __ldg(cb + s);
        recon[i] = failed ? nanv : r;
        const double d = (double)r - (double)__ldg(seq + i);
        e2 += d * d;
        const int h = s >> kB;
        if (t > 0) {
            const int byte = bp_all[((size_t)b * N + t) * kNR + (h >> 2)];
            s = (((byte >> (2 * (h & 3))) & 3) << kM) | h;
        } else {
            s = h;   // step 0's backpointers are all 0
        }
    }
    starts[b] = s;
    mse[b] = failed ? nanv : (float)(e2 / (double)N);
}

}  // namespace vb2

// ---------------------------------------------------------------------------
// Host side (called by bcjr_viterbi in bcjr_viterbi.cu).

namespace {

int vit_b2_max_clusters() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev] > 0) return cached[dev];
    if (cudaFuncSetAttribute(vb2::vit_b2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(vb2::Smem)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(sms / vb2::kCL * vb2::kCL), 1, 1);
    cfg.blockDim = dim3(vb2::kNT, 1, 1);
    cfg.dynamicSmemBytes = sizeof(vb2::Smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = vb2::kCL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, vb2::vit_b2_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cached[dev] = n;
    return n;
}

// Sequences per forward + walk-back launch pair: their backpointers take at
// most 1 GiB (N * 4096 bytes per sequence), in whole waves of the grid.
long vit_b2_chunk(int B, int N) {
    long c = (1L << 18) / (N > 0 ? N : 1);
    const long wave = (long)vit_b2_max_clusters() * vb2::kSlots;
    if (wave > 0 && c >= wave) c -= c % wave;
    if (c < 1) c = 1;
    if (c > B) c = B > 0 ? B : 1;
    return c;
}

}  // namespace

bool vit_b2_applicable(int N, int L, int k, int V, const void *cb) {
    return L == vb2::kL && k == vb2::kB && V == 1 && N >= 1 && N <= vb2::kNMax &&
           (reinterpret_cast<uintptr_t>(cb) & 15u) == 0 && vit_b2_max_clusters() > 0;
}

int vit_b2_launches(int B, int N) {
    if (B <= 0) return 0;
    const long c = vit_b2_chunk(B, N);
    return (int)(2 * ((B + c - 1) / c));
}

size_t vit_b2_workspace_bytes(int B, int N) {
    const long c = vit_b2_chunk(B, N);
    return 256 + (size_t)c * N * vb2::kNR + (size_t)c * 4;
}

cudaError_t launch_vit_b2(const float *seq, const float *cb, int B, int N, int *bits,
                          int *starts, float *recon, float *mse, void *ws, size_t ws_bytes,
                          int *status, int drop_sends, cudaStream_t st) {
    const long c = vit_b2_chunk(B, N);
    unsigned char *bp = static_cast<unsigned char *>(ws) + 256;
    int *finals = reinterpret_cast<int *>(bp + (size_t)c * N * vb2::kNR);
    if (ws_bytes < vit_b2_workspace_bytes(B, N)) return cudaErrorInvalidValue;
    const int maxc = vit_b2_max_clusters();
    if (maxc <= 0) return cudaErrorInvalidConfiguration;
    for (long b0 = 0; b0 < B; b0 += c) {
        const int nb = (int)((B - b0) < c ? (B - b0) : c);
        long ncl = (nb + vb2::kSlots - 1) / vb2::kSlots;
        if (ncl > maxc) ncl = maxc;
        vb2::vit_b2_kernel<<<(unsigned)(ncl * vb2::kCL), vb2::kNT, sizeof(vb2::Smem), st>>>(
            seq + b0 * N, cb, nb, N, bp, finals, status, drop_sends);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        vb2::vit_b2_backtrace<<<(nb + 127) / 128, 128, 0, st>>>(
            bp, finals, seq + b0 * N, cb, nb, N, bits + b0 * N, starts + b0, recon + b0 * N,
            mse + b0, status);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace bcjr
