// Production kernel for the QTIP trellis L=16, k=2, V=2 (b = 4, 16
// predecessors per state): one 4-CTA thread-block cluster per pair of
// sequences, one CTA per SM.  Same exchange machinery as the b = 2 kernel
// (bcjr_l16.cu); the work decomposition is built around 16 x 16 butterflies.
//
// Work decomposition
// ------------------
// With M = 12, the 2^16 states split into 256 butterflies
//     r in [0, 256):  states s = p * 2^12 + 16 r + c,   p, c in 0..15.
// In the forward (alpha) direction butterfly r reads the 16 group values
// A_t(p 2^8 + r) and writes A_{t+1}(16 r + c); in the backward (beta)
// direction it reads Bt_{t+1}(16 r + c) and writes Bt_t(p 2^8 + r).  CTA k
// of the cluster owns butterflies [64 k, 64 k + 64): 16384 states, 32 per
// thread.  A butterfly is too large for one thread, so the two sweeps split
// it differently, each so that its soft-min is thread-local:
//   alpha: a thread owns one c and all 16 p of two butterflies r, r + 16;
//   beta:  a thread owns one p and all 16 c of two butterflies r, r + 1.
// Each thread loads the 64 codebook values (2 per state) of its states into
// registers at the start of each sweep.  All FMA-pipe work is f32x2 pairs
// along the reduced index (pairs of p in alpha, pairs of c in beta).
//
// Arithmetic (as in bcjr_l16.cu)
// ------------------------------
// Costs in squared-distance units, a = -A / kappa, kappa = log2(e)/T; the
// energy plus message of a state is  x = d0^2 + d1^2 + a  with the exact
// differences d = c(s) - w_t.  Soft-min over 16 states:
// m - lg2(sum 2^(kappa (m - x))) / kappa,  m = min x.  Each consumer
// renormalises by the global minimum of the previous step's outputs (it
// subtracts it from its outputs; shifts accumulate in double).
//
// Exchange and layouts
// --------------------
// Producers push outputs into the consumer CTA's shared-memory ring with
// st.async ... mbarrier::complete_tx (double-buffered, byte-counted, bounded
// waits, free-running warps that ship their minimum cost with their data;
// see bcjr_l16.cu).  Each warp's outputs go to one consumer CTA as one
// contiguous 256-byte block:
//   alpha ring [p/2][64 butterflies][p%2]: a thread's two outputs are the
//     p and p+1 inputs of one consumer butterfly (8-byte store); consumers
//     read (p, p+1) pairs with broadcast 8-byte loads;
//   beta ring [64 butterflies][16 c], 16-byte chunks XOR-swizzled by
//     (butterfly/2) % 8: a thread's two outputs are the c and c+1 inputs of
//     one consumer butterfly; consumers read 128 contiguous bytes per lane
//     without bank conflicts.
// The alpha history row t (A_t, and H_t for the gradient) is kept in global
// memory in the same layout as the consumers' alpha rings, chunk k holding
// CTA k's ring: producers write their outputs there too (each warp one
// contiguous 256-byte store per plane), and the beta sweep loads its own
// chunk back with one TMA bulk load per step (no multicast).  Per-step partial sums of
// soft / d_seq (2 components) are written per warp and added by CTA 0 in a
// fixed order: results are deterministic.
//
// Every wait is bounded (about 1 s); on timeout the kernel records
// BCJR_ERR_TIMEOUT in the workspace status word, stops waiting and sending,
// runs to completion, and writes NaN into the outputs it writes from then on
// (poison_value).  The recursions are documented in bcjr_common.cuh.
#include <cstdint>

#include "bcjr_cluster.cuh"
#include "bcjr_kernels.h"

namespace bcjr {
namespace b4 {

using namespace clu;

constexpr int kL = 16;
constexpr int kB = 4;                 // branch bits b = kV
constexpr int kV = 2;
constexpr int kG = 1 << (kL - kB);    // 4096 groups
constexpr int kNR = kG >> kB;         // 256 butterflies
constexpr int kCL = 4;                // CTAs per cluster
constexpr int kRPC = kNR / kCL;       // 64 butterflies per CTA
constexpr int kIn = kRPC * 16;        // 1024 inputs per CTA per step and plane
#ifndef BCJR_B4_VT
#define BCJR_B4_VT 2
#endif
constexpr int kVT = BCJR_B4_VT;       // work units ("virtual threads") per thread
constexpr int kNT = 512 / kVT;        // threads per CTA
constexpr int kWarps = kNT / 32;      // warps per CTA
// Three sequences in flight: measured on B200 (4096 x 128, V=2) 2 slots
// 5.37e12 transitions/s, 3 slots 5.46e12 (no spills at 255 registers).
#ifndef BCJR_B4_SLOTS
#define BCJR_B4_SLOTS 3
#endif
constexpr int kSlots = BCJR_B4_SLOTS; // sequences in flight per cluster
constexpr int kNMax = 512;            // longest sequence staged in shared memory

template <bool GRAD>
struct alignas(128) Smem {
    static constexpr int kPlanes = GRAD ? 2 : 1;
    float buf[kSlots][2][kPlanes][kIn];   // input ring (4 KB per plane)
    float hst[kSlots][kPlanes][kIn];      // history chunk staged by TMA (alpha layout)
    float zero[kPlanes][kIn];             // all-zero inputs of the first step of each sweep
    double offs[kSlots][kNMax];           // alpha shifts O_t
    float maxslot[kSlots][2][kCL * kWarps];   // per-warp minimum cost riding with the data
    float2 w[kSlots][kNMax];
    float2 g[kSlots][GRAD ? kNMax : 1];
    float2 sf[kSlots][GRAD ? kNMax : 1];
    float wmin[kSlots][kWarps];
    float wacc[kSlots][kWarps];
    float lz[kSlots][kCL][2];
    unsigned long long full[kSlots][2];
    unsigned long long hbar[kSlots];
    int cnt[kSlots][2];                   // warps finished with the step (backward sweep)
    int hiss[kSlots];                     // TMA row loads issued per slot
};

// Float offset of input (butterfly rl, c) in a beta-ring plane.
__device__ __forceinline__ uint32_t beta_off(uint32_t rl, uint32_t c) {
    const uint32_t chunk = (((rl & 1u) << 2) | (c >> 2)) ^ ((rl >> 1) & 7u);
    return (rl >> 1) * 32u + chunk * 4u + (c & 3u);
}

// Minimum of the kCL * kWarps per-warp minima riding with a consumption
// (called by whole warps).
__device__ __forceinline__ float cluster_min(const float *m, int lane) {
    float v = m[lane];
#pragma unroll
    for (int i = 32; i < kCL * kWarps; i += 32) v = fminf(v, m[lane + i]);
    return redux_min(v);
}

__device__ __forceinline__ float min16(const F2 (&x)[8]) {
    const float a = min3(x[0].x, x[0].y, x[1].x);
    const float b = min3(x[1].y, x[2].x, x[2].y);
    const float c = min3(x[3].x, x[3].y, x[4].x);
    const float d = min3(x[4].y, x[5].x, x[5].y);
    const float e = min3(x[6].x, x[6].y, x[7].x);
    return fminf(min3(a, b, c), min3(d, e, x[7].y));
}

__device__ __forceinline__ F2 sum8(const F2 (&e)[8]) {
    return add2(add2(add2(e[0], e[1]), add2(e[2], e[3])),
                add2(add2(e[4], e[5]), add2(e[6], e[7])));
}

// Workspace of one (cluster, slot): float offsets.
struct SlotLayout {
    long hist;      // N rows x [kCL][planes][kIn]: alpha cost rows S_t (+ H_t)
    long part;      // N x kCL x kWarps x 2 per-step per-warp partial sums
    long total;
};

__host__ __device__ inline SlotLayout slot_layout(int N, bool grad) {
    SlotLayout s;
    long p = 0;
    s.hist = p; p += (long)N * kCL * (grad ? 2 : 1) * kIn;
    s.part = p; p += (long)N * kCL * kWarps * 2;
    s.total = (p + 63) & ~63L;   // 256-byte aligned slots
    return s;
}

template <bool GRAD>
__global__ void __cluster_dims__(kCL, 1, 1) __launch_bounds__(kNT, 1)
b4_kernel(const float *__restrict__ seq, const float *__restrict__ cb,
          const float *__restrict__ T_dev, const float *__restrict__ soft_in,
          const float *__restrict__ grad, int B, int N,
          float *__restrict__ out, float *__restrict__ logZ_out,
          float *__restrict__ ws, int *status, int drop_sends) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    using SM = Smem<GRAD>;
    SM &sm = *reinterpret_cast<SM *>(smem_raw);
    constexpr int kPlanes = SM::kPlanes;
    constexpr uint32_t kBytes = kPlanes * kIn * 4 + kCL * kWarps * 4;   // per consumption
    constexpr uint32_t kChunkBytes = kPlanes * kIn * 4;          // history chunk per CTA
    constexpr long kRowFloats = (long)kCL * kPlanes * kIn;

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t rank = cluster_rank();
    const uint32_t cid = cluster_id();
    const uint32_t ncl = num_clusters();
    const SlotLayout lay = slot_layout(N, GRAD);

    const float T = __ldg(T_dev);
    const float kap = kLog2e / T;           // kappa
    const float ikap = T / kLog2e;
    const float two_over_T = 2.f / T;
    const float a0 = -(float)kB * ikap;     // cost of A_0 = b everywhere
    const bool bad_T = bad_temperature(T);  // outputs NaN (poison_value)

    // Each thread carries kVT work units; unit h of thread (warp, lane) is
    // virtual warp vw = warp + kWarps h, lane `lane` of a 512-unit layout.
    // Alpha-sweep ownership of a unit: one c, butterflies rla and rla + 16 (local).
    // Beta-sweep ownership: p = vw, butterflies 2 lane and 2 lane + 1 (local),
    // the same butterflies for every unit of the thread.
    int ac[kVT], arl[kVT], bp[kVT];
    uint32_t a_off[kVT], a_base[kVT], b_off[kVT], b_base[kVT];
    const int brl = 2 * lane;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem_raw);
#pragma unroll
    for (int h = 0; h < kVT; ++h) {
        const int vw = warp + kWarps * h;
        ac[h] = lane & 15;
        const int aq = 2 * vw + (lane >> 4);
        arl[h] = (aq & 15) + 32 * (aq >> 4);
        // alpha outputs: consumer CTA, and float offset in its alpha-ring plane
        a_base[h] = mapa(sbase, (uint32_t)((aq & 15) >> 2));
        a_off[h] = 2u * ((uint32_t)(2 * (int)rank + (aq >> 4)) * kRPC + (uint32_t)(16 * (aq & 3) + ac[h]));
        bp[h] = vw;
        b_base[h] = mapa(sbase, (uint32_t)(vw >> 2));
        b_off[h] = beta_off((uint32_t)(16 * (vw & 3) + 4 * (int)rank + (lane >> 3)),
                            (uint32_t)(2 * (lane & 7)));
    }
    // history-row chunk (global) of my alpha outputs: consumer CTA index
    uint32_t a_dst[kVT];
#pragma unroll
    for (int h = 0; h < kVT; ++h) {
        const int aq = 2 * (warp + kWarps * h) + (lane >> 4);
        a_dst[h] = (uint32_t)((aq & 15) >> 2);
    }

    // Codebook of the current sweep's 32 states per unit, f32x2 pairs along
    // the reduced index: C0 = first component, C1 = second.
    F2 C0[kVT][2][8], C1[kVT][2][8];
    const float2 *cb2 = reinterpret_cast<const float2 *>(cb);
    auto load_alpha_cb = [&]() {
#pragma unroll
        for (int h = 0; h < kVT; ++h)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = (int)rank * kRPC + arl[h] + 16 * rr;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float *u = reinterpret_cast<const float *>(cb2 + (2 * i) * kG + 16 * r + ac[h]);
                const float *v = reinterpret_cast<const float *>(cb2 + (2 * i + 1) * kG + 16 * r + ac[h]);
                C0[h][rr][i] = ldg_pair(u, v);
                C1[h][rr][i] = ldg_pair(u + 1, v + 1);
            }
        }
    };
    auto load_beta_cb = [&]() {
#pragma unroll
        for (int h = 0; h < kVT; ++h)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = (int)rank * kRPC + brl + rr;
            const float *base = reinterpret_cast<const float *>(cb2 + bp[h] * kG + 16 * r);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                C0[h][rr][i] = ldg_pair(base + 4 * i, base + 4 * i + 2);
                C1[h][rr][i] = ldg_pair(base + 4 * i + 1, base + 4 * i + 3);
            }
        }
    };

    auto soff = [&](const void *p) -> uint32_t {
        return (uint32_t)__cvta_generic_to_shared(p) - sbase;
    };

    for (int i = tid; i < kPlanes * kIn; i += kNT) (&sm.zero[0][0])[i] = 0.f;
    if (tid == 0) {
        for (int z = 0; z < kSlots; ++z) {
            sm.hiss[z] = 0;
            for (int x = 0; x < 2; ++x) {
                sm.cnt[z][x] = 0;
            }
        }
        for (int z = 0; z < kSlots; ++z) {
            for (int x = 0; x < 2; ++x) mbar_init(sbase + soff(&sm.full[z][x]), 1);
            mbar_init(sbase + soff(&sm.hbar[z]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    cluster_sync();

    bool failed = false;
    // Test-only fault injection (BCJR_OPT_TEST_DROP_SENDS): CTA rank 1 never
    // sends its alpha-sweep outputs, so every consumer's bounded wait expires.
    const bool drop = drop_sends != 0 && rank == 1;
    uint32_t use[kSlots], hcnt[kSlots];   // ring consumptions / TMA row loads waited, per slot
#pragma unroll
    for (int z = 0; z < kSlots; ++z) use[z] = hcnt[z] = 0;

    // TMA load of this CTA's chunk of history row tn into the staging buffer
    // of slot z; completion on hbar[z].
    auto issue_rows = [&](int z, int tn, float *const *slot_ws) {
        const uint32_t hb = sbase + soff(&sm.hbar[z]);
        if (failed) return;
        atomicAdd(&sm.hiss[z], 1);
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arm(hb, kChunkBytes);
        const float *src = slot_ws[z] + lay.hist + (long)tn * kRowFloats + rank * (kPlanes * kIn);
        bulk_g2s(sbase + soff(&sm.hst[z][0][0]), src, kChunkBytes, hb);
    };

    // End of a step, per warp (no block barrier): the warp's minimum output
    // cost goes into the step's shared-memory minimum, its two partial sums
    // into global memory, and the last warp to arrive sends the CTA minimum
    // to the four consumers and, in the beta sweep, issues the next TMA row.
    auto finish_step = [&](int z, int nb, bool send, float lmin, float *part_row, F2 acc,
                           int rows_tn, float *const *slot_ws) {
        // The warp's minimum output cost goes to every consumer CTA with the
        // data (part of the consumption's byte count).  Sent after the warp
        // has read this step's inputs, it also tells every producer that the
        // warp is done with the ring buffer the producer writes next.
        const float wmin = send ? redux_min(lmin) : 0.f;
        if (send && lane < kCL && !failed) {
            const uint32_t peer = mapa(sbase, (uint32_t)lane);
            st_async1(peer + soff(&sm.maxslot[z][nb][rank * kWarps + warp]), wmin,
                      peer + soff(&sm.full[z][nb]));
        }
        if (part_row) {
            // lanes 0-15 reduce component 0, lanes 16-31 component 1
            const bool hi = lane >= 16;
            float keep = hi ? acc.y : acc.x;
            keep += __shfl_xor_sync(0xffffffffu, hi ? acc.x : acc.y, 16);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
            if ((lane & 15) == 0) part_row[2 * warp + (lane >> 4)] = keep;
        }
        if (rows_tn >= 1) {
            // the last warp to finish the step has the staged history row to
            // itself: it loads the next one
            int last = 0;
            if (lane == 0) {
                __threadfence_block();
                last = atomicAdd(&sm.cnt[z][nb], 1) == kWarps - 1;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last && lane == 0) {
                __threadfence_block();
                issue_rows(z, rows_tn, slot_ws);
                sm.cnt[z][nb] = 0;
            }
        }
    };

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
                const long e = (sidx[z] * N + t) * kV;
                sm.w[z][t] = make_float2(__ldg(seq + e), __ldg(seq + e + 1));
                if (GRAD) {
                    sm.g[z][t] = make_float2(__ldg(grad + e), __ldg(grad + e + 1));
                    sm.sf[z][t] = make_float2(__ldg(soft_in + e), __ldg(soft_in + e + 1));
                }
            }
        }
        load_alpha_cb();
        __syncthreads();

        // ------------------------------------------------------------ alpha
        double O[kSlots];
        float lzm[kSlots], lzs[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) { O[z] = 0.0; lzm[z] = kPosInf; lzs[z] = 0.f; }
        for (int t = 0; t < N; ++t) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                // inputs: alpha costs S_t (raw; the global minimum `sub` is
                // removed from the outputs) and H_t
                float shift, sub;
                const float *in = &sm.zero[0][0];
                if (t == 0) {
                    shift = a0;                    // a_0 is the same for every group
                    sub = 0.f;
                } else {
                    const int x = use[z] & 1;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_bar(bar, (use[z] >> 1) & 1, status, failed);
                    shift = sub = cluster_min(sm.maxslot[z][x], lane);
                    in = &sm.buf[z][x][0][0];
                    ++use[z];
                }
                O[z] += (double)shift;
                if (tid == 0) sm.offs[z][t] = O[z];
                const int nb = use[z] & 1;
                const float2 wv = sm.w[z][t];
                float2 gv = make_float2(0.f, 0.f);
                float gs = 0.f;
                if (GRAD) {
                    gv = sm.g[z][t];
                    const float2 sv = sm.sf[z][t];
                    gs = gv.x * sv.x + gv.y * sv.y;
                }
                const bool last = (t == N - 1);
                const F2 W0 = bc(wv.x), W1 = bc(wv.y), G0 = bc(gv.x), G1 = bc(gv.y),
                         GS = bc(gs), NK = bc(-kap);
                float o[kVT][2], hh[kVT][2];
                float lmin = kPosInf;
#pragma unroll
                for (int h = 0; h < kVT; ++h) {
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int rl = arl[h] + 16 * rr;
                    F2 x[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const F2 A = *reinterpret_cast<const F2 *>(in + 2 * (i * kRPC + rl));
                        const F2 d0 = sub2(C0[h][rr][i], W0), d1 = sub2(C1[h][rr][i], W1);
                        x[i] = fma2(d1, d1, fma2(d0, d0, A));
                    }
                    const float m = min16(x);
                    const F2 KM = bc(kap * m);
                    // each pair's dependent FMA work right after its two ex2,
                    // so the MUFU and FMA pipes interleave (same sums, same order)
                    F2 e[8];
                    F2 hf = bc(0.f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        e[i] = ex2p(fma2(x[i], NK, KM));
                        if (GRAD) {
                            const F2 H = *reinterpret_cast<const F2 *>(in + kIn + 2 * (i * kRPC + rl));
                            const F2 f = fma2(C0[h][rr][i], G0, fma2(C1[h][rr][i], G1, sub2(H, GS)));
                            hf = fma2(e[i], f, hf);
                        }
                    }
                    const F2 S2 = sum8(e);
                    const float S = S2.x + S2.y;
                    o[h][rr] = fmaf(-lg2(S), ikap, m - sub);
                    if (GRAD) hh[h][rr] = (hf.x + hf.y) * rcp(S);
                }
                lmin = min3(lmin, o[h][0], o[h][1]);
                if (!last) {
                    if (!failed && !drop) {
                        const uint32_t bar = a_base[h] + soff(&sm.full[z][nb]);
                        const uint32_t o0 = a_base[h] + soff(&sm.buf[z][nb][0][0]) + 4u * a_off[h];
                        st_async2(o0, o[h][0], o[h][1], bar);
                        if (GRAD) st_async2(o0 + kIn * 4, hh[h][0], hh[h][1], bar);
                    }
                    // history row t + 1, in the consumer's chunk
                    float *hrow = slot_ws[z] + lay.hist + (long)(t + 1) * kRowFloats +
                                  a_dst[h] * (kPlanes * kIn) + a_off[h];
                    *reinterpret_cast<float2 *>(hrow) = make_float2(o[h][0], o[h][1]);
                    if (GRAD) *reinterpret_cast<float2 *>(hrow + kIn) = make_float2(hh[h][0], hh[h][1]);
                } else {
                    smin_merge(lzm[z], lzs[z], kap * o[h][0], 1.f);
                    smin_merge(lzm[z], lzs[z], kap * o[h][1], 1.f);
                }
                }
                finish_step(z, nb, !last && !drop, lmin, nullptr, bc(0.f), 0,
                            slot_ws);
            }
        }
        __syncthreads();

        // log2 Z = -(kappa O_{N-1} + log2-soft-min over all 4096 costs kappa S_N).
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            float m = lzm[z], s = lzs[z];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
                const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
                smin_merge(m, s, m2, s2);
            }
            if (lane == 0) { sm.wmin[z][warp] = m; sm.wacc[z][warp] = s; }
        }
        __syncthreads();
        if (tid == 0) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                float m = kPosInf, s = 0.f;
                for (int i = 0; i < kWarps; ++i) smin_merge(m, s, sm.wmin[z][i], sm.wacc[z][i]);
#pragma unroll
                for (int r = 0; r < kCL; ++r) {
                    st_cluster(mapa(sbase, (uint32_t)r) + soff(&sm.lz[z][rank][0]), m);
                    st_cluster(mapa(sbase, (uint32_t)r) + soff(&sm.lz[z][rank][1]), s);
                }
            }
        }
        load_beta_cb();
        cluster_sync();   // also publishes every CTA's history rows

        double logZ2[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            logZ2[z] = 0.0;
            if (!active[z]) continue;
            float m = kPosInf, s = 0.f;
#pragma unroll
            for (int r = 0; r < kCL; ++r) smin_merge(m, s, sm.lz[z][r][0], sm.lz[z][r][1]);
            logZ2[z] = -((double)kap * O[z] + (double)m - (double)log2f(s));
            if (!GRAD && rank == 0 && tid == 0 && logZ_out)
                logZ_out[sidx[z]] = (float)(logZ2[z] * (double)kLn2) + poison_value(bad_T, status);
        }
        if (tid == 0) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z)
                if (active[z] && N - 1 >= 1) issue_rows(z, N - 1, slot_ws);
        }

        // ------------------------------------------------------------- beta
        double U[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) U[z] = 0.0;
        for (int t = N - 2; t >= -1; --t) {
            const int tn = t + 1;
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                // inputs: beta costs of Bt_{t+1} (raw; minus sigma), Bb_{t+1},
                // and this step's alpha / H history values
                float sigma = 0.f;
                const float *in = &sm.zero[0][0];
                if (t != N - 2) {
                    const int x = use[z] & 1;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_bar(bar, (use[z] >> 1) & 1, status, failed);
                    sigma = cluster_min(sm.maxslot[z][x], lane);
                    in = &sm.buf[z][x][0][0];
                    ++use[z];
                }
                U[z] += (double)sigma;
                float ah[kVT][2], hp[kVT][2];
#pragma unroll
                for (int h = 0; h < kVT; ++h) { ah[h][0] = ah[h][1] = a0; hp[h][0] = hp[h][1] = 0.f; }
                if (tn > 0) {
                    wait_bar(sbase + soff(&sm.hbar[z]), hcnt[z] & 1, status, failed);
                    ++hcnt[z];
#pragma unroll
                    for (int h = 0; h < kVT; ++h) {
                        const int o4 = 2 * ((bp[h] >> 1) * kRPC + brl);
                        const float4 va = *reinterpret_cast<const float4 *>(&sm.hst[z][0][o4]);
                        ah[h][0] = (bp[h] & 1) ? va.y : va.x;
                        ah[h][1] = (bp[h] & 1) ? va.w : va.z;
                        if (GRAD) {
                            const float4 vh = *reinterpret_cast<const float4 *>(&sm.hst[z][kPlanes - 1][o4]);
                            hp[h][0] = (bp[h] & 1) ? vh.y : vh.x;
                            hp[h][1] = (bp[h] & 1) ? vh.w : vh.z;
                        }
                    }
                }
                const double Oa = tn > 0 ? sm.offs[z][tn - 1] : 0.0;
                const float Cb = (float)(-(logZ2[z] + (double)kap * (Oa + U[z])));
                const int nb = use[z] & 1;
                const float2 wv = sm.w[z][tn];
                float2 gv = make_float2(0.f, 0.f), st = make_float2(0.f, 0.f);
                float gs = 0.f;
                if (GRAD) {
                    gv = sm.g[z][tn];
                    st = sm.sf[z][tn];
                    gs = gv.x * st.x + gv.y * st.y;
                }
                const F2 W0 = bc(wv.x), W1 = bc(wv.y), G0 = bc(gv.x), G1 = bc(gv.y),
                         GS = bc(gs), NK = bc(-kap);
                F2 acc = bc(0.f);
                float ob[kVT][2], bbo[kVT][2];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    // this lane's 128-byte region: butterflies 2 lane, 2 lane + 1,
                    // the inputs of every unit of the thread
                    auto chunk = [&](int plane, int q) -> float4 {
                        const uint32_t off = (uint32_t)lane * 32u +
                                             ((uint32_t)((rr << 2) | q) ^ ((uint32_t)lane & 7u)) * 4u;
                        return *reinterpret_cast<const float4 *>(in + plane * kIn + off);
                    };
                    F2 bin[8], bbin[8];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 v = chunk(0, q);
                        bin[2 * q] = mk(v.x, v.y);
                        bin[2 * q + 1] = mk(v.z, v.w);
                        if (GRAD) {
                            const float4 u = chunk(kPlanes - 1, q);
                            bbin[2 * q] = sub2(mk(u.x, u.y), GS);
                            bbin[2 * q + 1] = sub2(mk(u.z, u.w), GS);
                        }
                    }
#pragma unroll
                    for (int h = 0; h < kVT; ++h) {
                    F2 x[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const F2 d0 = sub2(C0[h][rr][i], W0), d1 = sub2(C1[h][rr][i], W1);
                        x[i] = fma2(d1, d1, fma2(d0, d0, bin[i]));
                    }
                    const float m = min16(x);
                    const F2 KM = bc(kap * m);
                    const float ms = m - sigma;
                    const float f = ex2(fmaf(ms + ah[h][rr], -kap, Cb));
                    // as in the alpha sweep: each pair's accumulations right after its ex2
                    F2 e[8];
                    F2 e0 = bc(0.f), e1 = bc(0.f);
                    const F2 HP = bc(GRAD ? hp[h][rr] : 0.f);
                    F2 ey = bc(0.f), sv = bc(0.f), s0 = bc(0.f), s1 = bc(0.f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        e[i] = ex2p(fma2(x[i], NK, KM));
                        if (!GRAD) {
                            e0 = i == 0 ? mul2(e[0], C0[h][rr][0]) : fma2(e[i], C0[h][rr][i], e0);
                            e1 = i == 0 ? mul2(e[0], C1[h][rr][0]) : fma2(e[i], C1[h][rr][i], e1);
                        } else {
                            const F2 y = fma2(C0[h][rr][i], G0, fma2(C1[h][rr][i], G1, bbin[i]));
                            ey = fma2(e[i], y, ey);
                            const F2 v = mul2(e[i], add2(y, HP));
                            sv = add2(sv, v);
                            s0 = fma2(v, C0[h][rr][i], s0);
                            s1 = fma2(v, C1[h][rr][i], s1);
                        }
                    }
                    const F2 S2 = sum8(e);
                    const float S = S2.x + S2.y;
                    ob[h][rr] = t >= 0 ? fmaf(-lg2(S), ikap, ms) : 0.f;
                    if (!GRAD) {
                        acc = fma2(bc(f), mk(e0.x + e0.y, e1.x + e1.y), acc);
                        bbo[h][rr] = 0.f;
                    } else {
                        bbo[h][rr] = (ey.x + ey.y) * rcp(S);
                        const float SV = sv.x + sv.y;
                        acc = fma2(bc(f), mk(fmaf(-st.x, SV, s0.x + s0.y), fmaf(-st.y, SV, s1.x + s1.y)),
                                   acc);
                    }
                    }
                }
                float lmin = kPosInf;
#pragma unroll
                for (int h = 0; h < kVT; ++h) {
                    lmin = min3(lmin, ob[h][0], ob[h][1]);
                    if (t >= 0 && !failed) {
                        const uint32_t bar = b_base[h] + soff(&sm.full[z][nb]);
                        const uint32_t o0 = b_base[h] + soff(&sm.buf[z][nb][0][0]) + 4u * b_off[h];
                        st_async2(o0, ob[h][0], ob[h][1], bar);
                        if (GRAD) st_async2(o0 + kIn * 4, bbo[h][0], bbo[h][1], bar);
                    }
                }
                float *part_row = slot_ws[z] + lay.part + ((long)tn * kCL + rank) * kWarps * 2;
                finish_step(z, nb, t >= 0, lmin, part_row, acc, tn - 1, slot_ws);
            }
        }
        __syncthreads();

        // Per-step partials of the 4 x 16 warps, added in a fixed order.
        cluster_sync();
        if (rank == 0) {
            const float scale = GRAD ? two_over_T : 1.f;
            const float poison = poison_value(bad_T, status);   // NaN after a failed wait
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                const float *part = slot_ws[z] + lay.part;
                for (int tn = tid; tn < N; tn += kNT) {
                    const float4 *p4 = reinterpret_cast<const float4 *>(part + (long)tn * kCL * kWarps * 2);
                    float s0 = 0.f, s1 = 0.f;
#pragma unroll
                    for (int i = 0; i < kCL * kWarps / 2; ++i) {
                        const float4 v = __ldcg(p4 + i);
                        s0 += v.x + v.z;
                        s1 += v.y + v.w;
                    }
                    out[(sidx[z] * N + tn) * kV] = scale * s0 + poison;
                    out[(sidx[z] * N + tn) * kV + 1] = scale * s1 + poison;
                }
            }
        }
    }
    // No CTA leaves with a TMA row copy in flight (only possible after a
    // failure): wait, bounded, for every issued load that was not consumed.
    __syncthreads();
    if (tid == 0) {
        bool f2 = false;
#pragma unroll
        for (int z = 0; z < kSlots; ++z)
            for (uint32_t k = hcnt[z]; k < (uint32_t)sm.hiss[z]; ++k)
                wait_bar(sbase + soff(&sm.hbar[z]), k & 1, status, f2);
    }
    cluster_sync();
}

}  // namespace b4

// ---------------------------------------------------------------------------
// Host side.

namespace {

template <bool GRAD>
int b4_max_clusters() {
    static int cached[2][64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    int &c = cached[GRAD ? 1 : 0][dev];
    if (c > 0) return c;
    const size_t smem = sizeof(b4::Smem<GRAD>);
    if (cudaFuncSetAttribute(b4::b4_kernel<GRAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(sms / b4::kCL * b4::kCL), 1, 1);
    cfg.blockDim = dim3(b4::kNT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = b4::kCL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, b4::b4_kernel<GRAD>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    c = n;
    return n;
}

}  // namespace

bool b4_applicable(int B, int N, int L, int BB, int V) {
    (void)B;
    return L == b4::kL && BB == b4::kB && V == b4::kV && N >= 2 && N <= b4::kNMax;
}

int b4_clusters(int B, int mode) {
    int maxc = (mode == kModeBackward) ? b4_max_clusters<true>() : b4_max_clusters<false>();
    // SMs left free for concurrent kernels (bcjr_set_reserved_sms)
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int cap = (sms - reserved_sms()) / b4::kCL;
    if (maxc > cap) maxc = cap;
    const long pairs = ((long)B + b4::kSlots - 1) / b4::kSlots;
    long n = maxc;
    if (n > pairs) n = pairs;
    return (int)n;
}

size_t b4_workspace_bytes(int B, int N, int mode) {
    const int ncl = b4_clusters(B, mode);
    if (ncl <= 0) return 0;
    const long slot = b4::slot_layout(N, mode == kModeBackward).total;
    return (size_t)ncl * b4::kSlots * slot * 4;
}

cudaError_t launch_b4(const LaunchArgs &a) {
    const bool grad = (a.mode == kModeBackward);
    const int ncl = b4_clusters(a.B, a.mode);
    if (ncl <= 0) return cudaErrorInvalidConfiguration;
    const long slot = b4::slot_layout(a.N, grad).total;
    if ((size_t)ncl * b4::kSlots * slot * 4 > a.ws_data_bytes) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)(ncl * b4::kCL)), block(b4::kNT);
    float *ws = reinterpret_cast<float *>(a.ws_data);
    if (grad) {
        b4::b4_kernel<true><<<grid, block, sizeof(b4::Smem<true>), a.stream>>>(
            a.seq, a.cb, a.T_dev, a.soft_in, a.grad, a.B, a.N, a.dseq, nullptr, ws, a.status,
            a.drop_sends);
    } else {
        b4::b4_kernel<false><<<grid, block, sizeof(b4::Smem<false>), a.stream>>>(
            a.seq, a.cb, a.T_dev, nullptr, nullptr, a.B, a.N, a.soft, a.logZ, ws, a.status,
            a.drop_sends);
    }
    return cudaGetLastError();
}

}  // namespace bcjr
