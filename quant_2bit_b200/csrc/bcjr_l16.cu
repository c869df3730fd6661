// Production kernel for the QTIP trellis L=16, k=2, V=1 (b = 2), one CTA per
// SM, in two instances: 2-CTA thread-block clusters (all 148 SMs of a B200,
// 74 clusters; two sequences in flight per cluster in the forward, one in the
// backward) and 4-CTA clusters (33 clusters on 132 SMs; two sequences in both
// calls).  The forward runs the 2-CTA instance; the backward runs the 4-CTA
// grid and, on the 16 SMs it leaves free, a 2-CTA grid beside it.
//
// Work decomposition
// ------------------
// With M = 14, the 2^16 states split into 4096 "butterflies"
//     j in [0, 4096):  states q = p * 2^14 + 4 j + c,   p, c in 0..3.
// In the forward (alpha) direction butterfly j reads the four group values
// A_t(p 2^12 + j) and writes A_{t+1}(4 j + c); in the backward (beta)
// direction it reads Bt_{t+1}(4 j + c) and writes Bt_t(p 2^12 + j).  Every
// step touches the same 16 states per butterfly, so each thread owns
// kJPT = 4 (2-CTA) or 2 (4-CTA) butterflies for the whole kernel and keeps
// their codebook values in registers: no codebook traffic after the first
// load.  CTA r of the cluster owns butterflies [r 4096/kCL, (r+1) 4096/kCL).
//
// Arithmetic
// ----------
// Messages are costs in squared-distance units, a = -A / kappa and
// b = -Bt / kappa (kappa = log2(e)/T), so that the energy-plus-message of a
// state is one fma of the exact difference d = c - w:  x = d*d + a.  The
// soft-min of four costs is  m - lg2(sum 2^(kappa (m - x))) / kappa,
// m = min x, with every exponent one fma  kappa m - kappa x.  All FMA-pipe
// work is issued as f32x2 pairs (add/sub/mul/fma.rn.f32x2): pairs over p in
// the alpha direction, pairs of output groups in the beta direction, from
// one register layout cq[jj][c][p/2].
//
// Exchange between steps
// ----------------------
// The outputs of a step are the inputs of butterflies spread over the whole
// cluster (a perfect shuffle).  Producers push them straight into the
// consumer CTA's shared memory with st.async ... mbarrier::complete_tx, into
// a double-buffered ring; the consumer arms each buffer's mbarrier with the
// expected byte count.  There is no block barrier per step: each warp that
// finishes a step sends its minimum output cost to every consumer CTA along
// with its data, as part of the same consumption's byte count, and every
// consumer warp takes the minimum over all of them with one redux.  A
// producer that has received the complete input of consumption u therefore
// knows that every warp of every CTA has finished reading consumption u-1,
// whose buffer it is about to overwrite.  Every consumer renormalises by the
// exact global minimum of the previous step; shifts accumulate in double.
//
// Two sequences ("slots") are interleaved step by step so that one slot's
// exchange latency hides behind the other's arithmetic (one in the 2-CTA
// backward: its two 32 KB planes per ring buffer fill shared memory).
// Alpha / H rows go to a global history with float4 stores; the
// backward-time sweep fetches
// the rows it needs one step ahead with TMA bulk copies (cp.async.bulk) into
// shared memory.  Per-step partial sums of soft / d_seq are written per
// (block of 1024 butterflies, warp) and added in a fixed order by CTA 0, log Z
// likewise: results are deterministic and the same in both instances, so
// sequences may go to either (they are claimed from a shared counter).
//
// Every wait is bounded (about 1 s); on timeout the kernel records
// BCJR_ERR_TIMEOUT in the workspace status word, stops waiting and sending,
// runs to completion, and writes NaN into the outputs it writes from then on
// (poison_value).  The recursions are documented in bcjr_common.cuh.
#include <cstdint>

#include "bcjr_cluster.cuh"
#include "bcjr_kernels.h"

// This file is compiled twice: as the 2-CTA instance (namespace l16, which
// also holds the dispatcher at the end) and, from bcjr_l16_cl4.cu, as the
// 4-CTA instance (namespace l16c4).
#ifndef BCJR_L16_CL
#define BCJR_L16_CL 2
#endif
#if BCJR_L16_CL == 2
#define BCJR_L16_NS l16
#else
#define BCJR_L16_NS l16c4
#endif

namespace bcjr {
namespace BCJR_L16_NS {

using namespace clu;

constexpr int kL = 16;
constexpr int kB = 2;                 // branch bits b = kV
constexpr int kG = 1 << (kL - kB);    // 16384 groups
constexpr int kNJ = kG >> kB;         // 4096 butterflies
constexpr int kCL = BCJR_L16_CL;      // CTAs per cluster (4 or 2)
constexpr int kJPC = kNJ / kCL;       // butterflies per CTA
constexpr int kIn = 4 * kJPC;         // inputs per CTA per step and plane
#ifndef BCJR_L16_NT
#define BCJR_L16_NT 512
#endif
constexpr int kNT = BCJR_L16_NT;      // threads per CTA
constexpr int kJPT = kJPC / kNT;      // butterflies per thread
static_assert(kCL == 2 || kCL == 4, "cluster of 2 or 4 CTAs");
// Sequences in flight per cluster, interleaved step by step: two, except in
// the 2-CTA backward, whose two 32 KB planes per ring buffer leave shared
// memory for one.
template <bool GRAD>
struct SlotsOf {
    static constexpr int value = (kCL == 2 && GRAD) ? 1 : 2;
};
constexpr int kNMax = 512;            // longest sequence staged in shared memory
// Sleep between tests of a bounded wait: a kernel with one slot in flight
// has no other work while it waits: it polls without sleeping (measured on
// B200: backward 117 ms with no sleep, 119 ms at 100 ns, 125 ms at 400 ns).
#ifndef BCJR_L16_SLEEP1_NS
#define BCJR_L16_SLEEP1_NS 0
#endif
template <bool GRAD>
struct SleepOf {
    static constexpr unsigned value = SlotsOf<GRAD>::value == 1 ? BCJR_L16_SLEEP1_NS : kWaitSleepNs;
};
constexpr int kWarps = kNT / 32;
// Virtual warps: the reductions below group butterflies as a 512-thread CTA
// would (32 lanes x 2 butterflies 512 apart per partial), whatever kNT is,
// so that every instance reduces in the same order.
constexpr int kVW = 16;
// Reduction blocks: the per-step sums (soft codewords, gradients) and log Z
// are reduced per (block of 1024 butterflies, virtual warp), then over the
// 4 x 16 partials in a fixed order.  Partial (b, v) holds butterflies
// b 1024 + 32 v + lane + 512 h (h = 0, 1), summed per lane in the order
// h = 0, 1 and then over the lanes; butterfly pair q = jj / 2 of a thread is
// partial number q kWarps + warp of its CTA (jl_of below).  Every instance
// forms the same 64 partials, so a sequence's results are bitwise the same
// whichever instance runs it.
constexpr int kRB = kNJ / 1024;       // 4 reduction blocks
constexpr int kParts = kRB * kVW;     // 64 partials per step
static_assert(kJPT % 2 == 0, "two butterflies of a thread per reduction partial");
static_assert((kJPC / 64) % kWarps == 0, "whole partials per warp");

// Local butterfly of the thread's jj-th slot, and its reduction partial.
__device__ __forceinline__ int jl_of(int tid, int jj) {
    const int q = (jj >> 1) * kWarps + (tid >> 5);       // partial within the CTA
    return (q / kVW) * 1024 + 32 * (q % kVW) + (tid & 31) + 512 * (jj & 1);
}
__device__ __forceinline__ int part_of(uint32_t rank, int tid, int jj) {
    const int q = (jj >> 1) * kWarps + (tid >> 5);
    return ((int)rank * (kJPC / 1024) + q / kVW) * kVW + q % kVW;
}

template <bool GRAD>
struct alignas(128) Smem {
    static constexpr int kPlanes = GRAD ? 2 : 1;
    static constexpr int kSlots = SlotsOf<GRAD>::value;
    float buf[kSlots][2][kPlanes][kIn];   // input ring (kIn floats per plane)
    float hst[kSlots][kPlanes][kIn];      // history rows staged by TMA: [p * kJPC + jl]
    double offs[kSlots][kNMax];           // alpha shifts O_t
    float maxslot[kSlots][2][kCL * kWarps];   // per-warp minimum cost riding with the data
    float w[kSlots][kNMax];
    float g[kSlots][GRAD ? kNMax : 4];
    float sf[kSlots][GRAD ? kNMax : 4];
    float lz[kSlots][kParts][2];          // log Z partials, every (block, warp) of the cluster
    unsigned long long full[kSlots][2];
    unsigned long long hbar[kSlots];
    int cnt[kSlots][2];                   // warps finished with the step (backward sweep)
    int hiss[kSlots];                     // TMA row loads issued per slot
    unsigned next;                        // first sequence of the cluster's current claim
};

// Minimum of the kCL * kWarps per-warp minima riding with a consumption
// (called by whole warps).
__device__ __forceinline__ float cluster_min(const float *m, int lane) {
    float v = m[lane];
#pragma unroll
    for (int i = 32; i < kCL * kWarps; i += 32) v = fminf(v, m[lane + i]);
    return redux_min(v);
}

// Workspace of one (cluster, slot): float offsets.
struct SlotLayout {
    long hist;      // alpha cost rows: N x kG  (row t holds S_t, t >= 1)
    long hhist;     // H rows: N x kG  (backward only)
    long part;      // N x kParts per-step (block, warp) partial sums
    long total;
};

__host__ __device__ inline SlotLayout slot_layout(int N, bool grad) {
    SlotLayout s;
    long p = 0;
    s.hist = p; p += (long)N * kG;
    s.hhist = p; if (grad) p += (long)N * kG;
    s.part = p; p += (long)N * kParts;
    s.total = (p + 63) & ~63L;   // 256-byte aligned slots
    return s;
}

template <bool GRAD>
__global__ void __cluster_dims__(kCL, 1, 1) __launch_bounds__(kNT, 1)
l16_kernel(const float *__restrict__ seq, const float *__restrict__ cb,
           const float *__restrict__ T_dev, const float *__restrict__ soft_in,
           const float *__restrict__ grad, int B, int N,
           float *__restrict__ out, float *__restrict__ logZ_out,
           float *__restrict__ ws, int *status, unsigned *claim, int drop_sends) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    using SM = Smem<GRAD>;
    // A kernel launched after this one with programmatic stream serialization
    // (the 2-CTA backward on the SMs that 4-CTA clusters leave free) may start
    // now; it takes sequences from the same counter and waits for this grid
    // before it completes.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    SM &sm = *reinterpret_cast<SM *>(smem_raw);
    constexpr int kPlanes = SM::kPlanes;
    constexpr int kSlots = SM::kSlots;
    constexpr uint32_t kBytes = kPlanes * kIn * 4 + kCL * kWarps * 4;   // per consumption
    constexpr uint32_t kRowBytes = kJPC * 4;                    // one TMA chunk

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t rank = cluster_rank();
    const uint32_t cid = cluster_id();
    const SlotLayout lay = slot_layout(N, GRAD);

    const float T = __ldg(T_dev);
    const float kap = kLog2e / T;           // kappa
    const float ikap = T / kLog2e;
    const float two_over_T = 2.f / T;
    const float a0 = -(float)kB * ikap;     // cost of A_0 = b everywhere
    const bool bad_T = bad_temperature(T);  // outputs NaN (poison_value)

    // Codebook of my kJPT butterflies:
    // cq[jj][c][h] = (c(2h, c), c(2h+1, c)),  c(p, c) = cb[p 2^14 + 4 j + c].
    int jg[kJPT];
    F2 cq[kJPT][4][2];
#pragma unroll
    for (int jj = 0; jj < kJPT; ++jj) {
        jg[jj] = (int)rank * kJPC + jl_of(tid, jj);
        const float *q = cb + 4 * jg[jj];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            cq[jj][c][0] = ldg_pair(q + c, q + kG + c);
            cq[jj][c][1] = ldg_pair(q + 2 * kG + c, q + 3 * kG + c);
        }
    }

    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem_raw);
    uint32_t cbase[kCL];
#pragma unroll
    for (int r = 0; r < kCL; ++r) cbase[r] = mapa(sbase, r);
    auto soff = [&](const void *p) -> uint32_t {
        return (uint32_t)__cvta_generic_to_shared(p) - sbase;
    };

    // Remote CTA of my alpha outputs and their offset inside an input plane.
    uint32_t rdst[kJPT], aoff[kJPT];
#pragma unroll
    for (int jj = 0; jj < kJPT; ++jj) {
        // output A(4 j + c) is input p' = j >> 10 of butterfly (4 j + c) mod 4096
        const int j = jg[jj];
        rdst[jj] = cbase[0];
        const uint32_t d = (uint32_t)(j & 1023) / (uint32_t)(kJPC / 4);
#pragma unroll
        for (int r = 1; r < kCL; ++r) rdst[jj] = (d == (uint32_t)r) ? cbase[r] : rdst[jj];
        aoff[jj] = 4u * (uint32_t)((j >> 10) * kJPC + 4 * (j & (kJPC / 4 - 1)));
    }

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

    // End of a step, per warp (no block barrier): the warp's minimum output
    // cost goes into the step's shared-memory minimum, its partial sum into
    // global memory, and the last warp to arrive sends the CTA minimum to the
    // kCL consumers and, in the beta sweep, issues the next TMA rows (every
    // warp of the CTA has read this step's inputs by then).
    // TMA rows of step tn (alpha costs, and H for the backward) into the
    // staging buffer of slot z; completion on hbar[z].
    auto issue_rows = [&](int z, int tn, float *const *slot_ws) {
        const uint32_t hb = sbase + soff(&sm.hbar[z]);
        if (failed) return;
        atomicAdd(&sm.hiss[z], 1);
        mbar_arm(hb, kPlanes * kIn * 4);
        const float *hist = slot_ws[z] + lay.hist + (long)tn * kG + rank * kJPC;
#pragma unroll
        for (int p = 0; p < 4; ++p)
            bulk_g2s(sbase + soff(&sm.hst[z][0][p * kJPC]), hist + p * kNJ, kRowBytes, hb);
        if (GRAD) {
            const float *hh = slot_ws[z] + lay.hhist + (long)tn * kG + rank * kJPC;
#pragma unroll
            for (int p = 0; p < 4; ++p)
                bulk_g2s(sbase + soff(&sm.hst[z][kPlanes - 1][p * kJPC]), hh + p * kNJ, kRowBytes, hb);
        }
    };

    auto finish_step = [&](int z, int nb, bool send, float lmin, int rows_tn,
                           float *const *slot_ws) {
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

    // Beta-sweep outputs of butterfly j, output-group pair h: Bt(p' 4096 + j)
    // (p' = 2h, 2h+1) is input (j & 3) of butterfly p' 1024 + (j >> 2), i.e. of
    // CTA p' kCL / 4 at offset (p' 4096 + j) mod kIn; Bb likewise in the
    // second plane.
    auto send_beta = [&](int j, int h, F2 ob, F2 bbo, uint32_t buf_off, uint32_t bar_off) {
        const int d0 = (2 * h) * kCL / 4, d1 = (2 * h + 1) * kCL / 4;
        const uint32_t s0 = 4u * ((2 * h) % (4 / kCL)) * 4096u;
        const uint32_t s1 = 4u * ((2 * h + 1) % (4 / kCL)) * 4096u;
        const uint32_t ob0 = buf_off + 4u * (uint32_t)j;
        st_async1(cbase[d0] + ob0 + s0, ob.x, cbase[d0] + bar_off);
        st_async1(cbase[d1] + ob0 + s1, ob.y, cbase[d1] + bar_off);
        if (GRAD) {
            const uint32_t ob1 = ob0 + kIn * 4;
            st_async1(cbase[d0] + ob1 + s0, bbo.x, cbase[d0] + bar_off);
            st_async1(cbase[d1] + ob1 + s1, bbo.y, cbase[d1] + bar_off);
        }
    };
    // The forward sends its beta outputs after all of the step's arithmetic
    // (one basic block for the compiler to schedule: 6 % faster on B200);
    // the backward sends each as it is computed (holding them there measured
    // 1.5 % slower).
    constexpr bool kHoistSends = !GRAD;

    // Sequences are claimed kSlots at a time from a counter shared by every
    // cluster of the call (of both instances, when two run side by side):
    // CTA 0 takes the claim and publishes it to the cluster, with the top bit
    // set once the call has failed (a bounded wait gave up anywhere).  A
    // failed call keeps claiming, but its clusters only write NaN into the
    // claimed sequences' outputs: no output of a failed call is left
    // unwritten or looks valid.
    auto claim_next = [&]() -> unsigned {
        if (rank == 0 && tid == 0) {
            unsigned s0 = atomicAdd(claim, (unsigned)kSlots);
            if (*reinterpret_cast<volatile int *>(status) != 0) s0 |= 0x80000000u;
#pragma unroll
            for (int r = 0; r < kCL; ++r) st_cluster_u32(cbase[r] + soff(&sm.next), s0);
        }
        cluster_sync();
        return sm.next;
    };
    for (unsigned cl = claim_next(); (long)(cl & 0x7fffffffu) < B; cl = claim_next()) {
        const long first = (long)(cl & 0x7fffffffu);
        if (cl >> 31) {
            if (rank == 0) {
                const float nanv = __int_as_float(0x7fffffff);
#pragma unroll
                for (int z = 0; z < kSlots; ++z) {
                    const long sz = first + z;
                    if (sz >= B) continue;
                    for (int t = tid; t < N; t += kNT) out[sz * N + t] = nanv;
                    if (!GRAD && tid == 0 && logZ_out) logZ_out[sz] = nanv;
                }
            }
            cluster_sync();   // every thread has read this claim before the next one is published
            continue;
        }
        bool active[kSlots];
        long sidx[kSlots];
        float *slot_ws[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            sidx[z] = first + z;
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
        double O[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) O[z] = 0.0;
        for (int t = 0; t < N; ++t) {
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                // inputs: costs of A_t minus the global minimum, and H_t
                float shift;
                const float *in = nullptr;   // this step's inputs (none at t = 0: all a_0)
                if (t == 0) {
                    shift = a0;                    // a_0 is the same for every group
                } else {
                    const int x = use[z] & 1;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_bar<SleepOf<GRAD>::value>(bar, (use[z] >> 1) & 1, status, failed);
                    shift = cluster_min(sm.maxslot[z][x], lane);
                    in = &sm.buf[z][x][0][0];
                    ++use[z];
                }
                O[z] += (double)shift;
                if (tid == 0) sm.offs[z][t] = O[z];
                const int nb = use[z] & 1;
                const float w = sm.w[z][t];
                float gq = 0.f, gs = 0.f;
                if (GRAD) {
                    gq = sm.g[z][t];
                    gs = gq * sm.sf[z][t];
                }
                const bool last = (t == N - 1);
                const uint32_t bar_off = soff(&sm.full[z][nb]);
                const uint32_t buf_off = soff(&sm.buf[z][nb][0][0]);
                const F2 W = bc(w), Gq = bc(gq), GS = bc(-gs), NK = bc(-kap);
                float lmin = kPosInf;
                float lzm = kPosInf, lzs = 0.f;   // log Z soft-min of a block (last step)
                float *hist = slot_ws[z] + lay.hist + (long)(t + 1) * kG;
                float *hhist = slot_ws[z] + lay.hhist + (long)(t + 1) * kG;
#pragma unroll
                for (int jj = 0; jj < kJPT; ++jj) {
                    // costs of A_t minus the global minimum, and H_t, of my butterfly
                    float ain[4] = {0.f, 0.f, 0.f, 0.f}, hin[4] = {0.f, 0.f, 0.f, 0.f};
                    if (in) {
                        const int jl = jl_of(tid, jj);
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            ain[p] = in[p * kJPC + jl] - shift;
                            if (GRAD) hin[p] = in[kIn + p * kJPC + jl];
                        }
                    }
                    const F2 A01 = mk(ain[0], ain[1]), A23 = mk(ain[2], ain[3]);
                    const F2 H01 = mk(hin[0], hin[1]), H23 = mk(hin[2], hin[3]);
                    float o4[4], h4[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const F2 d0 = sub2(cq[jj][c][0], W), d1 = sub2(cq[jj][c][1], W);
                        const F2 x0 = fma2(d0, d0, A01), x1 = fma2(d1, d1, A23);
                        const float m = min4(x0.x, x0.y, x1.x, x1.y);
                        const F2 KM = bc(kap * m);
                        const F2 e0 = ex2p(fma2(x0, NK, KM)), e1 = ex2p(fma2(x1, NK, KM));
                        const F2 s2 = add2(e0, e1);
                        const float s = s2.x + s2.y;
                        o4[c] = fmaf(-lg2(s), ikap, m);
                        if (GRAD) {
                            const F2 f0 = add2(fma2(cq[jj][c][0], Gq, GS), H01);
                            const F2 f1 = add2(fma2(cq[jj][c][1], Gq, GS), H23);
                            const F2 hf = fma2(e0, f0, mul2(e1, f1));
                            h4[c] = (hf.x + hf.y) * rcp(s);
                        }
                    }
                    lmin = fminf(lmin, min4(o4[0], o4[1], o4[2], o4[3]));
                    const int j = jg[jj];
                    if (!last) {
                        const uint32_t bar = rdst[jj] + bar_off;
                        const uint32_t o0 = rdst[jj] + buf_off + aoff[jj];
                        if (!failed && !drop) {
                            st_async4(o0, o4[0], o4[1], o4[2], o4[3], bar);
                            if (GRAD)
                                st_async4(o0 + kIn * 4, h4[0], h4[1], h4[2], h4[3], bar);
                        }
                        *reinterpret_cast<float4 *>(hist + 4 * j) = make_float4(o4[0], o4[1], o4[2], o4[3]);
                        if (GRAD)
                            *reinterpret_cast<float4 *>(hhist + 4 * j) = make_float4(h4[0], h4[1], h4[2], h4[3]);
                    } else {
                        // log Z: soft-min of the last costs per (block, warp)
                        if ((jj & 1) == 0) { lzm = kPosInf; lzs = 0.f; }
#pragma unroll
                        for (int c = 0; c < 4; ++c) smin_merge(lzm, lzs, kap * o4[c], 1.f);
                        if (jj & 1) {
                            float m = lzm, s = lzs;
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
                                const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
                                smin_merge(m, s, m2, s2);
                            }
                            if (lane == 0) {
                                const int part = part_of(rank, tid, jj);
#pragma unroll
                                for (int r = 0; r < kCL; ++r) {
                                    st_cluster(cbase[r] + soff(&sm.lz[z][part][0]), m);
                                    st_cluster(cbase[r] + soff(&sm.lz[z][part][1]), s);
                                }
                            }
                        }
                    }
                }
                finish_step(z, nb, !last && !drop, lmin, 0, slot_ws);
            }
        }
        // log2 Z = -(kappa O_{N-1} + log2-soft-min over all 16384 costs kappa S_N),
        // the soft-min merged over the 64 (block, warp) partials in order.
        cluster_sync();   // also publishes every CTA's history rows

        double logZ2[kSlots];
#pragma unroll
        for (int z = 0; z < kSlots; ++z) logZ2[z] = 0.0;
#pragma unroll
        for (int z = 0; z < kSlots; ++z) {
            if (!active[z]) continue;
            float m = kPosInf, s = 0.f;
            for (int i = 0; i < kParts; ++i) smin_merge(m, s, sm.lz[z][i][0], sm.lz[z][i][1]);
            logZ2[z] = -((double)kap * O[z] + (double)m - (double)log2f(s));
            if (!GRAD && rank == 0 && tid == 0 && logZ_out)
                logZ_out[sidx[z]] = (float)(logZ2[z] * (double)kLn2) + poison_value(bad_T, status);
        }
        if (tid == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
#pragma unroll
            for (int z = 0; z < kSlots; ++z)
                if (active[z]) issue_rows(z, N - 1, slot_ws);
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
                // inputs: costs of Bt_{t+1} minus the global minimum, Bb_{t+1},
                // and this step's alpha / H rows
                float sigma = 0.f;
                const float *in = nullptr;   // Bt_{t+1}, Bb_{t+1} (none at t = N-2: all zero)
                if (t != N - 2) {
                    const int x = use[z] & 1;
                    const uint32_t bar = sbase + soff(&sm.full[z][x]);
                    if (tid == 0 && !failed) mbar_arm(bar, kBytes);
                    wait_bar<SleepOf<GRAD>::value>(bar, (use[z] >> 1) & 1, status, failed);
                    sigma = cluster_min(sm.maxslot[z][x], lane);
                    in = &sm.buf[z][x][0][0];
                    ++use[z];
                }
                U[z] += (double)sigma;
                const bool hrow = tn > 0;    // this step's alpha / H rows are staged
                if (hrow) {
                    wait_bar<SleepOf<GRAD>::value>(sbase + soff(&sm.hbar[z]), hcnt[z] & 1, status, failed);
                    ++hcnt[z];
                }
                const double Oa = tn > 0 ? sm.offs[z][tn - 1] : 0.0;
                const float Cb = (float)(-(logZ2[z] + (double)kap * (Oa + U[z])));
                const int nb = use[z] & 1;
                const float w = sm.w[z][tn];
                float gq = 0.f, gs = 0.f, st = 0.f;
                if (GRAD) {
                    gq = sm.g[z][tn];
                    st = sm.sf[z][tn];
                    gs = gq * st;
                }
                const uint32_t bar_off = soff(&sm.full[z][nb]);
                const uint32_t buf_off = soff(&sm.buf[z][nb][0][0]);
                const F2 W = bc(w), Gq = bc(gq), CB = bc(Cb), NK = bc(-kap), MIK = bc(-ikap),
                         ST = bc(st);
                F2 acc = bc(0.f);
                float lmin = kPosInf;
                F2 obs[kJPT][2], bbos[kJPT][2];   // the step's outputs, when sent after the arithmetic
#pragma unroll
                for (int jj = 0; jj < kJPT; ++jj) {
                    const int j = jg[jj];
                    const int jl = jl_of(tid, jj);
                    if ((jj & 1) == 0) acc = bc(0.f);   // first butterfly of a reduction block
                    // my butterfly's inputs (minus the global minimum) and history values
                    float bin[4] = {0.f, 0.f, 0.f, 0.f}, bbin[4] = {0.f, 0.f, 0.f, 0.f};
                    if (in) {
                        const float4 v = *reinterpret_cast<const float4 *>(in + 4 * jl);
                        bin[0] = v.x - sigma; bin[1] = v.y - sigma;
                        bin[2] = v.z - sigma; bin[3] = v.w - sigma;
                        if (GRAD) {
                            const float4 u = *reinterpret_cast<const float4 *>(in + kIn + 4 * jl);
                            bbin[0] = u.x; bbin[1] = u.y; bbin[2] = u.z; bbin[3] = u.w;
                        }
                    }
                    float a4[4] = {a0, a0, a0, a0}, h4[4] = {0.f, 0.f, 0.f, 0.f};
                    if (hrow) {
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            a4[p] = sm.hst[z][0][p * kJPC + jl];
                            if (GRAD) h4[p] = sm.hst[z][kPlanes - 1][p * kJPC + jl];
                        }
                    }
                    // inputs shared by both output-group pairs, as f32x2 broadcasts
                    F2 Bb[4], Yb[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        Bb[c] = bc(bin[c]);
                        Yb[c] = bc(bbin[c] - gs);
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {          // output groups p' = 2h, 2h+1
                        F2 xc[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const F2 d = sub2(cq[jj][c][h], W);
                            xc[c] = fma2(d, d, Bb[c]);
                        }
                        const F2 M = mk(min4(xc[0].x, xc[1].x, xc[2].x, xc[3].x),
                                        min4(xc[0].y, xc[1].y, xc[2].y, xc[3].y));
                        const F2 KM = mul2(M, bc(kap));
                        F2 e[4];
#pragma unroll
                        for (int c = 0; c < 4; ++c) e[c] = ex2p(fma2(xc[c], NK, KM));
                        const F2 S = add2(add2(e[0], e[1]), add2(e[2], e[3]));
                        const F2 f = ex2p(fma2(add2(M, mk(a4[2 * h], a4[2 * h + 1])), NK, CB));
                        F2 ob = bc(0.f), bbo = bc(0.f);
                        if (t >= 0) {
                            ob = fma2(mk(lg2(S.x), lg2(S.y)), MIK, M);
                            lmin = min3(lmin, ob.x, ob.y);
                        }
                        if (!GRAD) {
                            F2 ec = mul2(e[0], cq[jj][0][h]);
#pragma unroll
                            for (int c = 1; c < 4; ++c) ec = fma2(e[c], cq[jj][c][h], ec);
                            acc = fma2(f, ec, acc);
                        } else {
                            const F2 Hh = mk(h4[2 * h], h4[2 * h + 1]);
                            F2 ey = bc(0.f), dl = bc(0.f);
#pragma unroll
                            for (int c = 0; c < 4; ++c) {
                                const F2 y = fma2(cq[jj][c][h], Gq, Yb[c]);
                                ey = fma2(e[c], y, ey);
                                const F2 cm = sub2(cq[jj][c][h], ST);
                                dl = fma2(mul2(e[c], add2(y, Hh)), cm, dl);
                            }
                            bbo = mul2(ey, mk(rcp(S.x), rcp(S.y)));
                            acc = fma2(f, dl, acc);
                        }
                        if (kHoistSends) {
                            obs[jj][h] = ob;
                            bbos[jj][h] = bbo;
                        } else if (t >= 0 && !failed) {
                            send_beta(j, h, ob, bbo, buf_off, bar_off);
                        }
                    }
                    if (jj & 1) {
                        // the (block, warp) partial of this step
                        float v = acc.x + acc.y;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                        if (lane == 0)
                            slot_ws[z][lay.part + (long)tn * kParts + part_of(rank, tid, jj)] = v;
                    }
                }
                if (kHoistSends && t >= 0 && !failed) {
#pragma unroll
                    for (int jj = 0; jj < kJPT; ++jj)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            send_beta(jg[jj], h, obs[jj][h], bbos[jj][h], buf_off, bar_off);
                }
                finish_step(z, nb, t >= 0, lmin, tn - 1, slot_ws);
            }
        }
        __syncthreads();

        // Per-step partials of the 4 x 16 (block, warp) pairs, added in a fixed order.
        cluster_sync();
        if (rank == 0) {
            const float scale = GRAD ? two_over_T : 1.f;
            // NaN if a wait of this cluster (or any earlier failure of the
            // call) gave up: the cluster_sync above orders its status write
            const float poison = poison_value(bad_T, status);
#pragma unroll
            for (int z = 0; z < kSlots; ++z) {
                if (!active[z]) continue;
                const float *part = slot_ws[z] + lay.part;
                for (int tn = tid; tn < N; tn += kNT) {
                    const float4 *p4 = reinterpret_cast<const float4 *>(part + (long)tn * kParts);
                    float sum = 0.f;
#pragma unroll
                    for (int i = 0; i < kParts / 4; ++i) {
                        const float4 v = __ldcg(p4 + i);
                        sum += ((v.x + v.y) + v.z) + v.w;
                    }
                    out[sidx[z] * N + tn] = scale * sum + poison;
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
                wait_bar<SleepOf<GRAD>::value>(sbase + soff(&sm.hbar[z]), k & 1, status, f2);
    }
    cluster_sync();
    // Launched as the dependent of another grid (programmatic stream
    // serialization), this grid completes only after that one has, so later
    // work in the stream sees the results of both.  Otherwise a no-op.
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Host side of this instance.

namespace {

template <bool GRAD>
int max_clusters_of() {
    static int cached[2][64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    int &c = cached[GRAD ? 1 : 0][dev];
    if (c > 0) return c;
    const size_t smem = sizeof(Smem<GRAD>);
    if (cudaFuncSetAttribute(l16_kernel<GRAD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(sms / kCL * kCL), 1, 1);
    cfg.blockDim = dim3(kNT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, l16_kernel<GRAD>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    c = n;
    return n;
}

template <bool GRAD>
cudaError_t launch_of(const LaunchArgs &a, int ncl, float *ws, bool dependent) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(ncl * kCL), 1, 1);
    cfg.blockDim = dim3(kNT, 1, 1);
    cfg.dynamicSmemBytes = sizeof(Smem<GRAD>);
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    if (GRAD)
        return cudaLaunchKernelEx(&cfg, l16_kernel<GRAD>, a.seq, a.cb, a.T_dev, a.soft_in, a.grad,
                                  a.B, a.N, a.dseq, (float *)nullptr, ws, a.status, a.claim,
                                  a.drop_sends);
    return cudaLaunchKernelEx(&cfg, l16_kernel<GRAD>, a.seq, a.cb, a.T_dev, (const float *)nullptr,
                              (const float *)nullptr, a.B, a.N, a.soft, a.logZ, ws, a.status,
                              a.claim, a.drop_sends);
}

}  // namespace

int max_clusters(int mode) {
    return mode == kModeBackward ? max_clusters_of<true>() : max_clusters_of<false>();
}

int slots(int mode) {
    return mode == kModeBackward ? SlotsOf<true>::value : SlotsOf<false>::value;
}

size_t slot_bytes(int N, int mode) {
    return (size_t)slot_layout(N, mode == kModeBackward).total * 4;
}

cudaError_t launch(const LaunchArgs &a, int ncl, float *ws, bool dependent) {
    if (ncl <= 0) return cudaErrorInvalidConfiguration;
    return a.mode == kModeBackward ? launch_of<true>(a, ncl, ws, dependent)
                                   : launch_of<false>(a, ncl, ws, dependent);
}

}  // namespace BCJR_L16_NS

#if BCJR_L16_CL == 2
// ---------------------------------------------------------------------------
// Dispatcher for L=16, k=2, V=1.
//
// Forward: the 2-CTA instance (two slots) on every SM.  Backward: the 2-CTA
// instance has room for one slot, the 4-CTA instance for two but tiles only
// 132 of the 148 SMs.  Both run side by side: the 4-CTA grid first, then the
// 2-CTA grid on the SMs it leaves free, launched as its programmatic
// dependent; both take sequences from one counter (measured on B200 with
// 4096 sequences: 2-CTA alone 114 ms, 4-CTA alone 116 ms, both ~105 ms).
// The BCJR_OPT_L16_BACKWARD_CLUSTER option (2 or 4) runs one instance alone
// in the backward, BCJR_OPT_L16_FORWARD_CLUSTER=4 the 4-CTA instance in the
// forward (tests).  Results do not depend on the instance that runs a
// sequence.

namespace {

struct Plan {
    int n4 = 0;   // 4-CTA clusters
    int n2 = 0;   // 2-CTA clusters
};

Plan plan_for(int B, int mode) {
    Plan p;
    const long b = B > 0 ? B : 1;
    const bool bwd = mode == kModeBackward;
    const int force = test_option(bwd ? kOptL16Backward : kOptL16Forward);
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // SMs left free for concurrent kernels (bcjr_set_reserved_sms)
    const int free_sms = sms - reserved_sms();
    int max2 = l16::max_clusters(mode);
    if (max2 > free_sms / 2) max2 = free_sms / 2;
    const long need2 = (b + l16::slots(mode) - 1) / l16::slots(mode);
    int max4 = l16c4::max_clusters(mode);
    if (max4 > free_sms / 4) max4 = free_sms / 4;
    const long need4 = (b + l16c4::slots(mode) - 1) / l16c4::slots(mode);
    if (force == 4 && max4 > 0) {
        p.n4 = (int)(need4 < max4 ? need4 : max4);
        return p;
    }
    // the forward, and a batch that one round of the 2-CTA instance covers:
    // the 2-CTA instance alone
    if (!bwd || force == 2 || max4 <= 0 || need2 <= max2) {
        p.n2 = (int)(need2 < max2 ? need2 : max2);
        if (p.n2 < 0) p.n2 = 0;
        return p;
    }
    p.n4 = max4;
    p.n2 = (free_sms - 4 * max4) / 2;
    if (p.n2 < 0) p.n2 = 0;
    return p;
}

size_t region4(const Plan &p, int N, int mode) {
    return ((size_t)p.n4 * l16c4::slots(mode) * l16c4::slot_bytes(N, mode) + 255) & ~(size_t)255;
}

}  // namespace

bool l16_applicable(int B, int N, int L, int BB, int V) {
    (void)B;
    return L == l16::kL && BB == l16::kB && V == 1 && N >= 2 && N <= l16::kNMax;
}

int l16_clusters(int B, int mode) {
    const Plan p = plan_for(B, mode);
    return p.n2 + p.n4;
}

size_t l16_workspace_bytes(int B, int N, int mode) {
    const Plan p = plan_for(B, mode);
    if (p.n2 + p.n4 <= 0) return 0;
    return region4(p, N, mode) + (size_t)p.n2 * l16::slots(mode) * l16::slot_bytes(N, mode);
}

int l16_launches(int B, int mode) {
    const Plan p = plan_for(B, mode);
    return (p.n4 > 0) + (p.n2 > 0);
}

cudaError_t launch_l16(const LaunchArgs &a) {
    const Plan p = plan_for(a.B, a.mode);
    if (p.n2 + p.n4 <= 0) return cudaErrorInvalidConfiguration;
    if (l16_workspace_bytes(a.B, a.N, a.mode) > a.ws_data_bytes) return cudaErrorInvalidValue;
    char *ws = static_cast<char *>(a.ws_data);
    cudaError_t e = cudaSuccess;
    if (p.n4 > 0) {
        e = l16c4::launch(a, p.n4, reinterpret_cast<float *>(ws), false);
        if (e != cudaSuccess) return e;
    }
    if (p.n2 > 0)
        e = l16::launch(a, p.n2, reinterpret_cast<float *>(ws + region4(p, a.N, a.mode)), p.n4 > 0);
    return e;
}
#endif  // BCJR_L16_CL == 2

}  // namespace bcjr
