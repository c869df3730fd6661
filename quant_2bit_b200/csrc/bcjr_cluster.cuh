// Device helpers shared by the thread-block-cluster kernels (bcjr_l16.cu,
// bcjr_b4.cu): cluster special registers, mbarriers with bounded waits,
// st.async into a peer CTA's shared memory, TMA bulk copies between global
// and shared memory (never with .multicast::cluster), f32x2 arithmetic and
// order-preserving float keys.
#pragma once

#include <cstdint>

#include "bcjr_common.cuh"

namespace bcjr {
namespace clu {

constexpr float kPosInf = __builtin_huge_valf();

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
// Non-blocking test of the phase (test_wait returns at once).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;"
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
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t a) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(a) : "memory");
}
// One TMA bulk copy global -> own shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: ~1 s, then BCJR_ERR_TIMEOUT in the status word.  Once any
// thread of the grid has failed, every later wait returns at once.
//
// A warp whose data is not there yet sleeps kWaitSleepNs between tests
// instead of polling: polling (including the retry loop a suspending
// try_wait compiles to) takes issue slots from the warps that have work,
// and measured on B200 a fixed ~400 ns sleep ran both cluster kernels
// ~15 % faster than a suspending try_wait (shorter sleeps poll too often,
// 800 ns and more oversleep).  A kernel with a single sequence in flight has
// nothing else to run while it waits, and prefers a shorter sleep (template
// argument).
#ifndef BCJR_WAIT_SLEEP_NS
#define BCJR_WAIT_SLEEP_NS 400
#endif
constexpr unsigned kWaitSleepNs = BCJR_WAIT_SLEEP_NS;

template <unsigned kSleepNs = kWaitSleepNs>
__device__ __forceinline__ void wait_bar(uint32_t bar, uint32_t parity, int *status,
                                         bool &failed) {
    if (failed) return;
    if (mbar_test(bar, parity)) return;
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (kSleepNs) __nanosleep(kSleepNs);
        if (mbar_test(bar, parity)) return;
        if ((i & 7) == 0) {
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

// f32x2 pairs (FADD2 / FMUL2 / FFMA2 through the sm_100 float2 builtins).
using F2 = float2;
__device__ __forceinline__ F2 mk(float a, float b) { return make_float2(a, b); }

// One float through the read-only path, as a load of its own (opaque to the
// load vectoriser).  A register-resident pair built from two such loads can
// be allocated straight into the register pair that the f32x2 instructions
// read.  Built from two lanes of different vector loads instead, the pair's
// halves are pinned to non-adjacent registers, and under register pressure
// the pair is re-formed with moves at every use (measured on B200: about two
// extra instructions per f32x2 use of a codebook pair).
__device__ __forceinline__ float ldg1(const float *p) {
    float v;
    asm("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ F2 ldg_pair(const float *p0, const float *p1) {
    return make_float2(ldg1(p0), ldg1(p1));
}
__device__ __forceinline__ F2 bc(float a) { return make_float2(a, a); }
__device__ __forceinline__ F2 add2(F2 a, F2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ F2 sub2(F2 a, F2 b) { return __fadd2_rn(a, make_float2(-b.x, -b.y)); }
__device__ __forceinline__ F2 mul2(F2 a, F2 b) { return __fmul2_rn(a, b); }

// Separately rounded sums for arithmetic that must equal the reference's
// bit for bit (the hard Viterbi costs a + d*d).  The compiler merges an
// f32x2 multiply and a following f32x2 add into one fused multiply-add, also
// when both are written as inline PTX with an explicit .rn and also under
// -fmad=false (measured on B200: the costs then followed fma(d, d, a), and a
// one-ulp near-tie between two predecessors took the other one); the scalar
// __fadd_rn is never merged.
__device__ __forceinline__ F2 add2_sep(F2 a, F2 b) {
    return mk(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
}
__device__ __forceinline__ F2 fma2(F2 a, F2 b, F2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float min3(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float min4(float a, float b, float c, float d) {
    return fminf(min3(a, b, c), d);
}
__device__ __forceinline__ F2 ex2p(F2 a) { return F2{ex2(a.x), ex2(a.y)}; }

// Minimum over the warp (all 32 lanes active).
__device__ __forceinline__ float redux_min(float v) {
    float r;
    asm volatile("redux.sync.min.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// Order-preserving map float -> int (and back): a < b  <=>  key(a) < key(b).
__device__ __forceinline__ int order_key(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float order_key_inv(int k) {
    return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff);
}

// Soft-min accumulator (m, s): value = m - lg2 s, s = sum 2^(m - x).
// A NaN partial makes the result NaN (NaN policy "propagate": a sequence
// with a NaN energy has a NaN log Z, hence NaN marginals, as in the
// reference); +inf partials (empty) are skipped.
__device__ __forceinline__ void smin_merge(float &m, float &s, float m2, float s2) {
    if (m2 < m) {
        s = s * ex2(m2 - m) + s2;
        m = m2;
    } else if (m2 < kPosInf) {
        s = s + s2 * ex2(m - m2);
    } else if (m2 != m2) {
        m = m2;
    }
}

// 8-byte st.async (two consecutive floats).
__device__ __forceinline__ void st_async2(uint32_t addr, float a, float b, uint32_t bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1,%2}, [%3];"
        ::"r"(addr), "f"(a), "f"(b), "r"(bar)
        : "memory");
}
// TMA bulk copy own shared memory -> global (bulk async-group of this thread).
__device__ __forceinline__ void bulk_s2g(void *dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(dst), "r"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Source shared memory of this thread's bulk stores may be overwritten.
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// This thread's bulk stores have completed (written to global memory).
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Order generic-proxy accesses to shared memory before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace clu
}  // namespace bcjr
