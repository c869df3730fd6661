// Shared device helpers for the BCJR kernels (sm_100a).
//
// Conventions used by every kernel in this library
// ------------------------------------------------
// * Messages are kept in log2 units: x2 = x * log2(e).  The local energy of
//   state q at step t is  e2_t(q) = -kappa * |c(q) - w_t|^2,  kappa = log2(e)/T,
//   which is the reference's _local_log_prob (src/bcjr/forward_backward.py:89-103)
//   times log2(e), written as a squared difference instead of the expanded
//   |c|^2 - 2<c,w> + |w|^2 (same value, less cancellation).
// * Group compression.  With b = kV branch bits and M = L - b, every state s
//   has the 2^b predecessors {p << M | s >> b}, shared by the 2^b states with
//   the same s >> b (forward_backward.py:78-80), and the 2^b successors
//   {(s << b | c) & mask}, shared by the states with the same s mod 2^M
//   (:82-84).  Hence
//       log_alpha_t(s) = e_t(s) + A_t(s >> b),
//       log_beta_t(s)  = Bt_t(s mod 2^M),
//   and only the 2^M group values A_t, Bt_t are carried between steps:
//       A_0 = b  (log2 of 2^b predecessors of log_alpha_{-1} = 0),
//       A_{t+1}(h) = LSE2_p [ e_t(p 2^M + h) + A_t((p 2^M + h) >> b) ],
//       Bt_{N-1} = 0,
//       Bt_t(r)   = LSE2_c [ e_{t+1}(r 2^b + c) + Bt_{t+1}((r 2^b + c) mod 2^M) ],
//       log2 Z    = LSE2_h A_N(h).
//   The marginal of a successor group reuses the exponentials of that LSE:
//       P_{t+1}(r 2^b + c) = 2^(x_c - m) * 2^(m + A_{t+1}(r) - log2 Z).
// * Gradient (the reference's analytic backward, bcjr_monolithic.py:191-243,
//   restated).  For the loss <g, soft>,  d loss / d log_local_u(s)
//   = P_u(s) (E[G | s_u = s] - E[G]) with G = sum_t <g_t, c(s_t)>.  With the
//   centred emission  gam_t(q) = <g_t, c(q) - soft_t>  the two conditional
//   expectations obey the same group-shared recursions as A and Bt:
//       H_0 = 0,    H_{t+1}(h) = sum_p pi_p [gam_t(q_p) + H_t(q_p >> b)],
//       Bb_{N-1}=0, Bb_t(r)    = sum_c sig_c [gam_{t+1}(s_c) + Bb_{t+1}(s_c mod 2^M)],
//   where pi, sig are the softmax weights of the A and Bt LSEs, and
//       dl_{t+1}(s_c) = P_{t+1}(s_c) (gam_{t+1}(s_c) + Bb_{t+1}(s_c mod 2^M) + H_{t+1}(r)),
//       d_seq_u       = (2/T) sum_s dl_u(s) (c(s) - w_u)
//                     = (2/T) sum_s dl_u(s) (c(s) - soft_u)     (sum_s dl_u(s) = 0).
//   The second form is the one evaluated: it is exact in the mathematics and
//   cancels any error common to all states (e.g. from rounding in soft_u).
//   No atomics, no (B,N,S) buffers.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace bcjr {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegInf = -__builtin_huge_valf();

// MUFU instructions, issued directly (ex2 / lg2 / rcp approximate forms).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float lg2(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Failure policy.  A call whose temperature is not positive and finite, or
// in which a bounded device-side wait gave up (non-zero status word), must
// not return numbers that look valid: every output gets poison_value() added,
// NaN in those cases and 0 otherwise, so the failure reaches the caller
// without a host synchronisation.
__device__ __forceinline__ bool bad_temperature(float T) {
    return !(T > 0.f && T < __builtin_huge_valf());
}
__device__ __forceinline__ float poison_value(bool bad, const int *status) {
    if (!bad && status) bad = *reinterpret_cast<const volatile int *>(status) != 0;
    return bad ? __int_as_float(0x7fffffff) : 0.f;
}

// Sum of NV values over a thread block; every thread gets the result.
// `sh` must hold (blockDim.x / 32) * NV floats plus NV.  Contains two
// __syncthreads().
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) sh[warp * NV + i] = v[i];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            float a = lane < nw ? sh[lane * NV + i] : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0) sh[nw * NV + i] = a;
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = sh[nw * NV + i];
}

// Merge two (max, sum-of-2^(x-max)) pairs.  A NaN partial makes the result
// NaN (NaN policy "propagate"); -inf partials (empty) are skipped.
__device__ __forceinline__ void lse_merge(float &m, float &s, float m2, float s2) {
    if (m2 > m) {
        s = s * ex2(m - m2) + s2;
        m = m2;
    } else if (m2 > kNegInf) {
        s = s + s2 * ex2(m2 - m);
    } else if (m2 != m2) {
        m = m2;
    }
}

// log2-sum-exp2 of per-thread (m, s) pairs over the block; every thread gets
// the result.  `sh` holds 2 * (blockDim.x / 32) + 1 floats.
__device__ __forceinline__ float block_lse2(float m, float s, float *sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        lse_merge(m, s, m2, s2);
    }
    if (lane == 0) {
        sh[2 * warp] = m;
        sh[2 * warp + 1] = s;
    }
    __syncthreads();
    if (warp == 0) {
        float a = lane < nw ? sh[2 * lane] : kNegInf;
        float b = lane < nw ? sh[2 * lane + 1] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float m2 = __shfl_xor_sync(0xffffffffu, a, o);
            float s2 = __shfl_xor_sync(0xffffffffu, b, o);
            lse_merge(a, b, m2, s2);
        }
        if (lane == 0) sh[2 * nw] = a + lg2(b);
    }
    __syncthreads();
    return sh[2 * nw];
}

}  // namespace bcjr
