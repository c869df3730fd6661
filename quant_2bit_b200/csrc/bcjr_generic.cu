// Generic BCJR kernels: any L <= 16, b = kV in 1..4, V in {1, 2}.
//
// One thread block per sequence (persistent loop over sequences), the group
// vectors A_t / H_t of every step kept in a per-block workspace slot in global
// memory (L2-resident for small L), Bt / Bb in ping-pong buffers.  These are
// the correctness path for every shape the reference accepts
// (build_pred_succ_tables(L, k, V), src/bcjr/forward_backward.py:62-86); the
// production shape L=16, b=2, V=1 has a dedicated cluster kernel
// (bcjr_l16.cu).  The recursions are documented in bcjr_common.cuh.
#include "bcjr_common.cuh"
#include "bcjr_kernels.h"

namespace bcjr {

namespace {

template <int V>
__device__ __forceinline__ float energy2(const float *__restrict__ cb, long q,
                                         const float (&w)[V], float kappa) {
    float d2 = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
        float d = __ldg(cb + q * V + v) - w[v];
        d2 = fmaf(d, d, d2);
    }
    return -kappa * d2;
}

template <int V>
__device__ __forceinline__ void load_w(const float *__restrict__ p, float (&w)[V]) {
#pragma unroll
    for (int v = 0; v < V; ++v) w[v] = __ldg(p + v);
}

// Per-step renormalisation.  Each sweep subtracts from its inputs the maximum
// of the values the previous step wrote (a block-wide max, published through
// per-warp slots in shared memory and read after the step's barrier), and
// accumulates those shifts in double.  Without it |A| grows ~linearly in t
// and the fp32 rounding of A (relative to |A|) dominates at low T.
struct StepMax {
    float *slots;  // 2 x 32 per-warp maxima, double-buffered by step parity
    __device__ __forceinline__ void publish(float m, int parity) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((threadIdx.x & 31) == 0) slots[parity * 32 + (threadIdx.x >> 5)] = m;
    }
    // Max over the warps of step `parity`; call after the step's barrier.
    __device__ __forceinline__ float read(int parity) const {
        const int nw = blockDim.x >> 5;
        float m = kNegInf;
        for (int i = 0; i < nw; ++i) m = fmaxf(m, slots[parity * 32 + i]);
        return m;
    }
};

// Forward alpha sweep for one sequence.  Row t+1 of Ah holds
// S_{t+1} = A_{t+1} - O_t, and Off[t] = O_t (double), where O_t is the sum of
// the shifts applied to the inputs up to step t (so A_t = S_t + O_{t-1},
// O_{-1} = 0, S_0 = A_0 = b).  With GRAD, Hh holds H_0..H_N (shift-free).
template <int BB, int V, bool GRAD>
__device__ void alpha_sweep(const float *__restrict__ w, const float *__restrict__ cb,
                            const float *__restrict__ g, const float *__restrict__ sf,
                            int N, int L, float kappa, float *Ah, float *Hh, double *Off,
                            StepMax smax) {
    constexpr int NB = 1 << BB;
    const int G = 1 << (L - BB);
    for (int h = threadIdx.x; h < G; h += blockDim.x) {
        Ah[h] = (float)BB;
        if (GRAD) Hh[h] = 0.f;
    }
    double O = 0.0;
    float shift = (float)BB;  // max of S_0
    for (int t = 0; t < N; ++t) {
        __syncthreads();
        if (t > 0) shift = smax.read((t - 1) & 1);
        O += (double)shift;
        if (threadIdx.x == 0) Off[t] = O;
        float wt[V], gt[V];
        load_w<V>(w + (long)t * V, wt);
        float gs = 0.f;
        if (GRAD) {
            load_w<V>(g + (long)t * V, gt);
#pragma unroll
            for (int v = 0; v < V; ++v) gs = fmaf(gt[v], __ldg(sf + (long)t * V + v), gs);
        }
        const float *Ain = Ah + (long)t * G;
        float *Aout = Ah + (long)(t + 1) * G;
        const float *Hin = GRAD ? Hh + (long)t * G : nullptr;
        float *Hout = GRAD ? Hh + (long)(t + 1) * G : nullptr;
        float lmax = kNegInf;
        for (int h = threadIdx.x; h < G; h += blockDim.x) {
            float x[NB], F[NB];
            float m = kNegInf;
#pragma unroll
            for (int p = 0; p < NB; ++p) {
                const long q = (long)p * G + h;
                const int src = (int)(q >> BB);
                x[p] = energy2<V>(cb, q, wt, kappa) + (Ain[src] - shift);
                m = fmaxf(m, x[p]);
                if (GRAD) {
                    float gam = -gs;
#pragma unroll
                    for (int v = 0; v < V; ++v) gam = fmaf(gt[v], __ldg(cb + q * V + v), gam);
                    F[p] = gam + Hin[src];
                }
            }
            float s = 0.f, hf = 0.f;
#pragma unroll
            for (int p = 0; p < NB; ++p) {
                const float e = ex2(x[p] - m);
                s += e;
                if (GRAD) hf = fmaf(e, F[p], hf);
            }
            const float a = m + lg2(s);
            Aout[h] = a;
            lmax = fmaxf(lmax, a);
            if (GRAD) Hout[h] = hf / s;
        }
        smax.publish(lmax, t & 1);
    }
    __syncthreads();
}

// log2 Z = O_{N-1} + LSE2_h S_N(h).
__device__ __forceinline__ double log2_partition(const float *SN, int G, const double *Off,
                                                 int N, float *sh) {
    float lm = kNegInf, ls = 0.f;
    for (int h = threadIdx.x; h < G; h += blockDim.x) lse_merge(lm, ls, SN[h], 1.f);
    const float l = block_lse2(lm, ls, sh);
    return Off[N - 1] + (double)l;
}

}  // namespace

// Workspace slot of one block (floats, then doubles at an 8-byte boundary):
//   Ah  (N+1) x G   S_t rows (alpha, shifted)
//   Hh  (N+1) x G   H_t rows                       [backward]
//   Bt  2 x G       beta ping-pong  (internals: N x G history)
//   Bb  2 x G       Bb ping-pong                   [backward]
//   Off N doubles   O_t;  Uoff N doubles (internals: beta shifts per step)
struct Slot {
    float *Ah, *Hh, *Bt, *Bb;
    double *Off, *Uoff;
};

__host__ __device__ inline long slot_float_count(int N, int L, int BB, int mode) {
    const long G = 1L << (L - BB);
    long f = (long)(N + 1) * G;                          // Ah
    if (mode == kModeBackward) f += (long)(N + 1) * G;   // Hh
    f += (mode == kModeInternals) ? (long)N * G : 2 * G; // Bt
    if (mode == kModeBackward) f += 2 * G;               // Bb
    f = (f + 1) & ~1L;                                   // align doubles
    f += 2L * N;                                         // Off
    if (mode == kModeInternals) f += 2L * N;             // Uoff
    return f;
}

__device__ inline Slot make_slot(float *base, int N, int L, int BB, int mode) {
    const long G = 1L << (L - BB);
    Slot s;
    float *p = base;
    s.Ah = p; p += (long)(N + 1) * G;
    s.Hh = nullptr;
    if (mode == kModeBackward) { s.Hh = p; p += (long)(N + 1) * G; }
    s.Bt = p; p += (mode == kModeInternals) ? (long)N * G : 2 * G;
    s.Bb = nullptr;
    if (mode == kModeBackward) { s.Bb = p; p += 2 * G; }
    long used = p - base;
    used = (used + 1) & ~1L;
    s.Off = reinterpret_cast<double *>(base + used);
    s.Uoff = (mode == kModeInternals) ? s.Off + N : nullptr;
    return s;
}

// O_{t-1}: the alpha shift of row t (A_t = S_t + O_{t-1}); O_{-1} = 0.
__device__ __forceinline__ double alpha_offset(const double *Off, int t) {
    return t > 0 ? Off[t - 1] : 0.0;
}

// mode: kModeForward (soft, logZ) or kModeInternals (P, log_alpha, log_beta).
template <int BB, int V>
__global__ void __launch_bounds__(512)
gen_forward_kernel(const float *__restrict__ seq, const float *__restrict__ cb,
                   const float *__restrict__ T_dev, int B, int N, int L,
                   float *__restrict__ soft, float *__restrict__ logZ,
                   float *__restrict__ ws, long slot_floats, int mode,
                   float *__restrict__ Pout, float *__restrict__ LAout,
                   float *__restrict__ LBout) {
    constexpr int NB = 1 << BB;
    __shared__ float sh[2 * 32 + 8 * (V + 1) + 64];
    __shared__ float smax_slots[64];
    StepMax smax{smax_slots};
    const int G = 1 << (L - BB);
    const float T = __ldg(T_dev);
    const float kappa = kLog2e / T;
    const float poison = poison_value(bad_temperature(T), nullptr);   // NaN for an unusable T
    const Slot sl = make_slot(ws + (long)blockIdx.x * slot_floats, N, L, BB, mode);
    const bool internals = (mode == kModeInternals);

    for (int bs = blockIdx.x; bs < B; bs += gridDim.x) {
        const float *w = seq + (long)bs * N * V;
        alpha_sweep<BB, V, false>(w, cb, nullptr, nullptr, N, L, kappa, sl.Ah, nullptr,
                                  sl.Off, smax);
        const double logZ2 = log2_partition(sl.Ah + (long)N * G, G, sl.Off, N, sh);
        if (threadIdx.x == 0 && logZ) logZ[bs] = (float)(logZ2 * (double)kLn2) + poison;

        // beta sweep (backward in time) with P and soft for step t+1
        float *Rlast = internals ? sl.Bt + (long)(N - 1) * G : sl.Bt + (long)((N - 1) & 1) * G;
        for (int r = threadIdx.x; r < G; r += blockDim.x) Rlast[r] = 0.f;
        if (internals && threadIdx.x == 0) sl.Uoff[N - 1] = 0.0;
        double U = 0.0;
        for (int t = N - 2; t >= -1; --t) {
            const int tn = t + 1;
            __syncthreads();
            const float sigma = (t == N - 2) ? 0.f : smax.read(tn & 1);
            U += (double)sigma;
            float wt[V];
            load_w<V>(w + (long)tn * V, wt);
            const float *Rn = internals ? sl.Bt + (long)tn * G : sl.Bt + (long)(tn & 1) * G;
            float *Ro = (t >= 0) ? (internals ? sl.Bt + (long)t * G : sl.Bt + (long)(t & 1) * G)
                                 : nullptr;
            const float *Sc = sl.Ah + (long)tn * G;
            const float C = (float)(logZ2 - alpha_offset(sl.Off, tn) - U);
            double acc[V];  // per-thread partial in double: up to G/blockDim groups
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = 0.0;
            float lmax = kNegInf;
            for (int r = threadIdx.x; r < G; r += blockDim.x) {
                float x[NB];
                float m = kNegInf;
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    const long q = (long)r * NB + c;
                    x[c] = energy2<V>(cb, q, wt, kappa) + (Rn[q & (G - 1)] - sigma);
                    m = fmaxf(m, x[c]);
                }
                float e[NB], s = 0.f;
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    e[c] = ex2(x[c] - m);
                    s += e[c];
                }
                if (Ro) {
                    const float bo = m + lg2(s);
                    Ro[r] = bo;
                    lmax = fmaxf(lmax, bo);
                }
                if (!internals) {
                    const float f = ex2(m + Sc[r] - C);
                    float gsum[V];
#pragma unroll
                    for (int v = 0; v < V; ++v) gsum[v] = 0.f;
#pragma unroll
                    for (int c = 0; c < NB; ++c) {
                        const long q = (long)r * NB + c;
#pragma unroll
                        for (int v = 0; v < V; ++v) gsum[v] = fmaf(e[c], __ldg(cb + q * V + v), gsum[v]);
                    }
#pragma unroll
                    for (int v = 0; v < V; ++v) acc[v] += (double)(f * gsum[v]);
                }
            }
            smax.publish(lmax, t & 1);
            if (internals) {
                // Ro holds Bt_t - U_t' where U_t' adds the shift of the next step:
                // record U (the shift of Rn's row) for row tn.
                if (threadIdx.x == 0) sl.Uoff[tn] = U - (double)sigma;
            } else {
                float accf[V];
#pragma unroll
                for (int v = 0; v < V; ++v) accf[v] = (float)acc[v];
                block_sum<V>(accf, sh);
                if (threadIdx.x == 0) {
#pragma unroll
                    for (int v = 0; v < V; ++v) soft[((long)bs * N + tn) * V + v] = accf[v] + poison;
                }
            }
        }
        __syncthreads();

        if (internals) {
            // Row t of Bt holds Bt_t - Uoff[t]; materialise (N, 2^L) outputs.
            const long S = 1L << L;
            for (int t = 0; t < N; ++t) {
                float wt[V];
                load_w<V>(w + (long)t * V, wt);
                const float *St = sl.Ah + (long)t * G;
                const float *Rt = sl.Bt + (long)t * G;
                const double Oa = alpha_offset(sl.Off, t), Ub = sl.Uoff[t];
                const float Cp = (float)(logZ2 - Oa - Ub);
                const long base = ((long)bs * N + t) * S;
                for (long s = threadIdx.x; s < S; s += blockDim.x) {
                    const float a2 = energy2<V>(cb, s, wt, kappa) + St[s >> BB];
                    const float b2 = Rt[s & (G - 1)];
                    if (LAout) LAout[base + s] = (float)(((double)a2 + Oa) * (double)kLn2) + poison;
                    if (LBout) LBout[base + s] = (float)(((double)b2 + Ub) * (double)kLn2) + poison;
                    if (Pout) Pout[base + s] = exp2f(a2 + b2 - Cp) + poison;
                }
            }
            __syncthreads();
        }
    }
}

template <int BB, int V>
__global__ void __launch_bounds__(512)
gen_backward_kernel(const float *__restrict__ seq, const float *__restrict__ cb,
                    const float *__restrict__ T_dev, const float *__restrict__ soft,
                    const float *__restrict__ grad, int B, int N, int L,
                    float *__restrict__ dseq, float *__restrict__ ws, long slot_floats) {
    constexpr int NB = 1 << BB;
    __shared__ float sh[2 * 32 + 8 * (V + 1) + 64];
    __shared__ float smax_slots[64];
    StepMax smax{smax_slots};
    const int G = 1 << (L - BB);
    const float T = __ldg(T_dev);
    const float kappa = kLog2e / T;
    const float poison = poison_value(bad_temperature(T), nullptr);   // NaN for an unusable T
    const float two_over_T = 2.f / T;
    const Slot sl = make_slot(ws + (long)blockIdx.x * slot_floats, N, L, BB, kModeBackward);

    for (int bs = blockIdx.x; bs < B; bs += gridDim.x) {
        const float *w = seq + (long)bs * N * V;
        const float *g = grad + (long)bs * N * V;
        const float *sf = soft + (long)bs * N * V;
        alpha_sweep<BB, V, true>(w, cb, g, sf, N, L, kappa, sl.Ah, sl.Hh, sl.Off, smax);
        const double logZ2 = log2_partition(sl.Ah + (long)N * G, G, sl.Off, N, sh);

        for (int r = threadIdx.x; r < G; r += blockDim.x) {
            sl.Bt[(long)((N - 1) & 1) * G + r] = 0.f;
            sl.Bb[(long)((N - 1) & 1) * G + r] = 0.f;
        }
        double U = 0.0;
        for (int t = N - 2; t >= -1; --t) {
            const int tn = t + 1;
            __syncthreads();
            const float sigma = (t == N - 2) ? 0.f : smax.read(tn & 1);
            U += (double)sigma;
            float wt[V], gt[V], st[V];
            load_w<V>(w + (long)tn * V, wt);
            load_w<V>(g + (long)tn * V, gt);
            load_w<V>(sf + (long)tn * V, st);
            float gs = 0.f;
#pragma unroll
            for (int v = 0; v < V; ++v) gs = fmaf(gt[v], st[v], gs);
            const float *Rn = sl.Bt + (long)(tn & 1) * G;
            const float *Bbn = sl.Bb + (long)(tn & 1) * G;
            float *Ro = sl.Bt + (long)(t & 1) * G;
            float *Bbo = sl.Bb + (long)(t & 1) * G;
            const float *Sc = sl.Ah + (long)tn * G;
            const float *Hc = sl.Hh + (long)tn * G;
            const float C = (float)(logZ2 - alpha_offset(sl.Off, tn) - U);
            // d_seq_u = (2/T) sum_s dl_u(s) (c(s) - soft_u): the reference's
            // (2/T)(sum dl c - w sum dl) with sum_s dl_u(s) = 0 used exactly, which
            // makes the result insensitive to a common shift of gam/H/Bb (e.g.
            // the rounding of soft_u used to centre gam).
            double acc[V];  // per-thread partial in double: up to G/blockDim groups
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = 0.0;
            float lmax = kNegInf;
            for (int r = threadIdx.x; r < G; r += blockDim.x) {
                float x[NB], y[NB];
                float m = kNegInf;
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    const long q = (long)r * NB + c;
                    const int nx = (int)(q & (G - 1));
                    x[c] = energy2<V>(cb, q, wt, kappa) + (Rn[nx] - sigma);
                    float gam = -gs;
#pragma unroll
                    for (int v = 0; v < V; ++v) gam = fmaf(gt[v], __ldg(cb + q * V + v), gam);
                    y[c] = gam + Bbn[nx];
                    m = fmaxf(m, x[c]);
                }
                float e[NB], s = 0.f, bb = 0.f;
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    e[c] = ex2(x[c] - m);
                    s += e[c];
                    bb = fmaf(e[c], y[c], bb);
                }
                if (t >= 0) {
                    const float bo = m + lg2(s);
                    Ro[r] = bo;
                    lmax = fmaxf(lmax, bo);
                    Bbo[r] = bb / s;
                }
                const float f = ex2(m + Sc[r] - C);
                const float hr = Hc[r];
                float gsum[V];
#pragma unroll
                for (int v = 0; v < V; ++v) gsum[v] = 0.f;
#pragma unroll
                for (int c = 0; c < NB; ++c) {
                    const long q = (long)r * NB + c;
                    const float dl = e[c] * (y[c] + hr);
#pragma unroll
                    for (int v = 0; v < V; ++v) gsum[v] = fmaf(dl, __ldg(cb + q * V + v) - st[v], gsum[v]);
                }
#pragma unroll
                for (int v = 0; v < V; ++v) acc[v] += (double)(f * gsum[v]);
            }
            smax.publish(lmax, t & 1);
            float accf[V];
#pragma unroll
            for (int v = 0; v < V; ++v) accf[v] = (float)acc[v];
            block_sum<V>(accf, sh);
            if (threadIdx.x == 0) {
#pragma unroll
                for (int v = 0; v < V; ++v) dseq[((long)bs * N + tn) * V + v] = two_over_T * accf[v] + poison;
            }
        }
        __syncthreads();
    }
}

// ----------------------------------------------------------------------------
// Host-side launchers.

namespace {

long gen_slot_floats(int N, int L, int BB, int mode) {
    return slot_float_count(N, L, BB, mode);
}

int gen_threads(int L, int BB) {
    const int G = 1 << (L - BB);
    if (G >= 4096) return 512;
    if (G >= 1024) return 256;
    return 128;
}

template <int BB, int V>
cudaError_t launch_gen(const LaunchArgs &a) {
    const int nt = gen_threads(a.L, BB);
    const long sf = gen_slot_floats(a.N, a.L, BB, a.mode);
    float *ws = reinterpret_cast<float *>(a.ws_data);
    if (a.mode == kModeBackward) {
        gen_backward_kernel<BB, V><<<a.grid, nt, 0, a.stream>>>(
            a.seq, a.cb, a.T_dev, a.soft_in, a.grad, a.B, a.N, a.L, a.dseq, ws, sf);
    } else {
        gen_forward_kernel<BB, V><<<a.grid, nt, 0, a.stream>>>(
            a.seq, a.cb, a.T_dev, a.B, a.N, a.L, a.soft, a.logZ, ws, sf,
            a.mode, a.P, a.LA, a.LB);
    }
    return cudaGetLastError();
}

}  // namespace

size_t generic_workspace_bytes(int B, int N, int L, int BB, int V, int mode, int num_sms) {
    (void)V;
    const long sf = gen_slot_floats(N, L, BB, mode);
    const long slot_bytes = sf * 4;
    // At most 2 blocks per SM in flight, and at most ~4 GiB of slots.
    long slots = 2L * num_sms;
    const long cap = (4L << 30) / slot_bytes;
    if (slots > cap) slots = cap > 0 ? cap : 1;
    if (slots > B) slots = B;
    if (slots < 1) slots = 1;
    return (size_t)(slots * slot_bytes);
}

int generic_grid(int B, int N, int L, int BB, int mode, size_t ws_data_bytes) {
    const long slot_bytes = gen_slot_floats(N, L, BB, mode) * 4;
    long slots = (long)(ws_data_bytes / slot_bytes);
    if (slots > B) slots = B;
    return (int)slots;
}

cudaError_t launch_generic(const LaunchArgs &a) {
    switch (a.BB * 10 + a.V) {
        case 11: return launch_gen<1, 1>(a);
        case 21: return launch_gen<2, 1>(a);
        case 31: return launch_gen<3, 1>(a);
        case 41: return launch_gen<4, 1>(a);
        case 22: return launch_gen<2, 2>(a);
        case 42: return launch_gen<4, 2>(a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bcjr
