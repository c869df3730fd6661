// MUFU throughput probe (declared in include/bcjr_b200.h): the measured
// denominator of the MUFU roofline that bench.py reports for the BCJR kernels.
//
// Every thread runs eight independent chains a <- ex2(-a / 2) (one
// ex2.approx.ftz.f32 on the MUFU pipe and one multiply on the FMA pipe per
// link; the values stay in (0, 1], no denormals).  Eight chains per thread
// and 32 warps per SM keep the MUFU pipe busy; the multiplies and the loop
// take FMA and issue slots that the MUFU pipe does not share, so the launch
// runs at the MUFU pipe's throughput.  The result is stored only under a
// condition that never holds (the values are positive) but that the
// compiler cannot rule out.
#include <cstdint>

#include "../../include/bcjr_b200.h"
#include "bcjr_common.cuh"

namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeBlocksPerSm = 4;
constexpr int kProbeChains = 8;

__global__ void __launch_bounds__(kProbeThreads)
mufu_probe_kernel(float *out, int iters) {
    float a[kProbeChains];
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) a[c] = 0.01f * (float)(threadIdx.x & 63) + 0.1f * c;
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int c = 0; c < kProbeChains; ++c) a[c] = bcjr::ex2(a[c] * -0.5f);
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) s += a[c];
    if (s == -1.f) out[0] = s;
}

}  // namespace

extern "C" BCJR_API int bcjr_probe_mufu(float *out, int iters, double *ops, bcjr_stream_t stream) {
    if (!out || !ops) return BCJR_ERR_NULL_POINTER;
    if (iters < 1) return BCJR_ERR_BAD_SHAPE;
    int dev = 0, sms = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return BCJR_ERR_DEVICE;
    if (major != 10) return BCJR_ERR_DEVICE;
    const int blocks = sms * kProbeBlocksPerSm;
    *ops = (double)blocks * kProbeThreads * (double)iters * kProbeChains;
    mufu_probe_kernel<<<blocks, kProbeThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(out, iters);
    return cudaGetLastError() == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH;
}
