// HYB codebook expansion: the (2^L, 2) per-state codebook of the QTIP "HYB"
// code from its (2^Q, 2) lookup table, as one kernel.  Replaces
// make_hyb_codebook_gpu (src/qat/ste.py:376-392) and decode_hyb_batch
// (src/codes/ref.py:116-128):
//
//   x(s)     = (s * s + s) mod 2^32
//   row(s)   = (x >> (15 - Q)) mod 2^Q
//   cb[s]    = (lut[row][0], lut[row][1] * (bit 15 of x ? -1 : 1))
//
// Unsigned 32-bit arithmetic gives x mod 2^32 for every L <= 24 exactly as
// the reference's int64 product masked to 32 bits.  The kernel writes 8 bytes
// per state (HBM-bound, 0.5 MB at L=16) and reads the LUT through L1.
#include <cstdint>

#include "../../include/bcjr_b200.h"

namespace bcjr {
namespace codes {

__global__ void __launch_bounds__(256) hyb_expand(const float2 *__restrict__ lut, int Q, int L,
                                                  float2 *__restrict__ cb) {
    const uint32_t n = 1u << L;
    const uint32_t qmask = (1u << Q) - 1u;
    for (uint32_t s = blockIdx.x * blockDim.x + threadIdx.x; s < n; s += gridDim.x * blockDim.x) {
        const uint32_t x = s * s + s;
        const float2 v = __ldg(lut + ((x >> (15 - Q)) & qmask));
        cb[s] = make_float2(v.x, ((x >> 15) & 1u) ? -v.y : v.y);
    }
}

}  // namespace codes
}  // namespace bcjr

extern "C" {

BCJR_API int bcjr_hyb_codebook(const float *lut, int Q, int L, float *cb_out, bcjr_stream_t stream) {
    if (Q < 1 || Q > 15 || L < 1 || L > 24) return BCJR_ERR_BAD_SHAPE;
    if (!lut || !cb_out) return BCJR_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(lut) | reinterpret_cast<uintptr_t>(cb_out)) & 7u)
        return BCJR_ERR_ALIGNMENT;
    int dev = 0, major = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        major != 10)
        return BCJR_ERR_DEVICE;
    const long n = 1L << L;
    long blocks = (n + 255) / 256;
    if (blocks > 8L * sms) blocks = 8L * sms;
    bcjr::codes::hyb_expand<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float2 *>(lut), Q, L, reinterpret_cast<float2 *>(cb_out));
    return cudaGetLastError() == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH;
}

}  // extern "C"
