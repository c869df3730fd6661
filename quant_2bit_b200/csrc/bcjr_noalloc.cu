// Allocation-free forward entry point (declared in include/bcjr_b200.h).
//
// Some callers cannot hand this library a workspace: a host that binds the C
// ABI from another language and has no device allocator of its own, or a
// training/serving loop that must not call cudaMalloc between steps (it
// synchronises the whole device) and has no caching allocator to borrow
// from.  For them, bcjr_fb_forward_noalloc runs the generic forward kernel on
// a fixed scratch array that is part of this library's device image instead
// of a caller-provided workspace.
//
// The scratch is kNoAllocScratchBytes (64 MiB).  Every GPU that loads the
// library holds it until the process exits.  A call whose single sequence
// slot does not fit (for L=16, k=2, V=1 that is N > ~980) is rejected with
// BCJR_ERR_WORKSPACE before anything is launched; otherwise the batch runs on
// as many slots as fit.
//
// Host code must not use `g_scratch` itself: in host code that name is only a
// host-side stand-in, not a device address.  The first call on each device
// (with that device current) looks up the array's device address with
// cudaGetSymbolAddress and caches it; make that first call before any stream
// capture.  All calls share the one array, so calls whose work overlaps on
// the GPU (different streams, or different host threads) race on it and must
// be serialised by the caller.  Nothing in the array needs to start at zero:
// the kernel writes every element it reads before reading it.
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/bcjr_b200.h"
#include "bcjr_kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;

static __device__ __align__(256) unsigned char g_scratch[kNoAllocScratchBytes];

// Device address of g_scratch on `dev` (looked up once per device).
int scratch_address(int dev, void **out) {
    static std::mutex mu;
    static void *addr[64] = {};
    if (dev < 0 || dev >= 64) return BCJR_ERR_DEVICE;
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return BCJR_ERR_DEVICE;
        }
        addr[dev] = p;
    }
    *out = addr[dev];
    return BCJR_OK;
}

}  // namespace

extern "C" BCJR_API int bcjr_fb_forward_noalloc(const float *seq, const float *cb,
                                                const float *T_dev, int B, int N, int L, int k,
                                                int V, float *soft, float *logZ,
                                                bcjr_stream_t stream) {
    const int st = bcjr_check_shape(B, N, L, k, V);
    if (st) return st;
    if (B == 0) return BCJR_OK;
    if (!seq || !cb || !T_dev || !soft) return BCJR_ERR_NULL_POINTER;
    const uintptr_t mis = reinterpret_cast<uintptr_t>(seq) | reinterpret_cast<uintptr_t>(cb) |
                          reinterpret_cast<uintptr_t>(T_dev) | reinterpret_cast<uintptr_t>(soft) |
                          reinterpret_cast<uintptr_t>(logZ);
    if (mis & 3u) return BCJR_ERR_ALIGNMENT;
    const int b = k * V;
    // One slot of the generic forward kernel must fit in the fixed scratch.
    const int slots = bcjr::generic_grid(B, N, L, b, bcjr::kModeForward, kNoAllocScratchBytes);
    if (slots < 1) return BCJR_ERR_WORKSPACE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return BCJR_ERR_DEVICE;
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10)
        return BCJR_ERR_DEVICE;
    void *scratch = nullptr;
    const int sa = scratch_address(dev, &scratch);
    if (sa) return sa;

    bcjr::LaunchArgs a;
    std::memset(&a, 0, sizeof(a));
    a.seq = seq; a.cb = cb; a.T_dev = T_dev;
    a.B = B; a.N = N; a.L = L; a.BB = b; a.V = V;
    a.soft = soft; a.logZ = logZ;
    a.ws_data = scratch;
    a.ws_data_bytes = kNoAllocScratchBytes;
    a.status = nullptr;
    a.claim = nullptr;
    a.mode = bcjr::kModeForward;
    a.kernel = bcjr::kKernelGeneric;
    a.grid = slots;
    a.stream = reinterpret_cast<cudaStream_t>(stream);
    return bcjr::launch_generic(a) == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH;
}
