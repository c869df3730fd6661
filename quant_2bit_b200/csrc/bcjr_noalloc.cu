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
// library holds it until the process exits.  One sequence slot of the
// generic forward takes (N + 3) 2^(L - kV) + 2N floats (+1 when odd); a call
// whose single slot does not fit (for L=16, k=2, V=1 that is N > 1020) is
// rejected with BCJR_ERR_WORKSPACE before anything is launched; otherwise
// the batch runs on as many slots as fit, a block taking the next sequence
// when it finishes one.
//
// Host code must not use `g_scratch` itself: in host code that name is only a
// host-side stand-in, not a device address.  The first call on each device
// (with that device current) looks up the array's device address with
// cudaGetSymbolAddress and caches it together with the identity of the
// device's current context; a call that finds another context (the device
// was reset and its context re-created, which reloads the module) looks the
// address up again.  Make the first call before any stream capture.  All
// calls share the one array, so calls whose work overlaps on the GPU
// (different streams, or different host threads) race on it and must be
// serialised by the caller.  The array keeps the last call's contents;
// nothing in it needs to start at zero: the kernel writes every element it
// reads before reading it.
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/bcjr_b200.h"
#include "bcjr_kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;

static __device__ __align__(256) unsigned char g_scratch[kNoAllocScratchBytes];

// Unique id of the calling thread's current CUDA context (cuCtxGetId), 0
// when there is none or it cannot be had.  The driver functions come through
// the runtime's entry-point query, so the library needs no link against the
// driver library.
unsigned long long current_context_id() {
    using GetCurrent = int (*)(void **);
    using GetId = int (*)(void *, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        p = nullptr;
        q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
        cudaGetLastError();
    });
    if (!get_current || !get_id) return 0;
    void *ctx = nullptr;
    if (get_current(&ctx) != 0 || !ctx) return 0;
    unsigned long long id = 0;
    return get_id(ctx, &id) == 0 ? id : 0;
}

// Device address of g_scratch on `dev` (the current device): looked up once
// per device and context.  Without a context id (none current yet, or the
// query unavailable) it is looked up on every call.
int scratch_address(int dev, void **out) {
    static std::mutex mu;
    static void *addr[64] = {};
    static unsigned long long ctx_of[64] = {};
    if (dev < 0 || dev >= 64) return BCJR_ERR_DEVICE;
    std::lock_guard<std::mutex> lk(mu);
    const unsigned long long ctx = current_context_id();
    if (!addr[dev] || ctx == 0 || ctx != ctx_of[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            addr[dev] = nullptr;
            return BCJR_ERR_DEVICE;
        }
        addr[dev] = p;
        ctx_of[dev] = current_context_id();   // the lookup made the context current
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
