// C ABI of libbcjr_b200 (declared in include/bcjr_b200.h).
//
// Validates shapes and pointers, sizes the persistent grid from the caller's
// workspace, and launches the kernels on the caller's stream.  No host
// synchronisation, no allocation, T is read on the device.
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/bcjr_b200.h"
#include "bcjr_kernels.h"

namespace bcjr {

namespace {
std::atomic<int> g_test_options[kOptCount];
std::atomic<int> g_reserved_sms{0};
}  // namespace

int test_option(int which) {
    return (which > 0 && which < kOptCount) ? g_test_options[which].load(std::memory_order_relaxed) : 0;
}

int reserved_sms() { return g_reserved_sms.load(std::memory_order_relaxed); }

}  // namespace bcjr

namespace {

constexpr size_t kHeaderBytes = 256;  // status word, sequence counter, padding (keeps data 256-B aligned)

struct DevInfo {
    int sms = 0;
    int major = 0;
    bool ok = false;
};

int query_device(DevInfo &d) {
    static std::mutex mu;
    static DevInfo cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BCJR_ERR_DEVICE;
    std::lock_guard<std::mutex> lk(mu);
    if (!cache[dev].ok) {
        int sms = 0, major = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
            return BCJR_ERR_DEVICE;
        cache[dev].sms = sms;
        cache[dev].major = major;
        cache[dev].ok = true;
    }
    d = cache[dev];
    if (d.major != 10) return BCJR_ERR_DEVICE;  // built for sm_100a only
    return BCJR_OK;
}

bool built_combo(int b, int V) {
    switch (b * 10 + V) {
        case 11: case 21: case 31: case 41: case 22: case 42: return true;
        default: return false;
    }
}

int check_shape(int B, int N, int L, int k, int V) {
    if (B < 0 || N < 1 || N > (1 << 20) || L < 1 || k < 1 || V < 1) return BCJR_ERR_BAD_SHAPE;
    if (V > 2 || k > 4) return BCJR_ERR_UNSUPPORTED;
    const int b = k * V;
    if (b > 4 || !built_combo(b, V)) return BCJR_ERR_UNSUPPORTED;
    if (L < b || L > 16) return BCJR_ERR_UNSUPPORTED;
    if ((long long)B * N * V > (1LL << 40)) return BCJR_ERR_BAD_SHAPE;
    return BCJR_OK;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Kernel choice.  The cluster kernels serve L=16, k=2 with V=1 (bcjr_l16.cu)
// and V=2 (bcjr_b4.cu), forward and backward, for 2 <= N <= 512; they read
// the codebook with 16-byte vector loads, so a codebook pointer that is not
// 16-byte aligned (a view at an odd offset) takes the generic kernels, as do
// every other shape, the internals, and the BCJR_OPT_FORCE_GENERIC option.
int pick_kernel(int B, int N, int L, int b, int V, int mode, const void *cb) {
    if (mode == bcjr::kModeInternals) return bcjr::kKernelGeneric;
    if (bcjr::test_option(bcjr::kOptForceGeneric)) return bcjr::kKernelGeneric;
    if (cb && !aligned(cb, 16)) return bcjr::kKernelGeneric;
    if (bcjr::l16_applicable(B, N, L, b, V) && bcjr::l16_clusters(B, mode) > 0)
        return bcjr::kKernelL16;
    if (bcjr::b4_applicable(B, N, L, b, V) && bcjr::b4_clusters(B, mode) > 0)
        return bcjr::kKernelB4;
    return bcjr::kKernelGeneric;
}

size_t kernel_bytes(int kernel, int B, int N, int L, int b, int V, int mode, int sms) {
    switch (kernel) {
        case bcjr::kKernelL16: return bcjr::l16_workspace_bytes(B, N, mode);
        case bcjr::kKernelB4: return bcjr::b4_workspace_bytes(B, N, mode);
        default: return bcjr::generic_workspace_bytes(B, N, L, b, V, mode, sms);
    }
}

// Workspace that bcjr_workspace_bytes reports: what the kernel chosen for an
// aligned codebook needs, and at least one sequence slot of the generic
// kernels (all they need), so that the same workspace serves a call whose
// codebook pointer sends it to the generic kernels.
size_t data_bytes(int B, int N, int L, int b, int V, int mode, int sms) {
    const size_t k = kernel_bytes(pick_kernel(B, N, L, b, V, mode, nullptr), B, N, L, b, V, mode, sms);
    const size_t g1 = bcjr::generic_workspace_bytes(1, N, L, b, V, mode, sms);
    return k > g1 ? k : g1;
}

int prepare(bcjr::LaunchArgs &a, void *ws, size_t ws_bytes, int mode) {
    DevInfo d;
    int st = query_device(d);
    if (st) return st;
    if (!ws) return BCJR_ERR_WORKSPACE;
    if (!aligned(ws, 256)) return BCJR_ERR_ALIGNMENT;
    a.kernel = pick_kernel(a.B, a.N, a.L, a.BB, a.V, mode, a.cb);
    // The cluster kernels need their full workspace; the generic kernels run
    // as many sequence slots as the workspace holds (at least one).
    const size_t need = a.kernel == bcjr::kKernelGeneric
                            ? 0
                            : kernel_bytes(a.kernel, a.B, a.N, a.L, a.BB, a.V, mode, d.sms);
    if (ws_bytes < kHeaderBytes + need) return BCJR_ERR_WORKSPACE;
    a.status = reinterpret_cast<int *>(ws);
    a.claim = reinterpret_cast<unsigned *>(static_cast<char *>(ws) + sizeof(int));
    a.ws_data = static_cast<char *>(ws) + kHeaderBytes;
    a.ws_data_bytes = ws_bytes - kHeaderBytes;
    a.mode = mode;
    // Test-only (BCJR_OPT_TEST_DROP_SENDS): the cluster kernel's CTA 1
    // withholds its outputs so that the bounded waits time out.
    a.drop_sends = bcjr::test_option(bcjr::kOptDropSends) ? 1 : 0;
    a.grid = a.kernel != bcjr::kKernelGeneric ? 1 : bcjr::generic_grid(a.B, a.N, a.L, a.BB, mode, a.ws_data_bytes);
    if (a.grid < 1) return BCJR_ERR_WORKSPACE;
    if (cudaMemsetAsync(a.status, 0, sizeof(int) + sizeof(unsigned), a.stream) != cudaSuccess)
        return BCJR_ERR_LAUNCH;
    return BCJR_OK;
}

int finish(cudaError_t e) {
    return e == cudaSuccess ? BCJR_OK : BCJR_ERR_LAUNCH;
}

cudaError_t launch(const bcjr::LaunchArgs &a) {
    switch (a.kernel) {
        case bcjr::kKernelL16: return bcjr::launch_l16(a);
        case bcjr::kKernelB4: return bcjr::launch_b4(a);
        default: return bcjr::launch_generic(a);
    }
}

}  // namespace

extern "C" {

int bcjr_version(void) { return 200; }

int bcjr_set_test_option(int option, int value) {
    if (option <= 0 || option >= bcjr::kOptCount) return -1;
    return bcjr::g_test_options[option].exchange(value);
}

int bcjr_set_reserved_sms(int sms) {
    if (sms < 0 || sms > 64) return -1;
    return bcjr::g_reserved_sms.exchange(sms);
}

const char *bcjr_status_string(int status) {
    switch (status) {
        case BCJR_OK: return "ok";
        case BCJR_ERR_BAD_SHAPE: return "bad shape (B, N, L, k, V inconsistent or out of range)";
        case BCJR_ERR_UNSUPPORTED: return "unsupported trellis (need 1 <= kV <= 4, V <= 2, kV <= L <= 16)";
        case BCJR_ERR_NULL_POINTER: return "a required pointer is NULL";
        case BCJR_ERR_ALIGNMENT: return "pointer misaligned";
        case BCJR_ERR_WORKSPACE: return "workspace missing or too small";
        case BCJR_ERR_LAUNCH: return "CUDA launch failed";
        case BCJR_ERR_DEVICE: return "no usable sm_100 device";
        case BCJR_ERR_TIMEOUT: return "a bounded device-side wait gave up";
        default: return "unknown status";
    }
}

int bcjr_check_shape(int B, int N, int L, int k, int V) { return check_shape(B, N, L, k, V); }

int bcjr_kernel_launches(int B, int N, int L, int k, int V, int flags) {
    if (check_shape(B, N, L, k, V) || B == 0) return 0;
    DevInfo d;
    if (query_device(d)) return 0;
    const int mode = flags == BCJR_WS_FORWARD    ? bcjr::kModeForward
                     : flags == BCJR_WS_BACKWARD ? bcjr::kModeBackward
                     : flags == BCJR_WS_INTERNALS ? bcjr::kModeInternals
                                                  : -1;
    if (mode < 0) return 0;
    const int b = k * V;
    if (pick_kernel(B, N, L, b, V, mode, nullptr) == bcjr::kKernelL16) return bcjr::l16_launches(B, mode);
    return 1;
}

size_t bcjr_workspace_bytes(int B, int N, int L, int k, int V, int flags) {
    if (check_shape(B, N, L, k, V)) return 0;
    DevInfo d;
    if (query_device(d)) return 0;
    const int b = k * V;
    size_t need = 0;
    if (flags & BCJR_WS_FORWARD) {
        size_t x = data_bytes(B, N, L, b, V, bcjr::kModeForward, d.sms);
        if (x > need) need = x;
    }
    if (flags & BCJR_WS_BACKWARD) {
        size_t x = data_bytes(B, N, L, b, V, bcjr::kModeBackward, d.sms);
        if (x > need) need = x;
    }
    if (flags & BCJR_WS_INTERNALS) {
        size_t x = data_bytes(B, N, L, b, V, bcjr::kModeInternals, d.sms);
        if (x > need) need = x;
    }
    return kHeaderBytes + need;
}

int bcjr_fb_forward(const float *seq, const float *cb, const float *T_dev,
                    int B, int N, int L, int k, int V,
                    float *soft, float *logZ,
                    void *ws, size_t ws_bytes, bcjr_stream_t stream) {
    int st = check_shape(B, N, L, k, V);
    if (st) return st;
    if (B == 0) return BCJR_OK;
    if (!seq || !cb || !T_dev || !soft) return BCJR_ERR_NULL_POINTER;
    if (!aligned(seq, 4) || !aligned(cb, 4) || !aligned(T_dev, 4) || !aligned(soft, 4) ||
        (logZ && !aligned(logZ, 4)))
        return BCJR_ERR_ALIGNMENT;
    bcjr::LaunchArgs a;
    std::memset(&a, 0, sizeof(a));
    a.seq = seq; a.cb = cb; a.T_dev = T_dev;
    a.B = B; a.N = N; a.L = L; a.BB = k * V; a.V = V;
    a.soft = soft; a.logZ = logZ;
    a.stream = reinterpret_cast<cudaStream_t>(stream);
    st = prepare(a, ws, ws_bytes, bcjr::kModeForward);
    if (st) return st;
    return finish(launch(a));
}

int bcjr_fb_backward(const float *seq, const float *cb, const float *T_dev,
                     const float *soft, const float *grad_soft,
                     int B, int N, int L, int k, int V,
                     float *d_seq,
                     void *ws, size_t ws_bytes, bcjr_stream_t stream) {
    int st = check_shape(B, N, L, k, V);
    if (st) return st;
    if (B == 0) return BCJR_OK;
    if (!seq || !cb || !T_dev || !soft || !grad_soft || !d_seq) return BCJR_ERR_NULL_POINTER;
    if (!aligned(seq, 4) || !aligned(cb, 4) || !aligned(T_dev, 4) || !aligned(soft, 4) ||
        !aligned(grad_soft, 4) || !aligned(d_seq, 4))
        return BCJR_ERR_ALIGNMENT;
    bcjr::LaunchArgs a;
    std::memset(&a, 0, sizeof(a));
    a.seq = seq; a.cb = cb; a.T_dev = T_dev;
    a.soft_in = soft; a.grad = grad_soft;
    a.B = B; a.N = N; a.L = L; a.BB = k * V; a.V = V;
    a.dseq = d_seq;
    a.stream = reinterpret_cast<cudaStream_t>(stream);
    st = prepare(a, ws, ws_bytes, bcjr::kModeBackward);
    if (st) return st;
    return finish(launch(a));
}

int bcjr_fb_internals(const float *seq, const float *cb, const float *T_dev,
                      int B, int N, int L, int k, int V,
                      float *P, float *log_alpha, float *log_beta,
                      void *ws, size_t ws_bytes, bcjr_stream_t stream) {
    int st = check_shape(B, N, L, k, V);
    if (st) return st;
    if (B == 0) return BCJR_OK;
    if (!seq || !cb || !T_dev) return BCJR_ERR_NULL_POINTER;
    bcjr::LaunchArgs a;
    std::memset(&a, 0, sizeof(a));
    a.seq = seq; a.cb = cb; a.T_dev = T_dev;
    a.B = B; a.N = N; a.L = L; a.BB = k * V; a.V = V;
    a.P = P; a.LA = log_alpha; a.LB = log_beta;
    a.stream = reinterpret_cast<cudaStream_t>(stream);
    st = prepare(a, ws, ws_bytes, bcjr::kModeInternals);
    if (st) return st;
    return finish(launch(a));
}

int bcjr_ws_status(const void *ws, bcjr_stream_t stream) {
    if (!ws) return BCJR_ERR_WORKSPACE;
    int h = 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&h, ws, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return BCJR_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return BCJR_ERR_LAUNCH;
    return h;
}

}  // extern "C"
