// Internal launch interface between the C ABI (bcjr_capi.cu) and the kernels.
#pragma once

#include <cstddef>
#include <cuda_runtime.h>

namespace bcjr {

enum { kModeForward = 0, kModeBackward = 1, kModeInternals = 2 };

struct LaunchArgs {
    const float *seq, *cb, *T_dev;
    const float *soft_in, *grad;  // backward inputs
    int B, N, L, BB, V;
    float *soft, *logZ;           // forward outputs
    float *dseq;                  // backward output
    float *P, *LA, *LB;           // internals outputs
    void *ws_data;                // workspace after the header
    size_t ws_data_bytes;
    int *status;                  // device status word in the workspace header
    int mode;
    int grid;
    bool fast;                    // cluster kernel (bcjr_l16.cu)
    int drop_sends;               // test-only fault injection (cluster kernel)
    cudaStream_t stream;
};

// Generic path (bcjr_generic.cu).
size_t generic_workspace_bytes(int B, int N, int L, int BB, int V, int mode, int num_sms);
int generic_grid(int B, int N, int L, int BB, int mode, size_t ws_data_bytes);
cudaError_t launch_generic(const LaunchArgs &a);

// Cluster path for L=16, k=2, V=1, 2 <= N <= 512 (bcjr_l16.cu).
bool l16_applicable(int B, int N, int L, int BB, int V);
int l16_clusters(int B, int mode);
size_t l16_workspace_bytes(int B, int N, int mode);
cudaError_t launch_l16(const LaunchArgs &a);

}  // namespace bcjr
