// Internal launch interface between the C ABI (bcjr_capi.cu) and the kernels.
#pragma once

#include <cstddef>
#include <cuda_runtime.h>

namespace bcjr {

enum { kModeForward = 0, kModeBackward = 1, kModeInternals = 2 };

// Test and diagnostic switches, set through bcjr_set_test_option() (C ABI);
// all zero unless a test sets them (nothing reads the environment).
enum {
    kOptDropSends = 1,       // BCJR_OPT_TEST_DROP_SENDS
    kOptForceGeneric = 2,    // BCJR_OPT_FORCE_GENERIC
    kOptL16Forward = 3,      // BCJR_OPT_L16_FORWARD_CLUSTER
    kOptL16Backward = 4,     // BCJR_OPT_L16_BACKWARD_CLUSTER
    kOptCount = 5
};
int test_option(int which);   // bcjr_capi.cu
// SMs the cluster kernels leave free for concurrent kernels (collectives),
// set through bcjr_set_reserved_sms() (C ABI); 0 by default.
int reserved_sms();           // bcjr_capi.cu
enum { kKernelGeneric = 0, kKernelL16 = 1, kKernelB4 = 2 };

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
    unsigned *claim;              // device sequence counter in the header (zeroed per call)
    int mode;
    int grid;
    int kernel;                   // kKernelGeneric / kKernelL16 / kKernelB4
    int drop_sends;               // test-only fault injection (cluster kernels)
    cudaStream_t stream;
};

// Generic path (bcjr_generic.cu).
size_t generic_workspace_bytes(int B, int N, int L, int BB, int V, int mode, int num_sms);
int generic_grid(int B, int N, int L, int BB, int mode, size_t ws_data_bytes);
cudaError_t launch_generic(const LaunchArgs &a);

// Cluster path for L=16, k=2, V=1, 2 <= N <= 512 (bcjr_l16.cu): the 2-CTA
// (l16) and 4-CTA (l16c4, bcjr_l16_cl4.cu) instances of one kernel, and the
// dispatcher that runs one or both.
namespace l16 {
int max_clusters(int mode);
int slots(int mode);
size_t slot_bytes(int N, int mode);
cudaError_t launch(const LaunchArgs &a, int ncl, float *ws, bool dependent);
}  // namespace l16
namespace l16c4 {
int max_clusters(int mode);
int slots(int mode);
size_t slot_bytes(int N, int mode);
cudaError_t launch(const LaunchArgs &a, int ncl, float *ws, bool dependent);
}  // namespace l16c4
bool l16_applicable(int B, int N, int L, int BB, int V);
int l16_clusters(int B, int mode);
int l16_launches(int B, int mode);
size_t l16_workspace_bytes(int B, int N, int mode);
cudaError_t launch_l16(const LaunchArgs &a);

// Cluster path for L=16, k=2, V=2 (b = 4), 2 <= N <= 512 (bcjr_b4.cu).
bool b4_applicable(int B, int N, int L, int BB, int V);
int b4_clusters(int B, int mode);
size_t b4_workspace_bytes(int B, int N, int mode);
cudaError_t launch_b4(const LaunchArgs &a);

// Cluster Viterbi for L=16, k=2, V=2, 1 <= N <= 512 (bcjr_vit_b4.cu).
bool vit_b4_applicable(int N, int L, int k, int V, const void *cb);
size_t vit_b4_workspace_bytes(int B, int N);
int vit_b4_launches(int B);
cudaError_t launch_vit_b4(const float *seq, const float *cb, int B, int N, int *bits,
                          int *starts, float *recon, float *mse, void *ws, size_t ws_bytes,
                          int *status, int drop_sends, cudaStream_t st);

// Cluster Viterbi for L=16, k=2, V=1, 1 <= N <= 512 (bcjr_vit_b2.cu).
bool vit_b2_applicable(int N, int L, int k, int V, const void *cb);
size_t vit_b2_workspace_bytes(int B, int N);
int vit_b2_launches(int B, int N);
cudaError_t launch_vit_b2(const float *seq, const float *cb, int B, int N, int *bits,
                          int *starts, float *recon, float *mse, void *ws, size_t ws_bytes,
                          int *status, int drop_sends, cudaStream_t st);

}  // namespace bcjr
