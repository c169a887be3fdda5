// Declarations shared by the translation units of the C ABI (kattn_api.cu,
// kblock.cu): the context, the last-error / launch-count reporting and the
// device scope of one call.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "kerr_attn.h"

constexpr unsigned long long kDefaultWaitNs = 1000000000ull;  // one second

struct kattn_ctx {
    int device = 0;
    int num_sms = 0;
    std::atomic<int> path{KATTN_PATH_AUTO};
    int* d_status = nullptr;        // device word set by kernels whose bounded waits give up
    cudaStream_t stream = nullptr;  // host-buffer entry points: kernels
    cudaStream_t h2d = nullptr;     // host-buffer entry points: host-to-device copies
    cudaStream_t d2h = nullptr;     // host-buffer entry points: device-to-host copies
    std::vector<cudaEvent_t> events;  // chunk hand-offs between those three streams
    std::mutex host_mu;             // serialises the host-buffer entry points
    char* arena = nullptr;          // device staging for the host-buffer entry points
    size_t arena_bytes = 0;
    float* noalloc_ws = nullptr;    // device address of g_noalloc_ws on this device
    cudaMemPool_t pool = nullptr;   // the context's own stream-ordered pool for per-call workspace
    std::atomic<unsigned long long> wait_ns{kDefaultWaitNs};  // limit of the kernels' bounded waits
    std::atomic<int> withhold_next_load{0};  // diagnostic hook (kattn_test_withhold_next_load)
    std::atomic<int> deterministic{0};       // dQ by ordered slices (kattn_set_deterministic)
};

namespace kattn_abi {

// Records a formatted message for kattn_last_error and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// KATTN_ERR_CUDA (KATTN_ERR_OUT_OF_MEMORY for an allocation failure) with
// the CUDA error's name and text.
int cuda_fail(cudaError_t e, const char* what);
// Records the number of kernels the call enqueued (kattn_last_launch_count)
// and returns KATTN_OK.
int ok_with_launches(int n);

// Makes ctx->device current for the scope of one call and restores the
// caller's device afterwards.
struct DeviceScope {
    int prev = -1;
    int dev;
    cudaError_t err = cudaSuccess;
    explicit DeviceScope(int d) : dev(d) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceScope() {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;
};

}  // namespace kattn_abi
