// Host-side launch interface between the C ABI (kattn_api.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>

#include "kerr_attn.h"

namespace kattn {

// Launches `kernel` on `stream` with programmatic stream serialisation, so it
// may start while the previous kernel in the stream drains (the kernel calls
// pdl_enter() before it reads global memory).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

struct FwdArgs {
    const float* q;
    const float* k;
    const float* v;
    long ld_qkv;
    float* o;
    long ld_o;
    float* lse;
    int B, T, H, d;
    float scale;
    int causal;
    // Wall-time limit of every bounded wait in the tensor-core kernels.
    unsigned long long wait_ns = 1000000000ull;
    // Diagnostic (kattn_test_withhold_next_load): the tensor-core forward
    // issues no copy of its first key tile, so its waits on it run out.
    int withhold_first_key_load = 0;
};

struct BwdArgs {
    const float* q;
    const float* k;
    const float* v;
    long ld_qkv;
    const float* o;
    const float* dout;
    long ld_o;
    const float* lse;
    float* dq;
    float* dk;
    float* dv;
    long ld_d;
    float* dsum;  // [B][H][T] workspace: rowsum(dout * o)
    int B, T, H, d;
    float scale;
    int causal;
    unsigned long long wait_ns = 1000000000ull;  // wall-time limit of every bounded wait
    // Deterministic dQ: when set, each key tile's dQ contribution is stored
    // (not added) into its slice of [key tiles][B*T][H*d] and
    // launch_bwd_dq_reduce sums the slices in key-tile order into dq.
    float* dq_part = nullptr;
};

// Key rows per backward work item (the dQ partial slices of the
// deterministic mode): tensor-core kernel, FFMA kernel.
constexpr int kBwdTcKeyRows = 128;
constexpr int kBwdF32KeyRows = 64;

// dq[b*T + t][h*d + c] = sum over key tiles j (in order; for causal, only
// j*key_rows <= t) of part[j][b*T + t][h*d + c].
cudaError_t launch_bwd_dq_reduce(const BwdArgs& a, int key_rows, int num_sms, cudaStream_t stream, int* launches);

// Each returns the CUDA launch status and adds the number of kernels it
// enqueued to *launches.
cudaError_t launch_fwd(const FwdArgs& a, int num_sms, cudaStream_t stream, int* launches);
cudaError_t launch_bwd(const BwdArgs& a, int num_sms, cudaStream_t stream, int* launches);

// Tensor-core (tcgen05) kernels.  `status` is a device word the kernels set
// (bit 0) when a bounded wait on the tensor core gives up.
bool fwd_tc_supported(const FwdArgs& a);
cudaError_t launch_fwd_tc(const FwdArgs& a, int num_sms, int* status, cudaStream_t stream, int* launches);
bool bwd_tc_supported(const BwdArgs& a);
cudaError_t launch_bwd_tc(const BwdArgs& a, int num_sms, int* status, cudaStream_t stream, int* launches);

// D = rowsum(dout * o) into a.dsum and dq = 0 (first kernel of every backward).
cudaError_t launch_bwd_prep(const BwdArgs& a, int num_sms, cudaStream_t stream, int* launches);

// The outcome of a call of the projection, LayerNorm and Kerr-ODE launchers:
// a CUDA error with the step that failed, or success.
struct ProjStatus {
    cudaError_t cuda = cudaSuccess;
    const char* what = nullptr;
    bool ok() const { return cuda == cudaSuccess; }
};

// C (+)= A B^T on the tensor cores (kgemm.cu): C[m][n] = (accumulate ? C : 0)
// + bias[n] + sum_k A(m, k) B(n, k) for m < M, n < N, k < K, the products in
// bf16 hi / lo pairs split on chip.  A(m, k) = a[m*lda + k] (K-major) or
// a[k*lda + m] (a_mn); B(n, k) likewise with b_mn.  Row-major f32, 16-byte
// aligned, every ld and N a multiple of 4 floats.  Split-K workspace comes
// from `pool`; `status` is the device word set when a bounded wait runs out.
ProjStatus gemm_tc(cudaStream_t s, cudaMemPool_t pool, int num_sms, const float* a, long lda, bool a_mn,
                   const float* b, long ldb, bool b_mn, float* c, long ldc, const float* bias, int M, int N, int K,
                   int accumulate, int* status, unsigned long long wait_ns, int* launches);

// Projection layers (kproj.cu).  Arrays are row-major f32; w is [N][K]
// contiguous, dw [N][K] contiguous.  *launches counts the kernels enqueued.
ProjStatus proj_forward(int num_sms, cudaStream_t s, cudaMemPool_t pool, int* status, unsigned long long wait_ns,
                        const float* x, long ld_x, const float* w, const float* b, float* y, long ld_y, int M, int N,
                        int K, int* launches);
ProjStatus proj_backward_dx(int num_sms, cudaStream_t s, cudaMemPool_t pool, int* status, unsigned long long wait_ns,
                            const float* dy, long ld_dy, const float* w, float* dx, long ld_dx, int M, int N, int K,
                            int* launches);
ProjStatus proj_backward_dw(int num_sms, cudaStream_t s, cudaMemPool_t pool, int* status, unsigned long long wait_ns,
                            const float* dy, long ld_dy, const float* x, long ld_x, float* dw, float* db, int M, int N,
                            int K, int accumulate, int* launches);

// LayerNorm over rows of n floats (kln.cu), eps 1e-5.  n a multiple of 4,
// at most LN_MAX_N; rows 16-byte aligned.  w, b, dw, db have n floats.
// Backward: dx written; dw / db (either may be NULL) added to when
// `accumulate`, written otherwise.  *launches counts the kernels enqueued.
constexpr int LN_MAX_N = KATTN_LN_MAX_N;
bool ln_supported(int n);
ProjStatus ln_forward(cudaStream_t s, int num_sms, const float* x, long ld_x, const float* w, const float* b, float* y,
                      long ld_y, int M, int n, int* launches);
ProjStatus ln_backward(cudaStream_t s, cudaMemPool_t pool, const float* dy, long ld_dy, const float* x, long ld_x, const float* w,
                       float* dx, long ld_dx, float* dw, float* db, int M, int n, int accumulate, int* launches);

// Kerr-ODE over rows of 2 nb interleaved (r, s) floats (kode.cu).  nb a
// multiple of 4, at most KODE_MAX_BANDS; rows 16-byte aligned, strides
// multiples of 4 floats.  gamma_raw / omega: nb floats, alpha_beta: 2 floats,
// all device memory.  The backward's `part` holds part_rows rows of
// kode_part_width(nb) floats, part_rows from kode_backward_grid; its parameter
// gradients are added to when `accumulate`, written otherwise.
constexpr int KODE_MAX_THREADS = 256;
// A partial row: d_gamma [nb], d_omega [nb], d_alpha, d_beta, padded to a
// multiple of 4 floats so that every row starts on a 16-byte boundary (the
// per-band sums are stored as float4).
inline __host__ __device__ int kode_part_width(int nb) { return 2 * nb + 4; }
constexpr int KODE_MAX_BANDS = 4 * KODE_MAX_THREADS;
constexpr size_t KODE_MAX_SMEM = 227 * 1024;
bool kode_supported(int nb, int n_steps);
ProjStatus kode_forward(cudaStream_t s, int num_sms, const float* x, long ld_x, float* y, long ld_y,
                        const float* gamma_raw, const float* omega, const float* alpha_beta, int M, int nb,
                        int n_steps, int* launches);
cudaError_t kode_backward_grid(int num_sms, int M, int nb, int n_steps, int* grid);
// The two halves of kode_backward: the backward kernel over M rows writing
// part_rows partial rows at `part`, and the fixed-order sum of part_rows
// partial rows into the parameter gradients.
ProjStatus kode_backward_rows(cudaStream_t s, const float* dy, long ld_dy, const float* x, long ld_x,
                              const float* gamma_raw, const float* omega, const float* alpha_beta, float* dx,
                              long ld_dx, int M, int nb, int n_steps, float* part, int part_rows, int* launches);
ProjStatus kode_backward_final(cudaStream_t s, const float* part, int part_rows, int nb, const float* gamma_raw,
                               float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int accumulate,
                               int* launches);
ProjStatus kode_backward(cudaStream_t s, int num_sms, const float* dy, long ld_dy, const float* x, long ld_x,
                         const float* gamma_raw, const float* omega, const float* alpha_beta, float* dx, long ld_dx,
                         float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int M, int nb, int n_steps,
                         int accumulate, float* part, int part_rows, int* launches);

}  // namespace kattn
