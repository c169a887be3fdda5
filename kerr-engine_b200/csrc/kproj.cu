// The attention projections c_attn and c_proj as dense GEMMs (sm_100a):
// forward y = x W^T + b, and the backward dx = dy W, dW (+)= dy^T x,
// db (+)= colsum(dy).  Replaces CpuBackend::linear_batch (src/backend.rs:296-298,
// :508-520), linear_backward_dx_batch (src/backend.rs:316-318 ->
// src/backward.rs:48-60) and outer_product_accum (src/backend.rs:320-342) at
// the call sites src/pipeline.rs:289, :353, :695-737.
//
// Every product runs on this library's tcgen05 GEMM (kgemm.cu), which splits
// the f32 operands into bf16 hi / lo on chip and accumulates hi*hi + hi*lo +
// lo*hi in f32 (relative error ~1e-5).  Row-major f32 [rows][ld] arrays enter
// it as they are:
//   forward: y[m][n]  = sum_k x[m][k] w[n][k]      A = x (K-major), B = w (K-major)
//   dx     : dx[m][k] = sum_n dy[m][n] w[n][k]     A = dy (K-major), B(k, n) = w[n][k] (MN-major)
//   dW     : dW[n][k] = sum_m dy[m][n] x[m][k]     A(n, m) = dy[m][n], B(k, m) = x[m][k] (both MN-major)
// The bias of the forward is added in the GEMM's epilogue; db is a column sum
// in a fixed order (the kernels below), so the same inputs give the same bits.
#include "kattn_common.cuh"
#include "kattn_launch.h"

namespace kattn {

namespace {

// y[m][n] = b[n] (the GEMMs then accumulate onto it).
__global__ void __launch_bounds__(256) proj_fill_bias(float* __restrict__ y, long ld, int rows, int cols,
                                                      const float* __restrict__ b) {
    pdl_enter();
    const long n = static_cast<long>(rows) * cols;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / cols;
        const int c = static_cast<int>(i - r * cols);
        y[r * ld + c] = b[c];
    }
}

// part[p][n] = sum of dy[m][n] over rows [p*R, min(M, (p+1)*R)), rows in order.
__global__ void __launch_bounds__(256) proj_colsum_part(const float* __restrict__ dy, long ld, int M, int N, int R,
                                                        float* __restrict__ part) {
    pdl_enter();
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int p = blockIdx.y;
    if (n >= N) return;
    const int m0 = p * R;
    const int m1 = min(M, m0 + R);
    float s = 0.f;
    for (int m = m0; m < m1; ++m) s += dy[static_cast<long>(m) * ld + n];
    part[static_cast<long>(p) * N + n] = s;
}

// db[n] (+)= sum over p of part[p][n]: a CTA of 32 x 32 threads takes 32
// columns, thread (x, y) sums partials y, y + 32, ... of column x, then
// thread (x, 0) adds the 32 sums in order of y.  The order is fixed:
// deterministic.
constexpr int COLSUM_COLS = 32;
constexpr int COLSUM_GROUPS = 32;

__global__ void __launch_bounds__(COLSUM_COLS* COLSUM_GROUPS)
    proj_colsum_final(const float* __restrict__ part, int P, int N, float* __restrict__ db, int accumulate) {
    __shared__ float sums[COLSUM_GROUPS][COLSUM_COLS + 1];
    pdl_enter();
    const int x = threadIdx.x, y = threadIdx.y;
    const int n = blockIdx.x * COLSUM_COLS + x;
    float s = 0.f;
    if (n < N)
        for (int p = y; p < P; p += COLSUM_GROUPS) s += part[static_cast<long>(p) * N + n];
    sums[y][x] = s;
    __syncthreads();
    if (y != 0 || n >= N) return;
    float t = 0.f;
    for (int g = 0; g < COLSUM_GROUPS; ++g) t += sums[g][x];
    db[n] = accumulate ? db[n] + t : t;
}

unsigned grid_for(long items, int num_sms) {
    long g = (items + 255) / 256;
    const long cap = static_cast<long>(num_sms > 0 ? num_sms : 148) * 16;
    if (g > cap) g = cap;
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

}  // namespace

ProjStatus proj_forward(int num_sms, cudaStream_t s, cudaMemPool_t pool, int* status, unsigned long long wait_ns,
                        const float* x, long ld_x, const float* w, const float* b, float* y, long ld_y, int M, int N,
                        int K, int* launches) {
    if (M == 0 || N == 0) return {};
    if (K == 0) {
        cudaError_t e;
        if (!b) {
            e = cudaMemset2DAsync(y, ld_y * 4, 0, static_cast<size_t>(N) * 4, M, s);
            return e == cudaSuccess ? ProjStatus{} : ProjStatus{e, "cudaMemset2DAsync"};
        }
        e = launch_pdl(proj_fill_bias, dim3(grid_for(static_cast<long>(M) * N, num_sms)), dim3(256), 0, s, y, ld_y, M,
                       N, b);
        if (e != cudaSuccess) return {e, "bias fill"};
        ++*launches;
        return {};
    }
    return gemm_tc(s, pool, num_sms, x, ld_x, false, w, K, false, y, ld_y, b, M, N, K, 0, status, wait_ns, launches);
}

ProjStatus proj_backward_dx(int num_sms, cudaStream_t s, cudaMemPool_t pool, int* status, unsigned long long wait_ns,
                            const float* dy, long ld_dy, const float* w, float* dx, long ld_dx, int M, int N, int K,
                            int* launches) {
    if (M == 0 || K == 0) return {};
    if (N == 0) {
        const cudaError_t e = cudaMemset2DAsync(dx, ld_dx * 4, 0, static_cast<size_t>(K) * 4, M, s);
        return e == cudaSuccess ? ProjStatus{} : ProjStatus{e, "cudaMemset2DAsync"};
    }
    (void)num_sms;
    return gemm_tc(s, pool, num_sms, dy, ld_dy, false, w, K, true, dx, ld_dx, nullptr, M, K, N, 0, status, wait_ns,
                   launches);
}

ProjStatus proj_backward_dw(int num_sms, cudaStream_t s, cudaMemPool_t pool, int* status, unsigned long long wait_ns,
                            const float* dy, long ld_dy, const float* x, long ld_x, float* dw, float* db, int M, int N,
                            int K, int accumulate, int* launches) {
    if (N == 0) return {};
    cudaError_t e;
    if (db) {
        const int R = 64;  // rows per column-sum partial
        const int P = M > 0 ? (M + R - 1) / R : 0;
        float* part = nullptr;
        if (P > 0) {
            e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&part), sizeof(float) * static_cast<size_t>(P) * N,
                                        pool, s);
            if (e != cudaSuccess) return {e, "column-sum workspace"};
            e = launch_pdl(proj_colsum_part, dim3((N + 255) / 256, P), dim3(256), 0, s, dy, ld_dy, M, N, R, part);
            if (e == cudaSuccess) ++*launches;
        } else {
            e = cudaSuccess;
        }
        if (e == cudaSuccess) {
            e = launch_pdl(proj_colsum_final, dim3((N + COLSUM_COLS - 1) / COLSUM_COLS),
                           dim3(COLSUM_COLS, COLSUM_GROUPS), 0, s, static_cast<const float*>(part), P, N, db,
                           accumulate);
            if (e == cudaSuccess) ++*launches;
        }
        const cudaError_t ef = part ? cudaFreeAsync(part, s) : cudaSuccess;
        if (e == cudaSuccess) e = ef;
        if (e != cudaSuccess) return {e, "column sums"};
    }
    if (K == 0) return {};
    if (M == 0) {
        if (accumulate) return {};
        e = cudaMemsetAsync(dw, 0, static_cast<size_t>(N) * K * 4, s);
        return e == cudaSuccess ? ProjStatus{} : ProjStatus{e, "cudaMemsetAsync"};
    }
    return gemm_tc(s, pool, num_sms, dy, ld_dy, true, x, ld_x, true, dw, K, nullptr, N, K, M, accumulate, status,
                   wait_ns, launches);
}

}  // namespace kattn
