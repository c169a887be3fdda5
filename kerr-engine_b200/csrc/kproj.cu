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
//   dW     : dW[n][k] = sum_m dy[m][n] x[m][k]     A(n, m) = dy[m][n] through a transposed copy dyT
//                                                   (K-major; MN-major dy when M % 4 != 0), B(k, m) = x[m][k]
//                                                   (MN-major)
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

// dyT[n][m] = dy[m][n] (dyT row stride M) and part[p][n] = sum of dy[m][n]
// over rows [32p, min(M, 32p + 32)) in row order, one 32 x 32 tile per
// block: the dW product then reads dy^T K-major (whole-row loads), and db
// comes from the same pass over dy.
__global__ void __launch_bounds__(256) proj_transpose_colsum(const float* __restrict__ dy, long ld, int M, int N,
                                                             float* __restrict__ dyT, float* __restrict__ part) {
    pdl_enter();
    __shared__ float tile[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = r0 + ty + 8 * i, c = c0 + tx;
        tile[ty + 8 * i][tx] = (r < M && c < N) ? dy[static_cast<long>(r) * ld + c] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = c0 + ty + 8 * i, r = r0 + tx;
        if (c < N && r < M) dyT[static_cast<long>(c) * M + r] = tile[tx][ty + 8 * i];
    }
    if (part && ty == 0 && c0 + tx < N) {
        float acc = 0.f;
        for (int r = 0; r < 32; ++r) acc += tile[r][tx];  // rows past M are zero
        part[static_cast<long>(blockIdx.y) * N + c0 + tx] = acc;
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
    cudaError_t e = cudaSuccess;
    // With M a multiple of 4, dy is transposed once (dyT [N][M]) so that the
    // GEMM reads its A operand K-major, and the same pass leaves db's 32-row
    // partial sums; otherwise the GEMM reads dy MN-major and db has its own
    // pass.
    const bool transpose = M > 0 && K > 0 && M % 4 == 0;
    float* dyT = nullptr;
    float* part = nullptr;
    auto release = [&]() {
        cudaError_t ef = cudaSuccess;
        if (dyT) ef = cudaFreeAsync(dyT, s);
        if (part) {
            const cudaError_t e2 = cudaFreeAsync(part, s);
            if (ef == cudaSuccess) ef = e2;
        }
        dyT = part = nullptr;
        return ef;
    };
    if (db || transpose) {
        const int R = transpose ? 32 : 64;  // rows per column-sum partial
        const int P = M > 0 ? (M + R - 1) / R : 0;
        if (db && P > 0)
            e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&part), sizeof(float) * static_cast<size_t>(P) * N, pool,
                                        s);
        if (e == cudaSuccess && transpose)
            e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&dyT), sizeof(float) * static_cast<size_t>(N) * M, pool,
                                        s);
        if (e != cudaSuccess) {
            release();
            return {e, "dW workspace"};
        }
        if (transpose) {
            e = launch_pdl(proj_transpose_colsum, dim3((N + 31) / 32, (M + 31) / 32), dim3(32, 8), 0, s, dy, ld_dy, M, N,
                           dyT, part);
        } else if (part) {
            e = launch_pdl(proj_colsum_part, dim3((N + 255) / 256, P), dim3(256), 0, s, dy, ld_dy, M, N, R, part);
        }
        if (e == cudaSuccess && (transpose || part)) ++*launches;
        if (e == cudaSuccess && db) {
            e = launch_pdl(proj_colsum_final, dim3((N + COLSUM_COLS - 1) / COLSUM_COLS),
                           dim3(COLSUM_COLS, COLSUM_GROUPS), 0, s, static_cast<const float*>(part), P, N, db,
                           accumulate);
            if (e == cudaSuccess) ++*launches;
        }
        if (e != cudaSuccess) {
            release();
            return {e, "dW prologue"};
        }
    }
    ProjStatus st;
    if (K > 0) {
        if (M == 0) {
            if (!accumulate) {
                e = cudaMemsetAsync(dw, 0, static_cast<size_t>(N) * K * 4, s);
                if (e != cudaSuccess) st = {e, "cudaMemsetAsync"};
            }
        } else if (transpose) {
            st = gemm_tc(s, pool, num_sms, dyT, M, false, x, ld_x, true, dw, K, nullptr, N, K, M, accumulate, status,
                         wait_ns, launches);
        } else {
            st = gemm_tc(s, pool, num_sms, dy, ld_dy, true, x, ld_x, true, dw, K, nullptr, N, K, M, accumulate, status,
                         wait_ns, launches);
        }
    }
    const cudaError_t ef = release();
    if (st.cuda == cudaSuccess && ef != cudaSuccess) st = {ef, "dW workspace release"};
    return st;
}

}  // namespace kattn
