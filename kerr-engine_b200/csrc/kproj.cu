// The attention projections c_attn and c_proj as dense GEMMs (sm_100a):
// forward y = x W^T + b, and the backward dx = dy W, dW (+)= dy^T x,
// db (+)= colsum(dy).  Replaces CpuBackend::linear_batch (src/backend.rs:296-298,
// :508-520), linear_backward_dx_batch (src/backend.rs:316-318 ->
// src/backward.rs:48-60) and outer_product_accum (src/backend.rs:320-342) at
// the call sites src/pipeline.rs:289, :353, :695-737.
//
// Numerics: each f32 operand is split by the kernels below into bf16 hi and
// lo = bf16(x - hi) (the same split as the attention kernels), and every
// product is formed as hi*hi + hi*lo + lo*hi with f32 accumulation: relative
// error ~1e-5, where a single bf16 or tf32 GEMM would give ~1e-3.  The three
// products run as ONE cuBLAS bf16 GEMM over a contraction three times as long:
// the split writes each operand three times along its contraction dimension,
// e.g. x' = [x_hi | x_hi | x_lo] against w' = [w_hi | w_lo | w_hi], so the f32
// output is written once instead of read and rewritten by three GEMMs.  These
// are plain GEMMs, so the library runs them; the split, bias and column-sum
// kernels are this library's.
//
// Row-major f32 [rows][ld] arrays map onto cuBLAS's column-major view as
// their transposes:
//   forward: y^T (N x M)  = W (T of the K x N view of w) * x^T (K x M)
//   dx     : dx^T (K x M) = w^T (K x N view of w)        * dy^T (N x M)
//   dW     : dW^T (K x N) = x^T (K x M)                 * dy (T of the N x M view)
#include <cublas_v2.h>
#include <cuda_bf16.h>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"

namespace kattn {

namespace {

// src [rows][ld] f32 -> three bf16 copies of it (each either hi or lo:
// segment g is lo when bit g of `lo_mask` is set), concatenated along the
// columns (dst [rows][pitch], pitch >= 3*cols) or along the rows
// (dst [3*rows][cols]).  cols % 4 == 0, ld % 4 == 0.  Along the columns, the
// pitch - 3*cols extra bf16 of each row (a multiple of 4) are written too:
// zeros, except the first two, which are (1, 1) for EXTRA_ONES and
// (bf16(b[r]), bf16(b[r] - bf16(b[r]))) for EXTRA_BIAS.  Contracting an
// operand that ends in ones against one that ends in the bias pair adds
// b_hi + b_lo (= b to ~1e-5 relative) to every output: the bias rides in
// the GEMM instead of a separate fill and a read-modify-write of y.
constexpr int EXTRA_NONE = 0;
constexpr int EXTRA_ONES = 1;
constexpr int EXTRA_BIAS = 2;

__global__ void __launch_bounds__(256) proj_split3(const float* __restrict__ src, long ld, int rows, int cols,
                                                   uint2* __restrict__ dst, int along_rows, int lo_mask, int pitch4,
                                                   int extra, const float* __restrict__ bias) {
    pdl_enter();
    const int c4 = cols / 4;
    const long n = static_cast<long>(rows) * c4;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / c4;
        const int c = static_cast<int>(i - r * c4);
        const float4 v = *reinterpret_cast<const float4*>(src + r * ld + 4 * c);
        uint2 h, l;
        sm100::split2(v.x, v.y, h.x, l.x);
        sm100::split2(v.z, v.w, h.y, l.y);
#pragma unroll
        for (int g = 0; g < 3; ++g) {
            const long o = along_rows ? (static_cast<long>(g) * rows + r) * c4 + c : r * pitch4 + g * c4 + c;
            dst[o] = (lo_mask >> g) & 1 ? l : h;
        }
        if (!along_rows && c == 0 && pitch4 > 3 * c4) {
            uint2 e = make_uint2(0u, 0u);
            if (extra == EXTRA_ONES) {
                e.x = sm100::pack_bf16(1.f, 1.f);
            } else if (extra == EXTRA_BIAS) {
                uint32_t bh, bl;
                sm100::split2(bias[r], 0.f, bh, bl);
                e.x = (bh & 0xFFFFu) | (bl << 16);  // (b_hi, b_lo)
            }
            uint2* row = dst + r * pitch4 + 3 * c4;
            row[0] = e;
            for (int k = 1; k < pitch4 - 3 * c4; ++k) row[k] = make_uint2(0u, 0u);
        }
    }
}

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

// One operand as three bf16 copies along its contraction (see proj_split3):
// along the columns, rows of `pitch` bf16 (3*cols plus any extra columns).
struct Cat3 {
    uint2* p;
    int along_rows;
    int lo_mask;
    int pitch = 0;
    int extra = EXTRA_NONE;
    const float* bias = nullptr;
};

ProjStatus launch_split3(const float* src, long ld, int rows, int cols, Cat3 out, int num_sms, cudaStream_t s,
                         int* launches) {
    const long n = static_cast<long>(rows) * (cols / 4);
    if (n == 0) return {};
    const int pitch4 = (out.pitch > 0 ? out.pitch : 3 * cols) / 4;
    const cudaError_t e = launch_pdl(proj_split3, dim3(grid_for(n, num_sms)), dim3(256), 0, s, src, ld, rows, cols,
                                     out.p, out.along_rows, out.lo_mask, pitch4, out.extra, out.bias);
    if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "operand split"};
    ++*launches;
    return {};
}

// C (column-major m x n, ldc) = beta * C + A * B, bf16 operands, f32 accumulation.
ProjStatus gemm(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k, const void* a,
                int lda, const void* b, int ldb, float beta, float* c, long ldc, int* gemms) {
    const float one = 1.f;
    const cublasStatus_t st = cublasGemmEx(h, ta, tb, m, n, k, &one, a, CUDA_R_16BF, lda, b, CUDA_R_16BF, ldb, &beta,
                                           c, CUDA_R_32F, static_cast<int>(ldc), CUBLAS_COMPUTE_32F,
                                           CUBLAS_GEMM_DEFAULT);
    if (st != CUBLAS_STATUS_SUCCESS) return {cudaSuccess, st, "cublasGemmEx"};
    ++*gemms;
    return {};
}

// Stream-ordered workspace for the split copies of the operands.
struct Workspace {
    char* base = nullptr;
    cudaStream_t s = nullptr;
    ~Workspace() {
        if (base) cudaFreeAsync(base, s);
    }
};

// Bytes of a three-copy bf16 operand of `elems` f32 elements, rounded to 256.
long cat3_bytes(long elems) { return ((elems * 6 + 255) / 256) * 256; }

Cat3 carve(char*& p, long elems, int along_rows, int lo_mask) {
    Cat3 c{reinterpret_cast<uint2*>(p), along_rows, lo_mask};
    p += cat3_bytes(elems);
    return c;
}

// Contraction length of the forward with a bias: 3K plus the two bias
// columns, rounded up to a multiple of 8 bf16 (16-byte rows for the GEMM).
int biased_pitch(int K) { return (3 * K + 2 + 7) / 8 * 8; }

// A [rows][pitch] bf16 operand (pitch a multiple of 4) carved from p.
Cat3 carve_pitched(char*& p, long rows, int pitch, int lo_mask, int extra, const float* bias) {
    Cat3 c{reinterpret_cast<uint2*>(p), 0, lo_mask, pitch, extra, bias};
    p += ((rows * pitch * 2 + 255) / 256) * 256;
    return c;
}

// Segment patterns (bit g set: lo in segment g) so that the three products
// are hi*hi + lo*hi + hi*lo.
constexpr int PAT_HHL = 0b100;  // hi, hi, lo
constexpr int PAT_HLH = 0b010;  // hi, lo, hi

}  // namespace

ProjStatus proj_forward(void* handle, int num_sms, cudaStream_t s, cudaMemPool_t pool, const float* x, long ld_x, const float* w,
                        const float* b, float* y, long ld_y, int M, int N, int K, int* launches, int* gemms) {
    if (M == 0 || N == 0) return {};
    cublasHandle_t h = static_cast<cublasHandle_t>(handle);
    cudaError_t e;
    if (K == 0) {
        if (!b) {
            e = cudaMemset2DAsync(y, ld_y * 4, 0, static_cast<size_t>(N) * 4, M, s);
            return e == cudaSuccess ? ProjStatus{} : ProjStatus{e, CUBLAS_STATUS_SUCCESS, "cudaMemset2DAsync"};
        }
        e = launch_pdl(proj_fill_bias, dim3(grid_for(static_cast<long>(M) * N, num_sms)), dim3(256), 0, s, y, ld_y, M,
                       N, b);
        if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "bias fill"};
        ++*launches;
        return {};
    }
    Workspace ws;
    ws.s = s;
    // x' [M][Kp] = [x_hi | x_hi | x_lo (| 1, 1, 0...)], w' [N][Kp] = [w_hi | w_lo | w_hi (| b_hi, b_lo, 0...)]:
    // with a bias, the contraction carries it (Kp = 3K + 2 rounded up to 8).
    const int Kp = b ? biased_pitch(K) : 3 * K;
    const long xb = ((static_cast<long>(M) * Kp * 2 + 255) / 256) * 256;
    const long wb = ((static_cast<long>(N) * Kp * 2 + 255) / 256) * 256;
    e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws.base), xb + wb, pool, s);
    if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "workspace allocation"};
    char* p = ws.base;
    const Cat3 xc = carve_pitched(p, M, Kp, PAT_HHL, b ? EXTRA_ONES : EXTRA_NONE, nullptr);
    const Cat3 wc = carve_pitched(p, N, Kp, PAT_HLH, b ? EXTRA_BIAS : EXTRA_NONE, b);
    ProjStatus st = launch_split3(x, ld_x, M, K, xc, num_sms, s, launches);
    if (!st.ok()) return st;
    st = launch_split3(w, K, N, K, wc, num_sms, s, launches);
    if (!st.ok()) return st;
    return gemm(h, CUBLAS_OP_T, CUBLAS_OP_N, N, M, Kp, wc.p, Kp, xc.p, Kp, 0.f, y, ld_y, gemms);
}

ProjStatus proj_backward_dx(void* handle, int num_sms, cudaStream_t s, cudaMemPool_t pool, const float* dy, long ld_dy, const float* w,
                            float* dx, long ld_dx, int M, int N, int K, int* launches, int* gemms) {
    if (M == 0 || K == 0) return {};
    cublasHandle_t h = static_cast<cublasHandle_t>(handle);
    if (N == 0) {
        const cudaError_t e = cudaMemset2DAsync(dx, ld_dx * 4, 0, static_cast<size_t>(K) * 4, M, s);
        return e == cudaSuccess ? ProjStatus{} : ProjStatus{e, CUBLAS_STATUS_SUCCESS, "cudaMemset2DAsync"};
    }
    Workspace ws;
    ws.s = s;
    const long ed = static_cast<long>(M) * N, ew = static_cast<long>(N) * K;
    const cudaError_t e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws.base), cat3_bytes(ed) + cat3_bytes(ew), pool, s);
    if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "workspace allocation"};
    char* p = ws.base;
    // dy' [M][3N] = [dy_hi | dy_hi | dy_lo], w' [3N][K] = [w_hi; w_lo; w_hi].
    const Cat3 dc = carve(p, ed, 0, PAT_HHL), wc = carve(p, ew, 1, PAT_HLH);
    ProjStatus st = launch_split3(dy, ld_dy, M, N, dc, num_sms, s, launches);
    if (!st.ok()) return st;
    st = launch_split3(w, K, N, K, wc, num_sms, s, launches);
    if (!st.ok()) return st;
    return gemm(h, CUBLAS_OP_N, CUBLAS_OP_N, K, M, 3 * N, wc.p, K, dc.p, 3 * N, 0.f, dx, ld_dx, gemms);
}

ProjStatus proj_backward_dw(void* handle, int num_sms, cudaStream_t s, cudaMemPool_t pool, const float* dy, long ld_dy, const float* x,
                            long ld_x, float* dw, float* db, int M, int N, int K, int accumulate, int* launches,
                            int* gemms) {
    if (N == 0) return {};
    cublasHandle_t h = static_cast<cublasHandle_t>(handle);
    Workspace ws;
    ws.s = s;
    const long ed = static_cast<long>(M) * N, ex = static_cast<long>(M) * K;
    const int R = 64;  // rows per column-sum partial
    const int P = M > 0 ? (M + R - 1) / R : 1;
    const long part_bytes = ((static_cast<long>(P) * N * 4 + 255) / 256) * 256;
    cudaError_t e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws.base),
                                            cat3_bytes(ed) + cat3_bytes(ex) + (db ? part_bytes : 0), pool, s);
    if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "workspace allocation"};
    char* p = ws.base;
    // x' [3M][K] = [x_hi; x_hi; x_lo], dy' [3M][N] = [dy_hi; dy_lo; dy_hi].
    const Cat3 xc = carve(p, ex, 1, PAT_HHL), dc = carve(p, ed, 1, PAT_HLH);
    float* part = reinterpret_cast<float*>(p);
    if (db) {
        if (M > 0) {
            e = launch_pdl(proj_colsum_part, dim3((N + 255) / 256, P), dim3(256), 0, s, dy, ld_dy, M, N, R, part);
            if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "column sums"};
            ++*launches;
        }
        e = launch_pdl(proj_colsum_final, dim3((N + COLSUM_COLS - 1) / COLSUM_COLS), dim3(COLSUM_COLS, COLSUM_GROUPS),
                       0, s, static_cast<const float*>(part), M > 0 ? P : 0, N, db, accumulate);
        if (e != cudaSuccess) return {e, CUBLAS_STATUS_SUCCESS, "column sums"};
        ++*launches;
    }
    if (K == 0) return {};
    if (M == 0) {
        if (accumulate) return {};
        e = cudaMemsetAsync(dw, 0, static_cast<size_t>(N) * K * 4, s);
        return e == cudaSuccess ? ProjStatus{} : ProjStatus{e, CUBLAS_STATUS_SUCCESS, "cudaMemsetAsync"};
    }
    ProjStatus st = launch_split3(dy, ld_dy, M, N, dc, num_sms, s, launches);
    if (!st.ok()) return st;
    st = launch_split3(x, ld_x, M, K, xc, num_sms, s, launches);
    if (!st.ok()) return st;
    return gemm(h, CUBLAS_OP_N, CUBLAS_OP_T, K, N, 3 * M, xc.p, K, dc.p, N, accumulate ? 1.f : 0.f, dw, K, gemms);
}

}  // namespace kattn
