// LayerNorm forward and backward over rows of n_embd floats (sm_100a), the
// LN1 / LN2 around the attention sublayer.  Replaces
// ComputeBackend::layer_norm / layer_norm_batch (src/backend.rs:103, :140-142,
// CPU :258-267) and layer_norm_backward / layer_norm_backward_batch
// (src/backend.rs:184, :195-206, CPU src/backward.rs:93-128), called at
// src/pipeline.rs:236, :250, :678 and :743.
//
//   forward : mean = sum(x)/n, var = sum((x-mean)^2)/n, r = 1/sqrt(var+1e-5),
//             y = (x-mean) r w + b
//   backward: xh = (x-mean) r, g = dy w,
//             dx = r/n (n g - sum(g) - xh sum(g xh)),
//             dw += sum over rows of dy xh, db += sum over rows of dy
//
// One warp per row, the row in registers: lane l holds float4 chunks l,
// l+32, ... (V of them, n <= 128 V <= LN_MAX_N), so x is read from HBM once;
// w and b are staged in shared memory once per block.  Rows are independent;
// the column sums of dw and db are formed without atomics in a fixed order
// (each lane accumulates its columns over its warp's rows, the warps of a
// block add theirs in turn, then one pass sums the per-block partials in a
// fixed grouping), so results do not depend on scheduling.  The two-pass variance
// (deviations from the mean, as the reference computes it) keeps the
// precision of the reference's formula.
#include <cuda_runtime.h>

#include "kattn_common.cuh"
#include "kattn_launch.h"

namespace kattn {

namespace {

constexpr int LN_WARPS = 8;     // warps (rows in flight) per block
constexpr int LN_ROWS = 16;     // rows per block in the backward (column partials): 256 blocks at 4096 rows
constexpr int LN_MAX_V = LN_MAX_N / 128;
constexpr float LN_EPS = 1e-5f;

// w (and b) of n floats into shared memory, by the whole block.
__device__ __forceinline__ void stage_vec(float4* dst, const float* src, int n4) {
    for (int c = threadIdx.x; c < n4; c += blockDim.x) dst[c] = reinterpret_cast<const float4*>(src)[c];
}

// Lane `lane`'s chunks of a staged vector.
template <int V>
__device__ __forceinline__ float4 staged(const float4* v, int n4, int lane, int k) {
    const int c = lane + 32 * k;
    return c < n4 ? v[c] : make_float4(0.f, 0.f, 0.f, 0.f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Loads lane `lane`'s chunks of a row of n floats (zeros past n).
template <int V>
__device__ __forceinline__ void load_row(const float* row, int n4, int lane, float4 (&x)[V]) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
        const int c = lane + 32 * v;
        x[v] = c < n4 ? reinterpret_cast<const float4*>(row)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Row mean and 1/sqrt(var + eps) (two passes over the registers).
template <int V>
__device__ __forceinline__ void row_stats(const float4 (&x)[V], int n, int n4, int lane, float& mean, float& rstd) {
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) s += (x[v].x + x[v].y) + (x[v].z + x[v].w);
    mean = warp_sum(s) / static_cast<float>(n);
    float q = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
        if (lane + 32 * v < n4) {
            const float a = x[v].x - mean, b = x[v].y - mean, c = x[v].z - mean, d = x[v].w - mean;
            q += (a * a + b * b) + (c * c + d * d);
        }
    }
    rstd = 1.f / sqrtf(warp_sum(q) / static_cast<float>(n) + LN_EPS);
}

template <int V>
__global__ void __launch_bounds__(32 * LN_WARPS) ln_fwd(const float* __restrict__ x, long ld_x,
                                                          const float* __restrict__ w, const float* __restrict__ b,
                                                          float* __restrict__ y, long ld_y, int M, int n) {
    pdl_enter();
    extern __shared__ float4 ln_smem[];
    const int lane = threadIdx.x & 31;
    const int n4 = n / 4;
    float4* ws = ln_smem;
    float4* bs = ln_smem + n4;
    stage_vec(ws, w, n4);
    stage_vec(bs, b, n4);
    __syncthreads();
    for (long m = static_cast<long>(blockIdx.x) * LN_WARPS + (threadIdx.x >> 5); m < M;
         m += static_cast<long>(gridDim.x) * LN_WARPS) {
        float4 xv[V];
        load_row<V>(x + m * ld_x, n4, lane, xv);
        float mean, rstd;
        row_stats<V>(xv, n, n4, lane, mean, rstd);
        float4* yr = reinterpret_cast<float4*>(y + m * ld_y);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const int c = lane + 32 * v;
            if (c < n4) {
                const float4 wv = ws[c], bv = bs[c];
                yr[c] = make_float4((xv[v].x - mean) * rstd * wv.x + bv.x, (xv[v].y - mean) * rstd * wv.y + bv.y,
                                    (xv[v].z - mean) * rstd * wv.z + bv.z, (xv[v].w - mean) * rstd * wv.w + bv.w);
            }
        }
    }
}

// dx of every row; block p also writes its LN_ROWS rows' column sums of
// dy*xh and dy into part[p][0][:] and part[p][1][:] (plain stores).
template <int V>
__global__ void __launch_bounds__(32 * LN_WARPS) ln_bwd(const float* __restrict__ dy, long ld_dy,
                                                          const float* __restrict__ x, long ld_x,
                                                          const float* __restrict__ w, float* __restrict__ dx,
                                                          long ld_dx, float* __restrict__ part, int M, int n) {
    pdl_enter();
    extern __shared__ float4 ln_smem[];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int n4 = n / 4;
    float4* ws = ln_smem;            // w
    float4* acc = ln_smem + n4;      // [2][n4]: column sums of dy*xh, dy
    stage_vec(ws, w, n4);
    __syncthreads();
    float4 sw[V], sb[V];
#pragma unroll
    for (int v = 0; v < V; ++v) sw[v] = sb[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    const long r0 = static_cast<long>(blockIdx.x) * LN_ROWS;
    for (int i = wid; i < LN_ROWS; i += LN_WARPS) {
        const long m = r0 + i;
        if (m >= M) break;
        float4 xv[V], gv[V];
        load_row<V>(x + m * ld_x, n4, lane, xv);
        load_row<V>(dy + m * ld_dy, n4, lane, gv);
        float mean, rstd;
        row_stats<V>(xv, n, n4, lane, mean, rstd);
        // xv <- xh; column sums of dy*xh and dy; gv <- g = dy w; row sums of g and g xh.
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int v = 0; v < V; ++v) {
            xv[v] = make_float4((xv[v].x - mean) * rstd, (xv[v].y - mean) * rstd, (xv[v].z - mean) * rstd,
                                (xv[v].w - mean) * rstd);
            sw[v].x += gv[v].x * xv[v].x;
            sw[v].y += gv[v].y * xv[v].y;
            sw[v].z += gv[v].z * xv[v].z;
            sw[v].w += gv[v].w * xv[v].w;
            sb[v].x += gv[v].x;
            sb[v].y += gv[v].y;
            sb[v].z += gv[v].z;
            sb[v].w += gv[v].w;
            const float4 wv = staged<V>(ws, n4, lane, v);
            const float4 g = make_float4(gv[v].x * wv.x, gv[v].y * wv.y, gv[v].z * wv.z, gv[v].w * wv.w);
            gv[v] = g;
            s1 += (g.x + g.y) + (g.z + g.w);
            s2 += (g.x * xv[v].x + g.y * xv[v].y) + (g.z * xv[v].z + g.w * xv[v].w);
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        const float nf = static_cast<float>(n);
        const float k = rstd / nf;
        float4* dr = reinterpret_cast<float4*>(dx + m * ld_dx);
#pragma unroll
        for (int v = 0; v < V; ++v) {
            const int c = lane + 32 * v;
            if (c < n4)
                dr[c] = make_float4(k * (nf * gv[v].x - s1 - xv[v].x * s2), k * (nf * gv[v].y - s1 - xv[v].y * s2),
                                    k * (nf * gv[v].z - s1 - xv[v].z * s2), k * (nf * gv[v].w - s1 - xv[v].w * s2));
        }
    }
    // The block's column sums: the warps add theirs in warp order.
    for (int k = 0; k < LN_WARPS; ++k) {
        if (wid == k) {
#pragma unroll
            for (int v = 0; v < V; ++v) {
                const int c = lane + 32 * v;
                if (c < n4) {
                    float4 a0 = sw[v], a1 = sb[v];
                    if (k > 0) {
                        const float4 p0 = acc[c], p1 = acc[n4 + c];
                        a0 = make_float4(p0.x + a0.x, p0.y + a0.y, p0.z + a0.z, p0.w + a0.w);
                        a1 = make_float4(p1.x + a1.x, p1.y + a1.y, p1.z + a1.z, p1.w + a1.w);
                    }
                    acc[c] = a0;
                    acc[n4 + c] = a1;
                }
            }
        }
        __syncthreads();
    }
    float4* out = reinterpret_cast<float4*>(part + static_cast<long>(blockIdx.x) * 2 * n);
    for (int c = threadIdx.x; c < 2 * n4; c += blockDim.x) out[c] = acc[c];
}

// dw[c] (+)= sum_p part[p][0][c], db[c] (+)= sum_p part[p][1][c]: a CTA of
// 32 x 32 threads takes 32 of the 2n outputs, thread (x, y) sums partials
// y, y + 32, ... of output x, then thread (x, 0) adds the 32 sums in order of
// y.  The order is fixed: deterministic.
constexpr int LN_FINAL_COLS = 32;
constexpr int LN_FINAL_GROUPS = 32;

__global__ void __launch_bounds__(LN_FINAL_COLS* LN_FINAL_GROUPS)
    ln_colsum(const float* __restrict__ part, int P, int n, float* __restrict__ dw, float* __restrict__ db,
              int accumulate) {
    __shared__ float sums[LN_FINAL_GROUPS][LN_FINAL_COLS + 1];
    pdl_enter();
    const int x = threadIdx.x, y = threadIdx.y;
    const int c = blockIdx.x * LN_FINAL_COLS + x;
    const bool valid = c < 2 * n;
    const int which = valid ? c / n : 0, cc = c - which * n;
    float s = 0.f;
    if (valid)
        for (int p = y; p < P; p += LN_FINAL_GROUPS) s += part[(static_cast<long>(p) * 2 + which) * n + cc];
    sums[y][x] = s;
    __syncthreads();
    if (y != 0 || !valid) return;
    float t = 0.f;
    for (int g = 0; g < LN_FINAL_GROUPS; ++g) t += sums[g][x];
    float* dst = which ? db : dw;
    if (dst) dst[cc] = accumulate ? dst[cc] + t : t;
}

template <int V>
cudaError_t launch_fwd_v(const float* x, long ld_x, const float* w, const float* b, float* y, long ld_y, int M, int n,
                         int num_sms, cudaStream_t s) {
    const long blocks_needed = (static_cast<long>(M) + LN_WARPS - 1) / LN_WARPS;
    const long cap = 8L * (num_sms > 0 ? num_sms : 148);
    const unsigned grid = static_cast<unsigned>(blocks_needed < cap ? blocks_needed : cap);
    return launch_pdl(ln_fwd<V>, dim3(grid), dim3(32 * LN_WARPS), sizeof(float) * 2 * static_cast<size_t>(n), s, x,
                      ld_x, w, b, y, ld_y, M, n);
}

template <int V>
cudaError_t launch_bwd_v(const float* dy, long ld_dy, const float* x, long ld_x, const float* w, float* dx, long ld_dx,
                         float* part, int P, int M, int n, cudaStream_t s) {
    return launch_pdl(ln_bwd<V>, dim3(static_cast<unsigned>(P)), dim3(32 * LN_WARPS),
                      sizeof(float) * 3 * static_cast<size_t>(n), s, dy, ld_dy, x, ld_x, w, dx, ld_dx, part, M, n);
}

}  // namespace

bool ln_supported(int n) { return n > 0 && n % 4 == 0 && n <= LN_MAX_N; }

ProjStatus ln_forward(cudaStream_t s, int num_sms, const float* x, long ld_x, const float* w, const float* b, float* y,
                      long ld_y, int M, int n, int* launches) {
    ProjStatus st;
    if (M == 0) return st;
    const int V = (n + 127) / 128;
    cudaError_t e;
    switch (V) {
        case 1: e = launch_fwd_v<1>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 2: e = launch_fwd_v<2>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 3: e = launch_fwd_v<3>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 4: e = launch_fwd_v<4>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 5: e = launch_fwd_v<5>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 6: e = launch_fwd_v<6>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 7: e = launch_fwd_v<7>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 8: e = launch_fwd_v<8>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        case 9:
        case 10: e = launch_fwd_v<10>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
        default: e = launch_fwd_v<LN_MAX_V>(x, ld_x, w, b, y, ld_y, M, n, num_sms, s); break;
    }
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "layer-norm forward launch";
        return st;
    }
    *launches += 1;
    return st;
}

ProjStatus ln_backward(cudaStream_t s, cudaMemPool_t pool, const float* dy, long ld_dy, const float* x, long ld_x, const float* w,
                       float* dx, long ld_dx, float* dw, float* db, int M, int n, int accumulate, int* launches) {
    ProjStatus st;
    if (M == 0) {
        // No rows: dw / db receive nothing (written as zeros unless accumulating).
        if (!accumulate) {
            cudaError_t e = cudaSuccess;
            if (dw) e = cudaMemsetAsync(dw, 0, sizeof(float) * n, s);
            if (e == cudaSuccess && db) e = cudaMemsetAsync(db, 0, sizeof(float) * n, s);
            if (e != cudaSuccess) {
                st.cuda = e;
                st.what = "layer-norm gradient clear";
            }
        }
        return st;
    }
    const int P = (M + LN_ROWS - 1) / LN_ROWS;
    float* part = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&part), sizeof(float) * 2 * static_cast<size_t>(P) * n, pool, s);
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "layer-norm workspace";
        return st;
    }
    const int V = (n + 127) / 128;
    switch (V) {
        case 1: e = launch_bwd_v<1>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 2: e = launch_bwd_v<2>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 3: e = launch_bwd_v<3>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 4: e = launch_bwd_v<4>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 5: e = launch_bwd_v<5>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 6: e = launch_bwd_v<6>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 7: e = launch_bwd_v<7>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 8: e = launch_bwd_v<8>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        case 9:
        case 10: e = launch_bwd_v<10>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
        default: e = launch_bwd_v<LN_MAX_V>(dy, ld_dy, x, ld_x, w, dx, ld_dx, part, P, M, n, s); break;
    }
    if (e == cudaSuccess) {
        *launches += 1;
        e = launch_pdl(ln_colsum, dim3(static_cast<unsigned>((2 * n + LN_FINAL_COLS - 1) / LN_FINAL_COLS)),
                       dim3(LN_FINAL_COLS, LN_FINAL_GROUPS), 0, s, static_cast<const float*>(part), P, n, dw, db,
                       accumulate);
        if (e == cudaSuccess) *launches += 1;
    }
    const cudaError_t ef = cudaFreeAsync(part, s);
    if (e == cudaSuccess) e = ef;
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "layer-norm backward launch";
    }
    return st;
}

}  // namespace kattn
