// Causal self-attention backward, f32 on the FFMA pipe (sm_100a).
//
// Replaces ComputeBackend::attention_backward (src/backend.rs:223-231; CPU
// src/backward.rs:464-514, WGSL attn_backward_scores / attn_backward_dkv).
// The reference backpropagates through the cached post-softmax weights P;
// here P is recomputed tile by tile from the saved row log-sum-exp, so nothing
// of size T^2 is stored.  With D_r = sum_c dO[r,c] * O[r,c] (= the reference's
// sum_j att[j] * d_att[j], src/backward.rs:501):
//   P  = exp(scale * Q K^T - lse)        dV = P^T dO
//   dP = dO V^T                          dS = P * (dP - D)
//   dQ = scale * dS K                    dK = scale * dS^T Q
//
// Kernel 1 (attn_bwd_rowdot) computes D into a [B][H][T] workspace and zeroes
// dQ.  Kernel 2 (attn_bwd_f32): one CTA per (64-row key tile, slab) keeps K, V
// and the dK, dV accumulators resident and walks the query tiles on or below
// the diagonal; dQ partial sums go to global memory with vector reductions.
#include <algorithm>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"

namespace kattn {

constexpr int BWD_BM = 64;  // query rows per tile
constexpr int BWD_BN = 64;  // key rows per CTA
constexpr int BWD_NT = 256;
static_assert(BWD_BN == kBwdF32KeyRows, "dQ slices of the deterministic mode");

struct BwdParams {
    const float* q;
    const float* k;
    const float* v;
    long ld_qkv;
    const float* o;
    const float* dout;
    long ld_o;
    const float* lse;
    float* dq;
    float* dq_part;  // deterministic mode: [key tiles][B*T][H*D] slices, or null
    float* dk;
    float* dv;
    long ld_d;
    float* dsum;
    int B, T, H;
    float scale;
    float scale_log2;
    int causal;
    int n_tiles;
};

// D[b,h,t] = dout[b,t,h,:] . o[b,t,h,:];  dq[b,t,h,:] = 0.
// D/W lanes per (b, t, h) row, W floats each (W = 8: one 256-bit load of
// dout and of o per lane, when their rows and dq's start on 32-byte
// boundaries; W = 4: 128-bit loads); a warp takes RPW*U consecutive rows
// (consecutive heads of a token are contiguous in memory) and issues all U
// rounds of loads before it reduces any.  U = 1 (one row per lane group,
// more warps) measured faster than U = 4 at the 768-dim shape.
constexpr int ROWDOT_U = 1;

template <int D, bool V8>
__global__ void __launch_bounds__(256) attn_bwd_rowdot(const BwdParams p) {
    // Wait for the grid before (the one that wrote o, dout or q, k, v), then
    // let the backward kernel behind this one launch.  That order matters:
    // attn_bwd_tc64 stages K and V before its own griddepcontrol.wait, which
    // is safe only because no grid before this one is still running once
    // this grid has passed its wait.  D must also be written only after this
    // wait: kattn_bwd_noalloc hands every call the same workspace array, and
    // the previous call's backward kernel, which reads it, is (or precedes)
    // the grid waited for here.
    pdl_wait();
    pdl_launch();
    constexpr int W = V8 ? 8 : 4;
    constexpr int LPR = D / W;
    constexpr int RPW = 32 / LPR;
    constexpr int U = ROWDOT_U;
    const long nrows = static_cast<long>(p.B) * p.T * p.H;
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int c = (lane % LPR) * W;
    const long warp = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long nwarps = (static_cast<long>(gridDim.x) * blockDim.x) >> 5;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long base = warp * RPW * U; base < nrows; base += nwarps * RPW * U) {
        float4 g[U][2], o[U][2];
        long bt[U];
        int h[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const long row = base + u * RPW + sub;
            bt[u] = row / p.H;
            h[u] = static_cast<int>(row - bt[u] * p.H);
            g[u][0] = g[u][1] = o[u][0] = o[u][1] = z;
            if (row < nrows) {
                const float* gp = p.dout + bt[u] * p.ld_o + h[u] * D + c;
                const float* op = p.o + bt[u] * p.ld_o + h[u] * D + c;
                if constexpr (V8) {
                    sm100::ldg_v8(gp, g[u][0], g[u][1]);
                    sm100::ldg_v8(op, o[u][0], o[u][1]);
                } else {
                    g[u][0] = *reinterpret_cast<const float4*>(gp);
                    o[u][0] = *reinterpret_cast<const float4*>(op);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const long row = base + u * RPW + sub;
            // Both paths add in one order, so D is bitwise the same: a sum of
            // four products per 4-column group, then a butterfly over the
            // groups.  A 256-bit lane holds groups 2l and 2l+1, which pair
            // up in the butterfly's last step.
            float acc = g[u][0].x * o[u][0].x + g[u][0].y * o[u][0].y + g[u][0].z * o[u][0].z + g[u][0].w * o[u][0].w;
            float acc1 = 0.f;
            if constexpr (V8)
                acc1 = g[u][1].x * o[u][1].x + g[u][1].y * o[u][1].y + g[u][1].z * o[u][1].z + g[u][1].w * o[u][1].w;
#pragma unroll
            for (int off = LPR / 2; off > 0; off >>= 1) {
                acc += __shfl_xor_sync(0xffffffffu, acc, off);
                if constexpr (V8) acc1 += __shfl_xor_sync(0xffffffffu, acc1, off);
            }
            if constexpr (V8) acc += acc1;
            if (row < nrows) {
                float* dqp = p.dq + bt[u] * p.ld_d + h[u] * D + c;
                if constexpr (V8)
                    sm100::stg_v8(dqp, z, z);
                else
                    *reinterpret_cast<float4*>(dqp) = z;
                if ((lane % LPR) == 0) {
                    const long b = bt[u] / p.T;
                    const long t = bt[u] - b * p.T;
                    p.dsum[(b * p.H + h[u]) * p.T + t] = acc;
                }
            }
        }
    }
}

template <int D>
struct BwdSmem {
    static constexpr int LDD = D + 4;       // pitch of q/dO/k/v tiles
    static constexpr int LDT = BWD_BM + 4;  // pitch of the transposed P / dS tiles ([key][query])
    float k[BWD_BN * LDD];
    float v[BWD_BN * LDD];
    float q[BWD_BM * LDD];
    float dO[BWD_BM * LDD];
    float pt[BWD_BN * LDT];
    float dst[BWD_BN * LDT];
    float lse[BWD_BM];
    float dsum[BWD_BM];
};

__device__ __forceinline__ float f4get(const float4& v, int u) {
    return u == 0 ? v.x : u == 1 ? v.y : u == 2 ? v.z : v.w;
}

template <int D>
__global__ void __launch_bounds__(BWD_NT, (D <= 64 ? 2 : 1)) attn_bwd_f32(const BwdParams p) {
    pdl_enter();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    BwdSmem<D>& sm = *reinterpret_cast<BwdSmem<D>*>(smem_raw);
    constexpr int LDD = BwdSmem<D>::LDD;
    constexpr int LDT = BwdSmem<D>::LDT;
    constexpr int DC = D / 16;
    constexpr int C4 = D / 4;

    const int nslab = p.B * p.H;
    const int jt = static_cast<int>(blockIdx.x / nslab);  // key tile 0 sees the most query tiles: first
    const int slab = static_cast<int>(blockIdx.x % nslab);
    const int b = slab / p.H;
    const int h = slab % p.H;
    const int tid = threadIdx.x;
    const int tx = tid & 15;
    const int ty = tid >> 4;
    const int k0 = jt * BWD_BN;

    const long row0 = static_cast<long>(b) * p.T;
    const float* qg = p.q + row0 * p.ld_qkv + h * D;
    const float* kg = p.k + row0 * p.ld_qkv + h * D;
    const float* vg = p.v + row0 * p.ld_qkv + h * D;
    const float* dog = p.dout + row0 * p.ld_o + h * D;
    const float* lseg = p.lse + (static_cast<long>(b) * p.H + h) * p.T;
    const float* dsg = p.dsum + (static_cast<long>(b) * p.H + h) * p.T;

    // Resident key / value tile.
#pragma unroll
    for (int i = tid; i < BWD_BN * C4; i += BWD_NT) {
        const int r = i / C4;
        const int c = (i % C4) * 4;
        const bool ok = k0 + r < p.T;
        const long off = static_cast<long>(ok ? k0 + r : 0) * p.ld_qkv + c;
        cp_async16(&sm.k[r * LDD + c], kg + off, ok ? 16 : 0);
        cp_async16(&sm.v[r * LDD + c], vg + off, ok ? 16 : 0);
    }

    auto load_q = [&](int it) {
        const int q0 = it * BWD_BM;
#pragma unroll
        for (int i = tid; i < BWD_BM * C4; i += BWD_NT) {
            const int r = i / C4;
            const int c = (i % C4) * 4;
            const bool ok = q0 + r < p.T;
            cp_async16(&sm.q[r * LDD + c], qg + static_cast<long>(ok ? q0 + r : 0) * p.ld_qkv + c, ok ? 16 : 0);
            cp_async16(&sm.dO[r * LDD + c], dog + static_cast<long>(ok ? q0 + r : 0) * p.ld_o + c, ok ? 16 : 0);
        }
        if (tid < BWD_BM) {
            const bool ok = q0 + tid < p.T;
            sm.lse[tid] = ok ? lseg[q0 + tid] * kLog2e : INFINITY;
            sm.dsum[tid] = ok ? dsg[q0 + tid] : 0.f;
        }
        cp_async_commit();
    };

    float dk[4][DC], dv[4][DC];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < DC; ++c) {
            dk[a][c] = 0.f;
            dv[a][c] = 0.f;
        }

    const int it0 = p.causal ? jt : 0;
    load_q(it0);

    for (int it = it0; it < p.n_tiles; ++it) {
        const int q0 = it * BWD_BM;
        cp_async_wait<0>();
        __syncthreads();

        // S = Q K^T and dP = dO V^T on rows ty+16a (query), columns tx+16c (key).
        float s[4][4], dp[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                s[a][c] = 0.f;
                dp[a][c] = 0.f;
            }
#pragma unroll 1
        for (int kk = 0; kk < D; kk += 4) {
            float4 xa[4], ga[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                xa[a] = *reinterpret_cast<const float4*>(&sm.q[(ty + 16 * a) * LDD + kk]);
                ga[a] = *reinterpret_cast<const float4*>(&sm.dO[(ty + 16 * a) * LDD + kk]);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float4 kb = *reinterpret_cast<const float4*>(&sm.k[(tx + 16 * c) * LDD + kk]);
                const float4 vb = *reinterpret_cast<const float4*>(&sm.v[(tx + 16 * c) * LDD + kk]);
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    s[a][c] = fmaf(xa[a].x, kb.x, s[a][c]);
                    s[a][c] = fmaf(xa[a].y, kb.y, s[a][c]);
                    s[a][c] = fmaf(xa[a].z, kb.z, s[a][c]);
                    s[a][c] = fmaf(xa[a].w, kb.w, s[a][c]);
                    dp[a][c] = fmaf(ga[a].x, vb.x, dp[a][c]);
                    dp[a][c] = fmaf(ga[a].y, vb.y, dp[a][c]);
                    dp[a][c] = fmaf(ga[a].z, vb.z, dp[a][c]);
                    dp[a][c] = fmaf(ga[a].w, vb.w, dp[a][c]);
                }
            }
        }

        // P and dS, stored transposed ([key][query]) for the dV / dK / dQ products.
        const bool need_mask = (p.causal && it == jt) || k0 + BWD_BN > p.T || q0 + BWD_BM > p.T;
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int rl = ty + 16 * a;
            const float lse2 = sm.lse[rl];
            const float dd = sm.dsum[rl];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int cl = tx + 16 * c;
                float pv = ex2(fmaf(s[a][c], p.scale_log2, -lse2));
                if (need_mask) {
                    const int r = q0 + rl;
                    const int col = k0 + cl;
                    if ((p.causal && col > r) || col >= p.T || r >= p.T) pv = 0.f;
                }
                sm.pt[cl * LDT + rl] = pv;
                sm.dst[cl * LDT + rl] = pv * (dp[a][c] - dd);
            }
        }
        __syncthreads();

        // dV += P^T dO, dK += dS^T Q on key rows ty+16a, columns tx*DC.
#pragma unroll 1
        for (int r = 0; r < BWD_BM; r += 4) {
            float4 pa[4], sa[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                pa[a] = *reinterpret_cast<const float4*>(&sm.pt[(ty + 16 * a) * LDT + r]);
                sa[a] = *reinterpret_cast<const float4*>(&sm.dst[(ty + 16 * a) * LDT + r]);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                Frag<DC> gr, qr;
                gr.load(&sm.dO[(r + u) * LDD + tx * DC]);
                qr.load(&sm.q[(r + u) * LDD + tx * DC]);
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float pu = f4get(pa[a], u);
                    const float su = f4get(sa[a], u);
#pragma unroll
                    for (int c = 0; c < DC; ++c) {
                        dv[a][c] = fmaf(pu, gr.x[c], dv[a][c]);
                        dk[a][c] = fmaf(su, qr.x[c], dk[a][c]);
                    }
                }
            }
        }
        __syncthreads();  // q / dO are refilled below while dQ is formed

        if (it + 1 < p.n_tiles) load_q(it + 1);

        // dQ(partial) = dS K on query rows ty*4+a, columns tx*DC.
        float dqa[4][DC];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < DC; ++c) dqa[a][c] = 0.f;
#pragma unroll 4
        for (int c = 0; c < BWD_BN; ++c) {
            const float4 sc = *reinterpret_cast<const float4*>(&sm.dst[c * LDT + ty * 4]);
            Frag<DC> kr;
            kr.load(&sm.k[c * LDD + tx * DC]);
#pragma unroll
            for (int cc = 0; cc < DC; ++cc) {
                dqa[0][cc] = fmaf(sc.x, kr.x[cc], dqa[0][cc]);
                dqa[1][cc] = fmaf(sc.y, kr.x[cc], dqa[1][cc]);
                dqa[2][cc] = fmaf(sc.z, kr.x[cc], dqa[2][cc]);
                dqa[3][cc] = fmaf(sc.w, kr.x[cc], dqa[3][cc]);
            }
        }
        // dQ: added into dq, or (deterministic mode) stored into this key
        // tile's slice for attn_bwd_dq_reduce.
        const long hd = static_cast<long>(p.H) * D;
        float* dqg = p.dq_part ? p.dq_part + (static_cast<long>(jt) * p.B * p.T + row0) * hd + h * D
                               : p.dq + row0 * p.ld_d + h * D;
        const long ldq = p.dq_part ? hd : p.ld_d;
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int r = q0 + ty * 4 + a;
            if (r < p.T) {
                Frag<DC> f;
#pragma unroll
                for (int cc = 0; cc < DC; ++cc) f.x[cc] = dqa[a][cc] * p.scale;
                if (p.dq_part) f.store(dqg + static_cast<long>(r) * ldq + tx * DC);
                else f.red_add(dqg + static_cast<long>(r) * ldq + tx * DC);
            }
        }
    }
    cp_async_wait<0>();

    float* dkg = p.dk + row0 * p.ld_d + h * D;
    float* dvg = p.dv + row0 * p.ld_d + h * D;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int r = k0 + ty + 16 * a;
        if (r < p.T) {
            Frag<DC> fk, fv;
#pragma unroll
            for (int c = 0; c < DC; ++c) {
                fk.x[c] = dk[a][c] * p.scale;
                fv.x[c] = dv[a][c];
            }
            fk.store(dkg + static_cast<long>(r) * p.ld_d + tx * DC);
            fv.store(dvg + static_cast<long>(r) * p.ld_d + tx * DC);
        }
    }
}

static BwdParams make_params(const BwdArgs& a) {
    BwdParams p;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.ld_qkv = a.ld_qkv;
    p.o = a.o;
    p.dout = a.dout;
    p.ld_o = a.ld_o;
    p.lse = a.lse;
    p.dq = a.dq;
    p.dq_part = a.dq_part;
    p.dk = a.dk;
    p.dv = a.dv;
    p.ld_d = a.ld_d;
    p.dsum = a.dsum;
    p.B = a.B;
    p.T = a.T;
    p.H = a.H;
    p.scale = a.scale;
    p.scale_log2 = a.scale * kLog2e;
    p.causal = a.causal;
    p.n_tiles = (a.T + BWD_BM - 1) / BWD_BM;
    return p;
}

template <int D>
static cudaError_t launch_prep_d(const BwdParams& p, int num_sms, cudaStream_t stream, int* launches) {
    // One wave when it fits (8 blocks of 256 threads per SM), every load
    // issued at once; larger problems take grid-stride rounds.
    // 256-bit accesses when every row of o, dout and dq starts on a 32-byte
    // boundary (the per-head offsets, D * 4 bytes, keep it).
    auto a32 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 31) == 0; };
    const bool v8 = a32(p.o) && a32(p.dout) && a32(p.dq) && p.ld_o % 8 == 0 && p.ld_d % 8 == 0;
    const long nrows = static_cast<long>(p.B) * p.T * p.H;
    const long rows_per_block = (256 / 32) * (32 / (D / (v8 ? 8 : 4))) * ROWDOT_U;
    long blocks = (nrows + rows_per_block - 1) / rows_per_block;
    const long cap = 8L * (num_sms > 0 ? num_sms : 148);
    if (blocks > cap) blocks = cap;
    cudaError_t e = launch_pdl(v8 ? attn_bwd_rowdot<D, true> : attn_bwd_rowdot<D, false>,
                               dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, p);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

cudaError_t launch_bwd_prep(const BwdArgs& a, int num_sms, cudaStream_t stream, int* launches) {
    const BwdParams p = make_params(a);
    switch (a.d) {
        case 32: return launch_prep_d<32>(p, num_sms, stream, launches);
        case 64: return launch_prep_d<64>(p, num_sms, stream, launches);
        case 128: return launch_prep_d<128>(p, num_sms, stream, launches);
        default: return cudaErrorInvalidValue;
    }
}

// Deterministic dQ: dq[row][h*D + c] = sum of the key tiles' slices in tile
// order.  One thread per float4 of dq's H*D columns, grid-stride.
__global__ void __launch_bounds__(256) attn_bwd_dq_reduce(float* dq, long ld_d, const float* __restrict__ part,
                                                          long rows, int T, int hd, int n_kt, int key_rows,
                                                          int causal) {
    pdl_enter();
    const int c4 = hd / 4;
    const long plane = rows * hd;
    const long total = rows * c4;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / c4;
        const int c = 4 * static_cast<int>(i - r * c4);
        const int t = static_cast<int>(r % T);
        const int jmax = causal ? min(n_kt - 1, t / key_rows) : n_kt - 1;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j <= jmax; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(part + j * plane + r * hd + c);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        *reinterpret_cast<float4*>(dq + r * ld_d + c) = acc;
    }
}

cudaError_t launch_bwd_dq_reduce(const BwdArgs& a, int key_rows, int num_sms, cudaStream_t stream, int* launches) {
    const long rows = static_cast<long>(a.B) * a.T;
    const int hd = a.H * a.d;
    const int n_kt = (a.T + key_rows - 1) / key_rows;
    const long n4 = rows * (hd / 4);
    const long grid = std::min<long>((n4 + 255) / 256, 8L * (num_sms > 0 ? num_sms : 148));
    cudaError_t e = launch_pdl(attn_bwd_dq_reduce, dim3(static_cast<unsigned>(grid)), dim3(256), 0, stream, a.dq,
                               a.ld_d, static_cast<const float*>(a.dq_part), rows, a.T, hd, n_kt, key_rows, a.causal);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

template <int D>
static cudaError_t launch_bwd_d(const BwdArgs& a, int num_sms, cudaStream_t stream, int* launches) {
    const BwdParams p = make_params(a);
    cudaError_t e = launch_prep_d<D>(p, num_sms, stream, launches);
    if (e != cudaSuccess) return e;
    const size_t smem = sizeof(BwdSmem<D>);
    e = cudaFuncSetAttribute(attn_bwd_f32<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const long nblocks = static_cast<long>(p.n_tiles) * a.B * a.H;
    e = launch_pdl(attn_bwd_f32<D>, dim3(static_cast<unsigned>(nblocks)), dim3(BWD_NT), smem, stream, p);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

cudaError_t launch_bwd(const BwdArgs& a, int num_sms, cudaStream_t stream, int* launches) {
    switch (a.d) {
        case 32: return launch_bwd_d<32>(a, num_sms, stream, launches);
        case 64: return launch_bwd_d<64>(a, num_sms, stream, launches);
        case 128: return launch_bwd_d<128>(a, num_sms, stream, launches);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace kattn
