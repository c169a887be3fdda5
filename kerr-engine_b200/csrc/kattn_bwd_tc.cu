// Causal self-attention backward on the 5th-generation tensor cores
// (sm_100a), head_dim 64.  Replaces ComputeBackend::attention_backward
// (src/backend.rs:223-231; CPU src/backward.rs:464-514; WGSL
// attn_backward_scores / attn_backward_dkv), recomputing the probabilities
// from the forward's log-sum-exp instead of reading a cached [H][T][T] P.
//
// CTA = one 128-row key tile of one (batch, head) slab; it keeps K, V and the
// dK, dV accumulators resident and walks the 64-row query tiles on or below
// the diagonal.  Products (bf16x3: hi*hi + hi*lo + lo*hi, f32 accumulation):
//   S^T  = K Q^T      M=128 (keys) N=64 (queries)   SS, both K-major
//   dP^T = V dO^T     M=128 N=64                    SS, both K-major
//   P = exp2(S^T * scale*log2e - lse*log2e),  dS = P * (dP^T - D)   (threads)
//   dV  += P^T dO     M=128 N=64 K=64    TS: P from TMEM, dO MN-major
//   dK  += dS^T Q     M=128 N=64 K=64    SS: dS^T K-major, Q MN-major
//   dQ_i = dS K       M=64  N=64 K=128   SS: dS^T read MN-major, K MN-major;
//                     added into global dq with vector reductions.
// D = rowsum(dO * O) and the zeroed dq come from attn_bwd_rowdot.
//
// Warp roles (288 threads, one CTA per SM):
//   warps 0-3  elementwise: thread t owns key row t (TMEM lane t); also the
//              dQ and final dK / dV epilogues
//   warps 4-7  loaders: K, V once; then Q, dO, lse, D per query tile into a
//              2-stage ring (full / empty mbarriers)
//   warp 8     one lane issues every tcgen05.mma and commit
// S^T / dP^T are double-buffered in TMEM so the tensor core computes tile
// i+1 while the elementwise warps work on tile i.
#include <atomic>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"
#include "tc_tiles.cuh"

namespace kattn {
using namespace sm100;

namespace {

constexpr int BK = 128;  // key rows per CTA
constexpr int BQ = 64;   // query rows per tile
constexpr int D = 64;
constexpr int NCOMP = 128;
constexpr int NLOAD = 128;
constexpr int NTHREADS = NCOMP + NLOAD + 32;

// TMEM columns (512 allocated)
__device__ __forceinline__ uint32_t col_s(int s) { return s ? 128u : 0u; }
__device__ __forceinline__ uint32_t col_dp(int s) { return s ? 192u : 64u; }
constexpr uint32_t COL_PH = 256;  // P^T hi: 64 queries as 32 bf16x2 columns
constexpr uint32_t COL_PL = 288;  // P^T lo
constexpr uint32_t COL_DQ = 320;  // dQ tile (M=64 layout)
constexpr uint32_t COL_DV = 384;
constexpr uint32_t COL_DK = 448;
constexpr uint32_t TMEM_COLS = 512;

struct alignas(1024) Smem {
    uint8_t kh[BK * 128];  // [key][64 bf16], 128B swizzle
    uint8_t kl[BK * 128];
    uint8_t vh[BK * 128];
    uint8_t vl[BK * 128];
    uint8_t qh[2][BQ * 128];  // [query][64 bf16]
    uint8_t ql[2][BQ * 128];
    uint8_t gh[2][BQ * 128];  // dO
    uint8_t gl[2][BQ * 128];
    uint8_t sh[BK * 128];  // dS^T [key][64 queries]
    uint8_t sl[BK * 128];
    float lse2[2][BQ];  // lse * log2(e), +inf beyond T
    float dsum[2][BQ];  // D, 0 beyond T
    uint64_t kv_full;
    uint64_t full[2];
    uint64_t empty[2];
    uint64_t bar_s[2];
    uint64_t pds;
    uint64_t bar_d;
    uint32_t tmem_slot;
};

struct Params {
    const float* q;
    const float* k;
    const float* v;
    long ld_qkv;
    const float* dout;
    long ld_o;
    const float* lse;
    const float* dsum;
    float* dq;
    float* dk;
    float* dv;
    long ld_d;
    int* status;
    int B, T, H;
    float scale;
    float scale_log2;
    int causal;
    int n_ktiles;  // 128-row key tiles
    int n_qtiles;  // 64-row query tiles
};

// S^T and dP^T of the query tile in stage s into TMEM buffer s.
__device__ __forceinline__ void issue_sdp(const Smem& sm, uint32_t tm, int s) {
    constexpr uint32_t idesc = idesc_bf16(BK, BQ, 0, 0);
    const uint32_t kh = smem_u32(sm.kh), kl = smem_u32(sm.kl), vh = smem_u32(sm.vh), vl = smem_u32(sm.vl);
    const uint32_t qh = smem_u32(sm.qh[s]), ql = smem_u32(sm.ql[s]), gh = smem_u32(sm.gh[s]), gl = smem_u32(sm.gl[s]);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
        const uint32_t o = ks * 32;
        const uint64_t akh = smem_desc(kh + o, 16, 1024), akl = smem_desc(kl + o, 16, 1024);
        const uint64_t bqh = smem_desc(qh + o, 16, 1024), bql = smem_desc(ql + o, 16, 1024);
        mma_ss(tm + col_s(s), akh, bqh, idesc, ks > 0);
        mma_ss(tm + col_s(s), akh, bql, idesc, 1);
        mma_ss(tm + col_s(s), akl, bqh, idesc, 1);
        const uint64_t avh = smem_desc(vh + o, 16, 1024), avl = smem_desc(vl + o, 16, 1024);
        const uint64_t bgh = smem_desc(gh + o, 16, 1024), bgl = smem_desc(gl + o, 16, 1024);
        mma_ss(tm + col_dp(s), avh, bgh, idesc, ks > 0);
        mma_ss(tm + col_dp(s), avh, bgl, idesc, 1);
        mma_ss(tm + col_dp(s), avl, bgh, idesc, 1);
    }
}

// dV += P^T dO, dK += dS^T Q (stage s), dQ = dS K.
__device__ __forceinline__ void issue_grads(const Smem& sm, uint32_t tm, int s, bool first) {
    constexpr uint32_t idesc_kv = idesc_bf16(BK, D, 0, 1);
    constexpr uint32_t idesc_q = idesc_bf16(BQ, D, 1, 1);
    const uint32_t qh = smem_u32(sm.qh[s]), ql = smem_u32(sm.ql[s]), gh = smem_u32(sm.gh[s]), gl = smem_u32(sm.gl[s]);
    const uint32_t sh = smem_u32(sm.sh), sl = smem_u32(sm.sl);
#pragma unroll
    for (int ks = 0; ks < BQ / 16; ++ks) {
        const uint32_t acc = (first && ks == 0) ? 0u : 1u;
        const uint64_t bgh = smem_desc(gh + ks * 2048, BQ * 128, 1024), bgl = smem_desc(gl + ks * 2048, BQ * 128, 1024);
        mma_ts(tm + COL_DV, tm + COL_PH + ks * 8, bgh, idesc_kv, acc);
        mma_ts(tm + COL_DV, tm + COL_PH + ks * 8, bgl, idesc_kv, 1);
        mma_ts(tm + COL_DV, tm + COL_PL + ks * 8, bgh, idesc_kv, 1);
        const uint64_t ash = smem_desc(sh + ks * 32, 16, 1024), asl = smem_desc(sl + ks * 32, 16, 1024);
        const uint64_t bqh = smem_desc(qh + ks * 2048, BQ * 128, 1024), bql = smem_desc(ql + ks * 2048, BQ * 128, 1024);
        mma_ss(tm + COL_DK, ash, bqh, idesc_kv, acc);
        mma_ss(tm + COL_DK, ash, bql, idesc_kv, 1);
        mma_ss(tm + COL_DK, asl, bqh, idesc_kv, 1);
    }
    const uint32_t kh = smem_u32(sm.kh), kl = smem_u32(sm.kl);
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
        const uint64_t ash = smem_desc(sh + ks * 2048, BK * 128, 1024), asl = smem_desc(sl + ks * 2048, BK * 128, 1024);
        const uint64_t bkh = smem_desc(kh + ks * 2048, BK * 128, 1024), bkl = smem_desc(kl + ks * 2048, BK * 128, 1024);
        mma_ss(tm + COL_DQ, ash, bkh, idesc_q, ks > 0);
        mma_ss(tm + COL_DQ, ash, bkl, idesc_q, 1);
        mma_ss(tm + COL_DQ, asl, bkh, idesc_q, 1);
    }
}

// dQ tile (M=64 accumulator: query row 16w + l sits in lane 32w + l, l < 16)
// scaled and added into global dq.
__device__ __forceinline__ void dq_epilogue(const Params& p, uint32_t tm, int warp, int lane, int q0, float* dqg) {
    float v0[32], v1[32];
    const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
    tmem_ld32(lb + tm + COL_DQ, v0);
    tmem_ld32(lb + tm + COL_DQ + 32, v1);
    tmem_wait_ld();
    const int r = q0 + warp * 16 + lane;
    if (lane < 16 && r < p.T) {
        float* dst = dqg + static_cast<long>(r) * p.ld_d;
#pragma unroll
        for (int c = 0; c < 32; c += 4)
            red_add_v4(dst + c, v0[c] * p.scale, v0[c + 1] * p.scale, v0[c + 2] * p.scale, v0[c + 3] * p.scale);
#pragma unroll
        for (int c = 0; c < 32; c += 4)
            red_add_v4(dst + 32 + c, v1[c] * p.scale, v1[c + 1] * p.scale, v1[c + 2] * p.scale,
                       v1[c + 3] * p.scale);
    }
}

__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_tc64(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int nslab = p.B * p.H;
    const int jt = static_cast<int>(blockIdx.x / nslab);  // key tile 0 sees the most query tiles: first
    const int slab = static_cast<int>(blockIdx.x % nslab);
    const int b = slab / p.H;
    const int h = slab % p.H;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int k0 = jt * BK;
    const int it0 = p.causal ? k0 / BQ : 0;  // first query tile with a row >= k0
    const int n_it = p.n_qtiles - it0;

    const long base = static_cast<long>(b) * p.T;
    const float* qg = p.q + base * p.ld_qkv + h * D;
    const float* kg = p.k + base * p.ld_qkv + h * D;
    const float* vg = p.v + base * p.ld_qkv + h * D;
    const float* dog = p.dout + base * p.ld_o + h * D;
    const float* lseg = p.lse + (static_cast<long>(b) * p.H + h) * p.T;
    const float* dsg = p.dsum + (static_cast<long>(b) * p.H + h) * p.T;
    float* dqg = p.dq + base * p.ld_d + h * D;

    if (warp == 0) {
        tmem_alloc(&sm.tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&sm.kv_full, NLOAD);
        mbar_init(&sm.full[0], NLOAD);
        mbar_init(&sm.full[1], NLOAD);
        mbar_init(&sm.empty[0], 1);
        mbar_init(&sm.empty[1], 1);
        mbar_init(&sm.bar_s[0], 1);
        mbar_init(&sm.bar_s[1], 1);
        mbar_init(&sm.pds, NCOMP);
        mbar_init(&sm.bar_d, 1);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sm.tmem_slot;
    bool failed = false;

    if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ loaders
        const int t = tid - NCOMP;
        tc::stage_rows<BK, NLOAD>(sm.kh, sm.kl, kg, p.ld_qkv, k0, p.T, 1.f, t);
        tc::stage_rows<BK, NLOAD>(sm.vh, sm.vl, vg, p.ld_qkv, k0, p.T, 1.f, t);
        fence_async_smem();
        mbar_arrive(&sm.kv_full);
        for (int n = 0; n < n_it; ++n) {
            const int s = n & 1;
            const int q0 = (it0 + n) * BQ;
            if (n >= 2 && !mbar_wait(&sm.empty[s], ((n - 2) >> 1) & 1)) {
                failed = true;
                break;
            }
            tc::stage_rows<BQ, NLOAD>(sm.qh[s], sm.ql[s], qg, p.ld_qkv, q0, p.T, 1.f, t);
            tc::stage_rows<BQ, NLOAD>(sm.gh[s], sm.gl[s], dog, p.ld_o, q0, p.T, 1.f, t);
            if (t < BQ) {
                const bool ok = q0 + t < p.T;
                sm.lse2[s][t] = ok ? lseg[q0 + t] * kLog2e : INFINITY;
                sm.dsum[s][t] = ok ? dsg[q0 + t] : 0.f;
            }
            fence_async_smem();
            mbar_arrive(&sm.full[s]);
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            failed = !mbar_wait(&sm.kv_full, 0);
            for (int n = 0; n < 2 && n < n_it && !failed; ++n) {
                if (!mbar_wait(&sm.full[n], 0)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                issue_sdp(sm, tm, n);
                mma_commit(&sm.bar_s[n]);
            }
            for (int n = 0; n < n_it && !failed; ++n) {
                const int s = n & 1;
                if (!mbar_wait(&sm.pds, n & 1)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                issue_grads(sm, tm, s, n == 0);
                mma_commit(&sm.empty[s]);
                mma_commit(&sm.bar_d);
                if (n + 2 < n_it) {
                    if (!mbar_wait(&sm.full[s], ((n + 2) >> 1) & 1)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    issue_sdp(sm, tm, s);
                    mma_commit(&sm.bar_s[s]);
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ elementwise (key row j)
        const int j = k0 + tid;
        const uint32_t lb = static_cast<uint32_t>(warp * 32) << 16;
        for (int n = 0; n < n_it; ++n) {
            const int s = n & 1;
            const int q0 = (it0 + n) * BQ;
            // full[s]: the loaders' lse / D writes for this tile are visible.
            if (!mbar_wait_warp(&sm.bar_s[s], (n >> 1) & 1) || !mbar_wait_warp(&sm.full[s], (n >> 1) & 1)) {
                failed = true;
                break;
            }
            if (n > 0) {
                // dQ of the previous tile; its MMAs also finished reading P^T and dS^T.
                if (!mbar_wait_warp(&sm.bar_d, (n - 1) & 1)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                dq_epilogue(p, tm, warp, lane, q0 - BQ, dqg);
            }
            tc_fence_after();
            const bool need_mask = (p.causal && q0 < k0 + BK - 1) || q0 + BQ > p.T || k0 + BK > p.T;
#pragma unroll
            for (int c = 0; c < BQ; c += 32) {
                float sv[32], dp[32];
                tmem_ld32(lb + tm + col_s(s) + c, sv);
                tmem_ld32(lb + tm + col_dp(s) + c, dp);
                tmem_wait_ld();
                uint32_t ph[16], pl[16], gh[16], gl[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    float p0 = ex2(fmaf(sv[i], p.scale_log2, -sm.lse2[s][c + i]));
                    float p1 = ex2(fmaf(sv[i + 1], p.scale_log2, -sm.lse2[s][c + i + 1]));
                    if (need_mask) {
                        const int qi = q0 + c + i;
                        if ((p.causal && qi < j) || qi >= p.T || j >= p.T) p0 = 0.f;
                        if ((p.causal && qi + 1 < j) || qi + 1 >= p.T || j >= p.T) p1 = 0.f;
                    }
                    const float g0 = p0 * (dp[i] - sm.dsum[s][c + i]);
                    const float g1 = p1 * (dp[i + 1] - sm.dsum[s][c + i + 1]);
                    split2(p0, p1, ph[i >> 1], pl[i >> 1]);
                    split2(g0, g1, gh[i >> 1], gl[i >> 1]);
                }
                tmem_st16(lb + tm + COL_PH + c / 2, ph);
                tmem_st16(lb + tm + COL_PL + c / 2, pl);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t off = sw128(tid, c / 8 + u);
                    *reinterpret_cast<uint4*>(sm.sh + off) =
                        make_uint4(gh[4 * u], gh[4 * u + 1], gh[4 * u + 2], gh[4 * u + 3]);
                    *reinterpret_cast<uint4*>(sm.sl + off) =
                        make_uint4(gl[4 * u], gl[4 * u + 1], gl[4 * u + 2], gl[4 * u + 3]);
                }
            }
            tmem_wait_st();
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(&sm.pds);
        }
        if (!failed) {
            if (!mbar_wait_warp(&sm.bar_d, (n_it - 1) & 1)) {
                failed = true;
            } else {
                tc_fence_after();
                dq_epilogue(p, tm, warp, lane, (it0 + n_it - 1) * BQ, dqg);
                // dK, dV for this key row: the TMEM loads are warp-collective and
                // run on every lane; only rows below T are stored.
                float* dkr = p.dk + (base + j) * p.ld_d + h * D;
                float* dvr = p.dv + (base + j) * p.ld_d + h * D;
                const bool store = j < p.T;
                float a[32];
#pragma unroll
                for (int c = 0; c < D; c += 32) {
                    tmem_ld32(lb + tm + COL_DV + c, a);
                    tmem_wait_ld();
                    if (store) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(dvr + c + i) = make_float4(a[i], a[i + 1], a[i + 2], a[i + 3]);
                    }
                    tmem_ld32(lb + tm + COL_DK + c, a);
                    tmem_wait_ld();
                    if (store) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(dkr + c + i) = make_float4(
                                a[i] * p.scale, a[i + 1] * p.scale, a[i + 2] * p.scale, a[i + 3] * p.scale);
                    }
                }
            }
        }
    }

    if (failed) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, TMEM_COLS);
}

}  // namespace

bool bwd_tc_supported(const BwdArgs& a) { return a.d == 64; }

cudaError_t launch_bwd_tc(const BwdArgs& a, int num_sms, int* status, cudaStream_t stream, int* launches) {
    cudaError_t e = launch_bwd_prep(a, num_sms, stream, launches);
    if (e != cudaSuccess) return e;
    Params p;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.ld_qkv = a.ld_qkv;
    p.dout = a.dout;
    p.ld_o = a.ld_o;
    p.lse = a.lse;
    p.dsum = a.dsum;
    p.dq = a.dq;
    p.dk = a.dk;
    p.dv = a.dv;
    p.ld_d = a.ld_d;
    p.status = status;
    p.B = a.B;
    p.T = a.T;
    p.H = a.H;
    p.scale = a.scale;
    p.scale_log2 = a.scale * kLog2e;
    p.causal = a.causal;
    p.n_ktiles = (a.T + BK - 1) / BK;
    p.n_qtiles = (a.T + BQ - 1) / BQ;
    const size_t smem = sizeof(Smem) + 1024;
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(attn_bwd_tc64, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    const long nblocks = static_cast<long>(p.n_ktiles) * a.B * a.H;
    attn_bwd_tc64<<<static_cast<unsigned>(nblocks), NTHREADS, smem, stream>>>(p);
    e = cudaGetLastError();
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
