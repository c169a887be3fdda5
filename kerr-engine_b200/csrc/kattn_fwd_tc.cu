// Causal self-attention forward on the 5th-generation tensor cores (sm_100a),
// head_dim 64.  Replaces the scalar head loop of src/pipeline.rs:305-347.
//
// Numerics: every f32 operand x is split into bf16 hi = bf16(x) and
// lo = bf16(x - hi); each product A*B is formed as hi*hi + hi*lo + lo*hi with
// f32 accumulation in tensor memory (relative error ~1e-5, inside the 1e-4
// forward tolerance; a single bf16 or tf32 product is not).
//
// CTA = 128 query rows of one (batch, head) slab, 128 threads; thread t owns
// query row t (TMEM lane t).  Per 64-row key tile j:
//   S_j = Q K_j^T           tcgen05.mma SS, M=128 N=64, 3 x 4 k-steps   -> TMEM
//   softmax (online, log2 domain) in registers; P_j hi/lo -> TMEM
//   O_j = P_j V_j           tcgen05.mma TS (P from TMEM), V MN-major    -> TMEM
//   O  <- O * alpha + O_j   in registers
// S_{j+1} is issued right behind O_j, so the tensor core computes it while the
// threads fold O_j in and stage key/value tile j+2.  ~99 KB of shared memory
// and 256 TMEM columns per CTA: two CTAs share an SM.
#include <atomic>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"
#include "tc_tiles.cuh"

namespace kattn {
using namespace sm100;

namespace {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 64;   // key rows per tile
constexpr int NT = 128;
constexpr int D = 64;

// TMEM columns
constexpr uint32_t COL_S = 0;    // S tile, 64 f32 columns
constexpr uint32_t COL_PH = 64;  // P hi, 64 bf16 packed in 32 columns
constexpr uint32_t COL_PL = 96;  // P lo
constexpr uint32_t COL_O = 128;  // O tile, 64 f32 columns
constexpr uint32_t TMEM_COLS = 256;

struct alignas(1024) Smem {
    uint8_t qh[BM * 128];  // [128 rows][64 bf16], 128B swizzle
    uint8_t ql[BM * 128];
    uint8_t kh[2][BN * 128];
    uint8_t kl[2][BN * 128];
    uint8_t vh[2][BN * 128];
    uint8_t vl[2][BN * 128];
    uint64_t bar_s;
    uint64_t bar_o;
    uint32_t tmem_slot;
};

struct Params {
    const float* q;
    const float* k;
    const float* v;
    long ld_qkv;
    float* o;
    long ld_o;
    float* lse;
    int* status;
    int B, T, H;
    float scale_log2;
    int causal;
    int n_qtiles;
    int n_ktiles;
};

__device__ __forceinline__ void issue_s(const Smem& sm, uint32_t tm, int stage) {
    constexpr uint32_t idesc = idesc_bf16(BM, BN, 0, 0);
    const uint32_t qh = smem_u32(sm.qh), ql = smem_u32(sm.ql);
    const uint32_t kh = smem_u32(sm.kh[stage]), kl = smem_u32(sm.kl[stage]);
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
        const uint64_t aqh = smem_desc(qh + s * 32, 16, 1024), aql = smem_desc(ql + s * 32, 16, 1024);
        const uint64_t bkh = smem_desc(kh + s * 32, 16, 1024), bkl = smem_desc(kl + s * 32, 16, 1024);
        mma_ss(tm + COL_S, aqh, bkh, idesc, s > 0);
        mma_ss(tm + COL_S, aqh, bkl, idesc, 1);
        mma_ss(tm + COL_S, aql, bkh, idesc, 1);
    }
}

__device__ __forceinline__ void issue_pv(const Smem& sm, uint32_t tm, int stage) {
    constexpr uint32_t idesc = idesc_bf16(BM, D, 0, 1);
    const uint32_t vh = smem_u32(sm.vh[stage]), vl = smem_u32(sm.vl[stage]);
#pragma unroll
    for (int s = 0; s < BN / 16; ++s) {
        const uint64_t bvh = smem_desc(vh + s * 2048, BN * 128, 1024);
        const uint64_t bvl = smem_desc(vl + s * 2048, BN * 128, 1024);
        mma_ts(tm + COL_O, tm + COL_PH + s * 8, bvh, idesc, s > 0);
        mma_ts(tm + COL_O, tm + COL_PH + s * 8, bvl, idesc, 1);
        mma_ts(tm + COL_O, tm + COL_PL + s * 8, bvh, idesc, 1);
    }
}

__global__ void __launch_bounds__(NT, 2) attn_fwd_tc64(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int nslab = p.B * p.H;
    const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x / nslab);  // longest rows first
    const int slab = static_cast<int>(blockIdx.x % nslab);
    const int b = slab / p.H;
    const int h = slab % p.H;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int q0 = qt * BM;
    const int row = q0 + tid;
    const int n_kv = p.causal ? min(p.n_ktiles, (q0 + BM + BN - 1) / BN) : p.n_ktiles;

    const long base = static_cast<long>(b) * p.T;
    const float* qg = p.q + base * p.ld_qkv + h * D;
    const float* kg = p.k + base * p.ld_qkv + h * D;
    const float* vg = p.v + base * p.ld_qkv + h * D;

    if (warp == 0) {
        tmem_alloc(&sm.tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&sm.bar_s, 1);
        mbar_init(&sm.bar_o, 1);
    }
    tc::stage_rows<BM, NT>(sm.qh, sm.ql, qg, p.ld_qkv, q0, p.T, p.scale_log2, tid);
    tc::stage_rows<BN, NT>(sm.kh[0], sm.kl[0], kg, p.ld_qkv, 0, p.T, 1.f, tid);
    tc::stage_rows<BN, NT>(sm.vh[0], sm.vl[0], vg, p.ld_qkv, 0, p.T, 1.f, tid);
    if (n_kv > 1) {
        tc::stage_rows<BN, NT>(sm.kh[1], sm.kl[1], kg, p.ld_qkv, BN, p.T, 1.f, tid);
        tc::stage_rows<BN, NT>(sm.vh[1], sm.vl[1], vg, p.ld_qkv, BN, p.T, 1.f, tid);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sm.tmem_slot;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

    if (tid == 0) {
        issue_s(sm, tm, 0);
        mma_commit(&sm.bar_s);
    }

    float o[D];
#pragma unroll
    for (int c = 0; c < D; ++c) o[c] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool failed = false;

    for (int j = 0; j < n_kv; ++j) {
        const int stage = j & 1;
        const int k0 = j * BN;
        const bool ok_s = mbar_wait(&sm.bar_s, j & 1);
        if (__syncthreads_or(!ok_s)) {
            failed = true;
            break;
        }
        tc_fence_after();
        const bool need_mask = (p.causal && k0 + BN - 1 > q0) || k0 + BN > p.T;

        // Pass 1: tile row max.
        float sv[32];
        float tmax = -INFINITY;
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
            tmem_ld32(lane_base + tm + COL_S + c, sv);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int col = k0 + c + i;
                if (need_mask && ((p.causal && col > row) || col >= p.T)) sv[i] = -INFINITY;
                tmax = fmaxf(tmax, sv[i]);
            }
        }
        const float mn = fmaxf(m, tmax);
        const float ms = (mn == -INFINITY) ? 0.f : mn;
        const float alpha = ex2(m - ms);
        m = mn;

        // Pass 2: probabilities -> TMEM as bf16 hi / lo.
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
            tmem_ld32(lane_base + tm + COL_S + c, sv);
            tmem_wait_ld();
            uint32_t ph[16], pl[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                float e0 = ex2(sv[i] - ms), e1 = ex2(sv[i + 1] - ms);
                if (need_mask) {
                    const int col = k0 + c + i;
                    if ((p.causal && col > row) || col >= p.T) e0 = 0.f;
                    if ((p.causal && col + 1 > row) || col + 1 >= p.T) e1 = 0.f;
                }
                rs += e0 + e1;
                split2(e0, e1, ph[i / 2], pl[i / 2]);
            }
            tmem_st16(lane_base + tm + COL_PH + c / 2, ph);
            tmem_st16(lane_base + tm + COL_PL + c / 2, pl);
        }
        l = l * alpha + rs;
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();

        if (tid == 0) {
            tc_fence_after();
            issue_pv(sm, tm, stage);
            mma_commit(&sm.bar_o);
            if (j + 1 < n_kv) {
                issue_s(sm, tm, stage ^ 1);
                mma_commit(&sm.bar_s);
            }
        }
        const bool ok_o = mbar_wait(&sm.bar_o, j & 1);
        if (__syncthreads_or(!ok_o)) {
            failed = true;
            break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D; c += 32) {
            tmem_ld32(lane_base + tm + COL_O + c, sv);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[c + i] = fmaf(o[c + i], alpha, sv[i]);
        }
        // Key / value tile j+2 into the stage that tile j used (its MMAs are done).
        if (j + 2 < n_kv) {
            tc::stage_rows<BN, NT>(sm.kh[stage], sm.kl[stage], kg, p.ld_qkv, (j + 2) * BN, p.T, 1.f, tid);
            tc::stage_rows<BN, NT>(sm.vh[stage], sm.vl[stage], vg, p.ld_qkv, (j + 2) * BN, p.T, 1.f, tid);
            fence_async_smem();
        }
    }

    if (failed) {
        if (tid == 0) atomicOr(p.status, 1);
        // Let any MMA still in flight drain (bounded) before the columns are freed.
        if (tid == 0) {
            mma_commit(&sm.bar_o);
        }
        mbar_wait(&sm.bar_o, 0, 10000000ull);
        mbar_wait(&sm.bar_o, 1, 10000000ull);
    } else {
        // Normalise and stage O through shared memory (reusing the Q tiles,
        // float4 chunks XOR-swizzled by row) for coalesced global stores.
        const float inv = 1.f / l;
        float4* stg = reinterpret_cast<float4*>(sm.qh);  // 128 rows x 16 float4 = 32 KB (qh + ql)
        __syncthreads();
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4)
            stg[tid * 16 + (c4 ^ (tid & 15))] =
                make_float4(o[4 * c4] * inv, o[4 * c4 + 1] * inv, o[4 * c4 + 2] * inv, o[4 * c4 + 3] * inv);
        if (row < p.T) p.lse[(static_cast<long>(b) * p.H + h) * p.T + row] = (m + log2f(l)) * kLn2;
        __syncthreads();
        float* og = p.o + base * p.ld_o + h * D;
#pragma unroll
        for (int it = 0; it < 16; ++it) {
            const int i = tid + it * NT;
            const int r = i >> 4;
            const int c4 = i & 15;
            if (q0 + r < p.T)
                *reinterpret_cast<float4*>(og + static_cast<long>(q0 + r) * p.ld_o + c4 * 4) =
                    stg[r * 16 + (c4 ^ (r & 15))];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, TMEM_COLS);
}

}  // namespace

bool fwd_tc_supported(const FwdArgs& a) { return a.d == 64; }

cudaError_t launch_fwd_tc(const FwdArgs& a, int* status, cudaStream_t stream, int* launches) {
    Params p;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.ld_qkv = a.ld_qkv;
    p.o = a.o;
    p.ld_o = a.ld_o;
    p.lse = a.lse;
    p.status = status;
    p.B = a.B;
    p.T = a.T;
    p.H = a.H;
    p.scale_log2 = a.scale * kLog2e;
    p.causal = a.causal;
    p.n_qtiles = (a.T + BM - 1) / BM;
    p.n_ktiles = (a.T + BN - 1) / BN;
    const size_t smem = sizeof(Smem) + 1024;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_done{0};  // one bit per device: the attribute is per device
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(attn_fwd_tc64, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    const long nblocks = static_cast<long>(p.n_qtiles) * a.B * a.H;
    attn_fwd_tc64<<<static_cast<unsigned>(nblocks), NT, smem, stream>>>(p);
    e = cudaGetLastError();
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
