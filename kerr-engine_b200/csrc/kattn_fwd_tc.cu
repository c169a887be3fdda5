// Causal self-attention forward on the 5th-generation tensor cores (sm_100a),
// head_dim 64.  Replaces the scalar head loop of src/pipeline.rs:305-347.
//
// Numerics: every f32 operand x is split into bf16 hi = bf16(x) and
// lo = bf16(x - hi); each product A*B is formed as hi*hi + hi*lo + lo*hi with
// f32 accumulation in tensor memory (relative error ~1e-5, inside the 1e-4
// forward tolerance; a single bf16 or tf32 product is not).
//
// Work item = 128 query rows of one (batch, head) slab.  The kernel is
// persistent: two CTAs of 128 threads per SM, CTA c taking items c, 2G-1-c,
// 2G+c, ... of the list ordered longest first (a snake order: at the 768-dim
// shape 192 CTAs run one long item, 88 run two short ones).  Thread t owns
// query row t (TMEM lane t).  Per 64-row key tile j:
//   S_j = Q K_j^T        tcgen05.mma SS, M=128 N=64, 3 x 4 k-steps -> TMEM buffer g&1
//   softmax (online, log2 domain) in registers; P_j hi/lo written over S_j
//   O_j = P_j V_j        tcgen05.mma TS (P from TMEM), V MN-major  -> TMEM buffer g&1
//   O <- O * alpha + O_j in registers, one tile later
// PV_j and S_{j+1} are issued together; while they run the threads fold in
// O_{j-1} and stage K_{j+2} and V_{j+1} (K and V tiles have separate
// lifetimes: K_j is free once S_j is done, V_j once PV_j is).  g counts the
// CTA's tiles across its items (buffers, stages and barrier phases).  ~99 KB
// of shared memory and 256 TMEM columns per CTA: two CTAs share an SM.
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

// TMEM columns.  Buffer b: S at col_s(b) (64 f32 columns; P packed over it:
// for key columns 32c..32c+31, bf16 hi in columns 32c..32c+15 and lo in
// 32c+16..32c+31), the P V tile at col_o(b) (64 f32 columns).
__device__ __forceinline__ uint32_t col_s(int b) { return b ? 64u : 0u; }
__device__ __forceinline__ uint32_t col_o(int b) { return b ? 192u : 128u; }
constexpr uint32_t TMEM_COLS = 256;

struct alignas(1024) Smem {
    uint8_t qh[BM * 128];  // [128 rows][64 bf16], 128B swizzle
    uint8_t ql[BM * 128];
    uint8_t kh[2][BN * 128];
    uint8_t kl[2][BN * 128];
    uint8_t vh[2][BN * 128];
    uint8_t vl[2][BN * 128];
    uint64_t bar_s[2];
    uint64_t bar_o[2];
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
    int n_work;  // items: n_qtiles * B * H
};

// Shared-memory descriptors of the Q tile and of K / V stage 0 (stage 1 is
// STAGE_BYTES further), built once by the issuing thread.
constexpr uint32_t STAGE_BYTES = BN * 128;
struct Descs {
    uint64_t qh, ql, kh, kl, vh, vl;
};

__device__ __forceinline__ Descs make_descs(const Smem& sm) {
    Descs d;
    d.qh = smem_desc(smem_u32(sm.qh), 16, 1024);
    d.ql = smem_desc(smem_u32(sm.ql), 16, 1024);
    d.kh = smem_desc(smem_u32(sm.kh[0]), 16, 1024);
    d.kl = smem_desc(smem_u32(sm.kl[0]), 16, 1024);
    d.vh = smem_desc(smem_u32(sm.vh[0]), BN * 128, 1024);  // MN-major (P V B operand)
    d.vl = smem_desc(smem_u32(sm.vl[0]), BN * 128, 1024);
    return d;
}

// S = Q K^T of the key tile in stage `stage` into TMEM buffer b.
__device__ __forceinline__ void issue_s(const Descs& d, uint32_t tm, int stage, int b) {
    constexpr uint32_t idesc = idesc_bf16(BM, BN, 0, 0);
    const uint32_t so = stage * STAGE_BYTES;
    const uint64_t kh = desc_add(d.kh, so), kl = desc_add(d.kl, so);
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
        const uint32_t o = s * 32;
        mma_ss(tm + col_s(b), desc_add(d.qh, o), desc_add(kh, o), idesc, s > 0);
        mma_ss(tm + col_s(b), desc_add(d.qh, o), desc_add(kl, o), idesc, 1);
        mma_ss(tm + col_s(b), desc_add(d.ql, o), desc_add(kh, o), idesc, 1);
    }
}

// O_tile = P V of the key tile in stage `stage`, P packed over S buffer b.
__device__ __forceinline__ void issue_pv(const Descs& d, uint32_t tm, int stage, int b) {
    constexpr uint32_t idesc = idesc_bf16(BM, D, 0, 1);
    const uint32_t so = stage * STAGE_BYTES;
    const uint64_t vh = desc_add(d.vh, so), vl = desc_add(d.vl, so);
#pragma unroll
    for (int s = 0; s < BN / 16; ++s) {
        const uint32_t o = s * 2048;
        const uint32_t ph = tm + col_s(b) + 32 * (s >> 1) + 8 * (s & 1);
        mma_ts(tm + col_o(b), ph, desc_add(vh, o), idesc, s > 0);
        mma_ts(tm + col_o(b), ph, desc_add(vl, o), idesc, 1);
        mma_ts(tm + col_o(b), ph + 16, desc_add(vh, o), idesc, 1);
    }
}

__global__ void __launch_bounds__(NT, 2) attn_fwd_tc64(const Params p) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int nslab = p.B * p.H;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int cta = static_cast<int>(blockIdx.x);
    const int G = static_cast<int>(gridDim.x);

    if (warp == 0) {
        tmem_alloc(&sm.tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.bar_s[i], 1);
            mbar_init(&sm.bar_o[i], 1);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sm.tmem_slot;
    Descs dsc;
    if (tid == 0) dsc = make_descs(sm);
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    bool failed = false;
    int g = 0;  // the CTA's tile sequence number: TMEM buffer and K / V stage g&1, barrier phases

    for (int r = 0; !failed; ++r) {
    // Item r of this CTA in the snake order over the items (longest first).
    const int w = r * G + ((r & 1) ? G - 1 - cta : cta);
    if (w >= p.n_work) break;
    const int qt = p.n_qtiles - 1 - w / nslab;
    const int slab = w % nslab;
    const int b = slab / p.H;
    const int h = slab % p.H;
    const int q0 = qt * BM;
    const int row = q0 + tid;
    const int n_kv = p.causal ? min(p.n_ktiles, (q0 + BM + BN - 1) / BN) : p.n_ktiles;

    const long base = static_cast<long>(b) * p.T;
    const float* qg = p.q + base * p.ld_qkv + h * D;
    const float* kg = p.k + base * p.ld_qkv + h * D;
    const float* vg = p.v + base * p.ld_qkv + h * D;
    const int g0 = g;

    // Every stage and buffer is free: the previous item's last P V is done.
    tc::stage_rows2<BN, NT>(sm.kh[g0 & 1], sm.kl[g0 & 1], kg, p.ld_qkv, sm.vh[g0 & 1], sm.vl[g0 & 1], vg, p.ld_qkv, 0,
                            p.T, tid);
    tc::stage_rows<BM, NT>(sm.qh, sm.ql, qg, p.ld_qkv, q0, p.T, p.scale_log2, tid);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
        issue_s(dsc, tm, g0 & 1, g0 & 1);
        mma_commit(&sm.bar_s[g0 & 1]);
    }
    if (n_kv > 1) tc::stage_rows<BN, NT>(sm.kh[(g0 + 1) & 1], sm.kl[(g0 + 1) & 1], kg, p.ld_qkv, BN, p.T, 1.f, tid);
    fence_async_smem();

    float o[D];
#pragma unroll
    for (int c = 0; c < D; ++c) o[c] = 0.f;
    float m = -INFINITY, l = 0.f;
    float alpha_prev = 1.f;  // rescale factor of the tile whose P V is still pending

    // O <- O * alpha + (P V tile in buffer b).
    auto fold = [&](int b, float alpha) {
        float sv[32];
#pragma unroll
        for (int c = 0; c < D; c += 32) {
            tmem_ld32(lane_base + tm + col_o(b) + c, sv);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[c + i] = fmaf(o[c + i], alpha, sv[i]);
        }
    };

    for (int j = 0; j < n_kv; ++j, ++g) {
        const int bf = g & 1;  // TMEM buffer / smem stage of tile j
        const int k0 = j * BN;
        const bool ok_s = mbar_wait(&sm.bar_s[bf], (g >> 1) & 1);
        if (__syncthreads_or(!ok_s)) {
            failed = true;
            break;
        }
        tc_fence_after();
        const bool need_mask = (p.causal && k0 + BN - 1 > q0) || k0 + BN > p.T;

        // Tile row max over the 64 scores (masked columns to -inf), eight
        // independent chains.  Columns >= nv of this row are masked.
        float sv[BN];
        tmem_ld32(lane_base + tm + col_s(bf), *reinterpret_cast<float(*)[32]>(&sv[0]));
        tmem_ld32(lane_base + tm + col_s(bf) + 32, *reinterpret_cast<float(*)[32]>(&sv[32]));
        tmem_wait_ld();
        if (need_mask) {
            const int nv = min(p.T - k0, p.causal ? row - k0 + 1 : BN);
#pragma unroll
            for (int i = 0; i < BN; ++i) sv[i] = (i < nv) ? sv[i] : -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mx[u] = fmaxf(sv[u], sv[u + 8]);
#pragma unroll
        for (int i = 16; i < BN; i += 8)
#pragma unroll
            for (int u = 0; u < 8; ++u) mx[u] = fmaxf(mx[u], sv[i + u]);
        const float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        const float mn = fmaxf(m, tmax);
        const float ms = (mn == -INFINITY) ? 0.f : mn;
        const float alpha = ex2(m - ms);
        m = mn;

        // Probabilities, packed bf16 hi / lo over the S columns just read.
        float acc8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc8[u] = 0.f;
#pragma unroll
        for (int c = 0; c < BN; c += 32) {
            uint32_t ph[16], pl[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const float e0 = ex2(sv[c + i] - ms), e1 = ex2(sv[c + i + 1] - ms);
                acc8[(i >> 1) & 7] += e0 + e1;
                split2(e0, e1, ph[i / 2], pl[i / 2]);
            }
            tmem_st16(lane_base + tm + col_s(bf) + c, ph);
            tmem_st16(lane_base + tm + col_s(bf) + c + 16, pl);
        }
        const float rs = ((acc8[0] + acc8[1]) + (acc8[2] + acc8[3])) + ((acc8[4] + acc8[5]) + (acc8[6] + acc8[7]));
        l = l * alpha + rs;
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();

        if (tid == 0) {
            tc_fence_after();
            issue_pv(dsc, tm, bf, bf);
            mma_commit(&sm.bar_o[bf]);
            if (j + 1 < n_kv) {
                issue_s(dsc, tm, bf ^ 1, bf ^ 1);
                mma_commit(&sm.bar_s[bf ^ 1]);
            }
        }
        if (j >= 1) {
            // Fold in the previous tile's P V (its buffer is the other one).
            const bool ok_o = mbar_wait(&sm.bar_o[bf ^ 1], ((g - 1) >> 1) & 1);
            if (__syncthreads_or(!ok_o)) {
                failed = true;
                break;
            }
            tc_fence_after();
            fold(bf ^ 1, alpha_prev);
        }
        alpha_prev = alpha;
        // K_{j+2} into this tile's K stage (S_j is done); V_{j+1} into the
        // other V stage (PV_{j-1} is done).  Both become visible to the tensor
        // core at the next iteration's barrier.
        const bool kn = j + 2 < n_kv, vn = j + 1 < n_kv && j >= 1;
        if (kn) tc::stage_rows<BN, NT>(sm.kh[bf], sm.kl[bf], kg, p.ld_qkv, (j + 2) * BN, p.T, 1.f, tid);
        if (vn) tc::stage_rows<BN, NT>(sm.vh[bf ^ 1], sm.vl[bf ^ 1], vg, p.ld_qkv, (j + 1) * BN, p.T, 1.f, tid);
        if (j == 0 && n_kv > 1) tc::stage_rows<BN, NT>(sm.vh[bf ^ 1], sm.vl[bf ^ 1], vg, p.ld_qkv, BN, p.T, 1.f, tid);
        if (kn || vn || j == 0) fence_async_smem();
    }

    if (!failed) {
        const int gl = g - 1;
        const bool ok_o = mbar_wait(&sm.bar_o[gl & 1], (gl >> 1) & 1);
        if (__syncthreads_or(!ok_o)) {
            failed = true;
        } else {
            tc_fence_after();
            fold(gl & 1, alpha_prev);
        }
    }

    if (failed) break;
    // Normalise and stage O through shared memory (reusing the Q tiles,
    // float4 chunks XOR-swizzled by row) for coalesced global stores.
    {
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
            const int rr = i >> 4;
            const int c4 = i & 15;
            if (q0 + rr < p.T)
                *reinterpret_cast<float4*>(og + static_cast<long>(q0 + rr) * p.ld_o + c4 * 4) =
                    stg[rr * 16 + (c4 ^ (rr & 15))];
        }
    }
    // The next item stages its Q over the rows just read, and its MMAs reuse
    // the TMEM buffers this item's threads have read.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    }

    if (failed) {
        if (tid == 0) atomicOr(p.status, 1);
        // Let any MMA still in flight drain (bounded) before the columns are freed.
        if (tid == 0) mma_commit(&sm.bar_s[0]);
        mbar_wait(&sm.bar_s[0], 0, 10000000ull);
        mbar_wait(&sm.bar_s[0], 1, 10000000ull);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, TMEM_COLS);
}

}  // namespace

bool fwd_tc_supported(const FwdArgs& a) { return a.d == 64; }

cudaError_t launch_fwd_tc(const FwdArgs& a, int num_sms, int* status, cudaStream_t stream, int* launches) {
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
    const long n_work = static_cast<long>(p.n_qtiles) * a.B * a.H;
    if (n_work <= 0 || n_work > INT32_MAX) return cudaErrorInvalidValue;
    p.n_work = static_cast<int>(n_work);
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
    // Persistent: two CTAs per SM (shared memory and TMEM allow two), each
    // walking its items in the snake order.
    const long slots = 2L * (num_sms > 0 ? num_sms : 148);
    const int grid = static_cast<int>(n_work < slots ? n_work : slots);
    e = launch_pdl(attn_fwd_tc64, dim3(static_cast<unsigned>(grid)), dim3(NT), smem, stream, p);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
