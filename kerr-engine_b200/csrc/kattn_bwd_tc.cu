// Causal self-attention backward on the 5th-generation tensor cores
// (sm_100a), head_dim 64 and 32 (one kernel body, templated on the head
// dimension D; the notes below give the D = 64 sizes).  Replaces
// ComputeBackend::attention_backward
// (src/backend.rs:223-231; CPU src/backward.rs:464-514; WGSL
// attn_backward_scores / attn_backward_dkv), recomputing the probabilities
// from the forward's log-sum-exp instead of reading a cached [H][T][T] P.
//
// Work item = one 128-row key tile of one (batch, head) slab: K, V and the
// dK, dV accumulators stay resident while the item walks the 64-row query
// tiles on or below the diagonal.  The kernel is persistent (one CTA per SM):
// CTA c takes items c, 2G-1-c, 2G+c, ... of the list ordered longest first
// (a snake order, which evens out the tile counts per CTA), and its query
// tiles form one pipeline across item boundaries.  Products (bf16x3: hi*hi + hi*lo + lo*hi, f32 accumulation):
//   S^T  = K Q^T      M=128 (keys) N=64 (queries)   SS, both K-major
//   dP^T = V dO^T     M=128 N=64                    SS, both K-major
//   P = exp2(S^T * scale*log2e - lse*log2e),  dS = P * (dP^T - D)   (threads)
//   dV  += P^T dO     M=128 N=64 K=64    TS: P from TMEM, dO MN-major
//   dK  += dS^T Q     M=128 N=64 K=64    TS: dS from TMEM, Q MN-major
//   dQ_i = dS K       M=128 N=64 K=128   SS: stacked dS (below), K MN-major;
//                     added into global dq with vector reductions.
// The dQ product's A operand stacks dS hi and lo as 128 rows, so two MMAs
// per 16 keys (times K hi, times K lo) form every term of the split product:
// stacked row 32*qd + l (l < 16) is dS_hi of query 16*qd + l and row
// 32*qd + 16 + l its dS_lo, so both parts of a query's dQ land in one warp's
// TMEM lane quadrant and a shuffle adds them.  In shared memory the rows are
// MN-major atoms: sh[b] holds stacked rows 0-63 (queries 0-31), sl[b] rows
// 64-127 (queries 32-63), each [key][64 bf16], 128B-swizzled.
// D = rowsum(dO * O) and the zeroed dq come from attn_bwd_rowdot.
//
// Warp roles (416 threads, one CTA per SM):
//   warps 0-7   elementwise.  Warp w reads TMEM lanes 32*(w%4).. (key rows)
//               and query columns 32*(w/4)..+31 of each 64-column tile; at
//               the end of an item it stores its half of the dK / dV rows.
//               They also stage K / V: the next item's rows are loaded into
//               registers at the end of an item and written to shared memory
//               as soon as the item's last dQ product (the last reader of K)
//               is done, while the tensor core still runs its dV / dK.
//   warps 8-11  loaders: Q, dO, lse, D per query tile into a 3-stage ring;
//               they also add each finished dQ tile into dq (reductions), so
//               that wait stays off the elementwise warps.
//   warp 12     one lane issues every tcgen05.mma and commit, from
//               descriptors built once, in whichever order its inputs become
//               ready (a tile's S^T / dP^T as soon as the tile is loaded and
//               its TMEM buffer is free; a tile's gradients as soon as its P
//               and dS are written).
// Everything a query tile touches is double-buffered (S^T / dP^T in TMEM,
// the stacked dS in shared memory, the dQ accumulator in TMEM), so the tensor core runs
// tile i's gradient products while the elementwise warps work on tile i+1.
// P and dS are packed over their own S^T / dP^T columns: for query columns
// 16c..16c+15, bf16 hi goes to columns 16c..16c+7 and lo to 16c+8..16c+15,
// which the owning warp has already read; the tensor core runs one thread's
// MMAs in issue order, so the next S^T lands only after dV / dK read them.
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
constexpr int NELEM = 256;  // elementwise threads (warps 0-7)
constexpr int NLOAD = 128;  // loader threads (warps 8-11)
constexpr int NTHREADS = NELEM + NLOAD + 32;
constexpr int MMA_WARP = (NELEM + NLOAD) / 32;
constexpr int STAGES = 3;  // query-tile ring depth (Q, dO, lse, D)
static_assert(BK == kBwdTcKeyRows, "dQ slices of the deterministic mode");

// TMEM columns (512 allocated).  Buffer b: S^T (then P packed) at col_s(b),
// dP^T (then dS packed) at col_dp(b), dQ tile (the stacked M=128 accumulator) at col_dq(b).
__device__ __forceinline__ uint32_t col_s(int b) { return b ? 128u : 0u; }
__device__ __forceinline__ uint32_t col_dp(int b) { return b ? 192u : 64u; }
__device__ __forceinline__ uint32_t col_dq(int b) { return b ? 320u : 256u; }
constexpr uint32_t COL_DV = 384;
constexpr uint32_t COL_DK = 448;
constexpr uint32_t TMEM_COLS = 512;

// Head dimension D = 64 or 32: K, V, Q and dO rows are D bf16 (2D bytes),
// 128B-swizzled at D = 64 and 64B-swizzled at D = 32.
template <int D>
struct BCfg {
    static_assert(D == 64 || D == 32, "head_dim 64 or 32");
    static constexpr uint32_t ROW = 2 * D;              // bytes of a bf16 row
    static constexpr uint32_t STAGE_BYTES = BQ * ROW;   // one stage of one Q / dO tile
};

template <int D>
struct alignas(1024) Smem {
    uint8_t kh[BK * 2 * D];  // [key][D bf16]
    uint8_t kl[BK * 2 * D];
    uint8_t vh[BK * 2 * D];
    uint8_t vl[BK * 2 * D];
    uint8_t qh[STAGES][BQ * 2 * D];  // [query][D bf16]
    uint8_t ql[STAGES][BQ * 2 * D];
    uint8_t gh[STAGES][BQ * 2 * D];  // dO
    uint8_t gl[STAGES][BQ * 2 * D];
    uint8_t sh[2][BK * 128];  // stacked dS, rows 0-63, [key][64], per TMEM buffer
    uint8_t sl[2][BK * 128];  // stacked dS, rows 64-127
    float lse2[STAGES][BQ];  // lse * log2(e), +inf beyond T
    float dsum[STAGES][BQ];  // D, 0 beyond T
    uint64_t kv_full;  // an item's K / V staged (phase r: the CTA's item r)
    uint64_t kv_free;  // an item's last dQ product done: K / V may be replaced
    uint64_t full[STAGES];
    uint64_t bar_s[2];
    uint64_t pds[2];      // P / dS of the tile in buffer b written
    uint64_t bar_d[2];    // gradient products of the tile in buffer b done
    uint64_t dq_free[2];  // dQ accumulator b read out by the loaders
    uint64_t stg_full;    // dK / dV staging written (phase r: item r)
    uint64_t stg_done;    // dK / dV staging stored to global
    uint32_t tmem_slot;
};

static_assert(sizeof(Smem<64>) + 1024 <= 232448, "shared memory (plus alignment slack) exceeds 227 KB");

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
    float* dq_part;  // deterministic mode: [key tiles][B*T][H*64] slices, or null
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
    int n_work;    // work items: n_ktiles * B * H
    unsigned long long wait_ns;  // wall-time limit of every bounded wait
};

// The r-th work item of CTA c in a grid of G: the snake order over the item
// list (key tile 0 of every slab first: it sees the most query tiles).
__device__ __forceinline__ int item_id(int c, int r, int G) { return r * G + ((r & 1) ? G - 1 - c : c); }

// A work item: key tile jt of slab (b, h).
struct Item {
    int b, h, k0, it0, n_it;
};

__device__ __forceinline__ Item make_item(const Params& p, int w) {
    const int nslab = p.B * p.H;
    const int jt = w / nslab;
    const int slab = w - jt * nslab;
    Item it;
    it.b = slab / p.H;
    it.h = slab - it.b * p.H;
    it.k0 = jt * BK;
    it.it0 = p.causal ? it.k0 / BQ : 0;  // first query tile with a row >= k0
    it.n_it = p.n_qtiles - it.it0;
    return it;
}

// Position in a CTA's sequence of query tiles: item round r (item id w, -1
// past the last), tile n of the item's n_it.
struct Cursor {
    int r, w, n, n_it, it0;
    __device__ __forceinline__ void set(const Params& p, int c, int G) {
        w = item_id(c, r, G);
        n = 0;
        if (w < p.n_work) {
            const Item it = make_item(p, w);
            n_it = it.n_it;
            it0 = it.it0;
        } else {
            w = -1;
        }
    }
    __device__ __forceinline__ void start(const Params& p, int c, int G) {
        r = 0;
        set(p, c, G);
    }
    __device__ __forceinline__ void next(const Params& p, int c, int G) {
        if (++n == n_it) {
            ++r;
            set(p, c, G);
        }
    }
    __device__ __forceinline__ bool valid() const { return w >= 0; }
};

// Shared-memory descriptors, built once by the issuing thread (two ring
// stages / two buffers, selected without indexing so they stay in registers).
// A K-major k-step advances 32 bytes inside the swizzled row; an MN-major
// k-step advances 16 rows (2048 bytes).  The K-major and MN-major
// descriptors of one tile differ only in the leading-byte offset.
struct Descs {
    uint64_t kh, kl, vh, vl;      // K / V, K-major (S^T, dP^T A operands)
    uint64_t kh_mn, kl_mn;        // K, MN-major (dQ B operand)
    uint64_t qh, ql, gh, gl;      // Q / dO ring stage 0, K-major; stage s is STAGE_BYTES * s further
    uint64_t s0, s1;              // stacked dS hi / lo of buffer 0 / 1, MN-major (dQ A, M=128)
};

constexpr uint32_t MN_LBO_Q = BQ * 128;     // leading-byte offset of a 64-row MN-major tile (one N atom: unused)
constexpr uint32_t MN_LBO_K = BK * 128;
// The dQ product's A operand (M=128) is two 64-row MN-major atoms: sh[b]
// (atom 0) and sl[b] (atom 1), this far apart.
constexpr uint32_t DQ_A_LBO = 2 * BK * 128;

__device__ __forceinline__ uint64_t as_mn(uint64_t kdesc, uint32_t lbo) {
    return (kdesc & ~(static_cast<uint64_t>(0x3FFFu) << 16)) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16);
}

// A K-major descriptor of rows of D bf16: 128B-swizzled at D = 64, 64B-swizzled
// (8-row atoms of 512 bytes) at D = 32.  The MN-major uses of these tiles
// have N = D, one swizzle atom, so their leading-byte offset is unused.
template <int D>
__device__ __forceinline__ uint64_t row_desc(uint32_t addr) {
    if constexpr (D == 64) return smem_desc(addr, 16, 1024);
    else return smem_desc_sw64(addr, 512);
}

template <int D>
__device__ __forceinline__ void make_descs(const Smem<D>& sm, Descs& d) {
    d.kh = row_desc<D>(smem_u32(sm.kh));
    d.kl = row_desc<D>(smem_u32(sm.kl));
    d.vh = row_desc<D>(smem_u32(sm.vh));
    d.vl = row_desc<D>(smem_u32(sm.vl));
    d.kh_mn = as_mn(d.kh, MN_LBO_K);
    d.kl_mn = as_mn(d.kl, MN_LBO_K);
    d.qh = row_desc<D>(smem_u32(sm.qh[0]));
    d.ql = row_desc<D>(smem_u32(sm.ql[0]));
    d.gh = row_desc<D>(smem_u32(sm.gh[0]));
    d.gl = row_desc<D>(smem_u32(sm.gl[0]));
    d.s0 = smem_desc(smem_u32(sm.sh[0]), DQ_A_LBO, 1024);
    d.s1 = smem_desc(smem_u32(sm.sh[1]), DQ_A_LBO, 1024);
}

// S^T and dP^T of the query tile in ring stage s into TMEM buffer b.
template <int D>
__device__ __forceinline__ void issue_sdp(const Descs& d, uint32_t tm, int s, int b) {
    constexpr uint32_t idesc = idesc_bf16(BK, BQ, 0, 0);
    const uint32_t cs = tm + col_s(b), cp = tm + col_dp(b);
    const uint32_t so = s * BCfg<D>::STAGE_BYTES;
    const uint64_t qh = desc_add(d.qh, so), ql = desc_add(d.ql, so);
    const uint64_t gh = desc_add(d.gh, so), gl = desc_add(d.gl, so);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
        const uint32_t o = ks * 32;
        mma_ss(cs, desc_add(d.kh, o), desc_add(qh, o), idesc, ks > 0);
        mma_ss(cs, desc_add(d.kh, o), desc_add(ql, o), idesc, 1);
        mma_ss(cs, desc_add(d.kl, o), desc_add(qh, o), idesc, 1);
        mma_ss(cp, desc_add(d.vh, o), desc_add(gh, o), idesc, ks > 0);
        mma_ss(cp, desc_add(d.vh, o), desc_add(gl, o), idesc, 1);
        mma_ss(cp, desc_add(d.vl, o), desc_add(gh, o), idesc, 1);
    }
}

// dQ_b = dS K as one M=128 product per K half: A stacks dS hi and lo (128
// rows, see the header), so [dS_hi; dS_lo] (K_hi + K_lo) accumulates
// dS_hi K and dS_lo K in separate TMEM lanes, which the read-out adds.  Two
// M=128 MMAs per 16 keys instead of three M=64 ones, at the same cost per
// MMA; the extra lo*lo term only adds precision.
template <int D>
__device__ __forceinline__ void issue_dq(const Descs& d, uint32_t tm, int b) {
    constexpr uint32_t idesc_q = idesc_bf16(2 * BQ, D, 1, 1);
    const uint32_t cq = tm + col_dq(b);
    const uint64_t sa = b ? d.s1 : d.s0;
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
        const uint32_t os = ks * 2048;                   // 16 keys of the stacked dS (128-byte rows)
        const uint32_t ok = ks * 16 * BCfg<D>::ROW;      // 16 keys of K
        mma_ss(cq, desc_add(sa, os), desc_add(d.kh_mn, ok), idesc_q, ks > 0);
        mma_ss(cq, desc_add(sa, os), desc_add(d.kl_mn, ok), idesc_q, 1);
    }
}

// dV += P^T dO, dK += dS^T Q (P, dS from TMEM buffer b; dO, Q of ring stage s).
template <int D>
__device__ __forceinline__ void issue_dkv(const Descs& d, uint32_t tm, int s, int b, bool first) {
    constexpr uint32_t idesc_kv = idesc_bf16(BK, D, 0, 1);
    const uint32_t so = s * BCfg<D>::STAGE_BYTES;
    const uint64_t qh = as_mn(desc_add(d.qh, so), MN_LBO_Q), ql = as_mn(desc_add(d.ql, so), MN_LBO_Q);
    const uint64_t gh = as_mn(desc_add(d.gh, so), MN_LBO_Q), gl = as_mn(desc_add(d.gl, so), MN_LBO_Q);
#pragma unroll
    for (int ks = 0; ks < BQ / 16; ++ks) {
        const uint32_t acc = (first && ks == 0) ? 0u : 1u;
        const uint32_t o = ks * 16 * BCfg<D>::ROW;  // 16 queries
        const uint32_t ph = tm + col_s(b) + 16 * ks, gph = tm + col_dp(b) + 16 * ks;  // hi; lo is 8 further
        mma_ts(tm + COL_DV, ph, desc_add(gh, o), idesc_kv, acc);
        mma_ts(tm + COL_DV, ph, desc_add(gl, o), idesc_kv, 1);
        mma_ts(tm + COL_DV, ph + 8, desc_add(gh, o), idesc_kv, 1);
        mma_ts(tm + COL_DK, gph, desc_add(qh, o), idesc_kv, acc);
        mma_ts(tm + COL_DK, gph, desc_add(ql, o), idesc_kv, 1);
        mma_ts(tm + COL_DK, gph + 8, desc_add(qh, o), idesc_kv, 1);
    }
}

// A dQ tile (the stacked M=128 accumulator: query row 16*qd + l has its
// dS_hi K part in lane 32*qd + l and its dS_lo K part in lane 32*qd + 16 + l,
// l < 16), scaled and added into dq by the loader warp of lane quadrant qd,
// 32 columns at a time.  Lanes l and l + 16 swap half of their columns, so
// lane l sums columns 0-15 of the 32 and lane l + 16 columns 16-31.
// The TMEM buffer is released on `dq_free` as soon as
// both halves are in registers, with a relaxed arrive: a release arrive
// would wait for this thread's outstanding global operations (the first
// half's reductions, the next tile's prefetch loads), and the next gradient
// products wait for this buffer.
template <bool DET, int D>
__device__ __forceinline__ void dq_epilogue(const Params& p, uint32_t tm, int b, int qd, int lane, int q0,
                                            float* dqg, long ldq, uint64_t* dq_free) {
    const uint32_t ta = (static_cast<uint32_t>(qd * 32) << 16) + tm + col_dq(b);
    const bool up = lane >= 16;  // sums columns 16-31 of each 32
    const int r = q0 + qd * 16 + (lane & 15);
    float* dst = dqg + static_cast<long>(r) * ldq + (up ? 16 : 0);
    const bool on = r < p.T;
#pragma unroll
    for (int h = 0; h < D / 32; ++h) {
        float v[32];
        tmem_ld32(ta + 32 * h, v);
        tmem_wait_ld();
        if (h == D / 32 - 1) {
            tc_fence_before();
            mbar_arrive_relaxed(dq_free);
        }
#pragma unroll
        for (int c = 0; c < 16; c += 4) {
            float x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float keep = up ? v[16 + c + u] : v[c + u];
                const float send = up ? v[c + u] : v[16 + c + u];
                x[u] = (keep + __shfl_xor_sync(0xffffffffu, send, 16)) * p.scale;
            }
            if (on) {
                if (DET)  // deterministic mode: this key tile's slice, summed in order later
                    *reinterpret_cast<float4*>(dst + 32 * h + c) = make_float4(x[0], x[1], x[2], x[3]);
                else
                    red_add_v4(dst + 32 * h + c, x[0], x[1], x[2], x[3]);
            }
        }
    }
}

// dK, dV of the CTA's item r -> global, by the elementwise warps.  Warp
// (qd, hf) reads its 32 key rows x 32 columns of each accumulator (TMEM loads
// are warp-collective and run on every lane) into the idle stacked-dS buffers, laid
// out [row][16 float4] with the float4 index XOR-swizzled by row; then the 256
// threads store whole 256-byte rows, two per warp instruction.  Rows past T
// are not stored.  Those buffers are free: the item's last dQ product has
// completed and the next item's tiles are written by these same warps after
// the second barrier.  The barriers are mbarriers with bounded waits, so a
// warp that gave up earlier cannot leave the others blocked.
template <int D>
__device__ __forceinline__ bool store_dkv(const Params& p, Smem<D>& sm, uint32_t tm, const Item& it, uint32_t lb,
                                          int row, int hf, int tid, int r) {
    constexpr int NCH = D / 4;  // float4 chunks of a row
    float4* stg_v = reinterpret_cast<float4*>(sm.sh[0]);  // BK rows x D floats (16 or 32 KB)
    float4* stg_k = reinterpret_cast<float4*>(sm.sl[0]);
    float a[32];
    if constexpr (D == 64) {
        tmem_ld32(lb + tm + COL_DV + 32 * hf, a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
            stg_v[row * 16 + ((8 * hf + i) ^ (row & 15))] = make_float4(a[4 * i], a[4 * i + 1], a[4 * i + 2], a[4 * i + 3]);
        tmem_ld32(lb + tm + COL_DK + 32 * hf, a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
            stg_k[row * 16 + ((8 * hf + i) ^ (row & 15))] =
                make_float4(a[4 * i] * p.scale, a[4 * i + 1] * p.scale, a[4 * i + 2] * p.scale, a[4 * i + 3] * p.scale);
    } else {
        // 32 columns per accumulator: the warps with hf = 0 take dV, hf = 1 dK.
        const float sc = hf ? p.scale : 1.f;
        float4* stg = hf ? stg_k : stg_v;
        tmem_ld32(lb + tm + (hf ? COL_DK : COL_DV), a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
            stg[row * 8 + (i ^ (row & 7))] = make_float4(a[4 * i] * sc, a[4 * i + 1] * sc, a[4 * i + 2] * sc, a[4 * i + 3] * sc);
    }
    mbar_arrive(&sm.stg_full);
    if (!mbar_wait_warp(&sm.stg_full, r & 1, p.wait_ns)) return false;
    const long row0 = static_cast<long>(it.b) * p.T + it.k0;
    float* dvg = p.dv + row0 * p.ld_d + it.h * D;
    float* dkg = p.dk + row0 * p.ld_d + it.h * D;
#pragma unroll
    for (int k = 0; k < BK * NCH / NELEM; ++k) {
        const int i = tid + k * NELEM;
        const int r = i / NCH;
        const int c4 = i % NCH;
        if (it.k0 + r < p.T) {
            const float4 v = stg_v[r * NCH + (c4 ^ (r & (NCH - 1)))];
            const float4 g = stg_k[r * NCH + (c4 ^ (r & (NCH - 1)))];
            *reinterpret_cast<float4*>(dvg + r * p.ld_d + c4 * 4) = v;
            *reinterpret_cast<float4*>(dkg + r * p.ld_d + c4 * 4) = g;
        }
    }
    mbar_arrive(&sm.stg_done);  // staging reads done before the next tile's dS writes
    return mbar_wait_warp(&sm.stg_done, r & 1, p.wait_ns);
}

// DET: the deterministic dQ mode (slices in p.dq_part instead of reductions into dq).
// V8: q, k, v, dout rows start on 32-byte boundaries (256-bit row loads).
template <bool DET, bool V8, int D>
__device__ __forceinline__ void bwd_body(const Params& p) {
    // Launched behind attn_bwd_rowdot, whose outputs (D, the zeroed dq) only
    // the loader warps touch: they wait for it; the elementwise warps stage
    // the first item's K / V meanwhile.  Those reads need no wait: rowdot
    // lets this grid launch only after its own griddepcontrol.wait, so every
    // grid before rowdot has finished by now.
    pdl_launch();
    extern __shared__ uint8_t smem_raw[];
    Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int c = static_cast<int>(blockIdx.x);
    const int G = static_cast<int>(gridDim.x);
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    if (warp == 0) {
        tmem_alloc(&sm.tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&sm.kv_full, NELEM);
        mbar_init(&sm.kv_free, 1);
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&sm.full[i], NLOAD);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.bar_s[i], 1);
            mbar_init(&sm.bar_d[i], 1);
            mbar_init(&sm.dq_free[i], NLOAD);
        }
        mbar_init(&sm.pds[0], NELEM);
        mbar_init(&sm.pds[1], NELEM);
        mbar_init(&sm.stg_full, NELEM);
        mbar_init(&sm.stg_done, NELEM);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sm.tmem_slot;
    bool failed = false;

    if (warp >= NELEM / 32 && warp < MMA_WARP) {
        // ------------------------------------------------------------ loaders
        // Step n writes the CTA's query tile n into its ring stage from
        // registers, issues the global loads of tile n+1 into registers, then
        // adds tile n-2's dQ into dq (gradient products finish in tile
        // order): the loads are in flight while the step waits for that dQ.
        pdl_wait();
        const int t = tid - NELEM;
        const int qd = warp & 3;
        Cursor cl, cq;  // tile to load, tile whose dQ is added
        cl.start(p, c, G);
        cq.start(p, c, G);
        tc::Rows2<BQ, NLOAD, D> x;
        float lse_t = 0.f, ds_t = 0.f;
        auto prefetch = [&]() {
            const Item it = make_item(p, cl.w);
            const long base = static_cast<long>(it.b) * p.T;
            const int q0 = (cl.it0 + cl.n) * BQ;
            x.template load<V8>(p.q + base * p.ld_qkv + it.h * D, p.ld_qkv, p.dout + base * p.ld_o + it.h * D,
                                p.ld_o, q0, p.T, t);
            if (t < BQ) {
                const long bh = (static_cast<long>(it.b) * p.H + it.h) * p.T;
                const bool ok = q0 + t < p.T;
                lse_t = ok ? p.lse[bh + q0 + t] * kLog2e : INFINITY;
                // D is read only after this warp's pdl_wait, and attn_bwd_rowdot
                // writes it only after its own griddepcontrol.wait: calls queued
                // on one stream may share one workspace array (kattn_bwd_noalloc).
                ds_t = ok ? p.dsum[bh + q0 + t] : 0.f;
            }
        };
        if (cl.valid()) prefetch();
        for (int n = 0; !failed; ++n) {
            if (cl.valid()) {
                // Stage s last held tile n - STAGES, whose gradient products
                // these warps saw complete (bar_d) before reading its dQ in
                // step n - 1, so the stage is free without another wait.
                static_assert(STAGES == 3, "tile n-3's dQ is read out in step n-1");
                const int s = n % STAGES;
                if (t < BQ) {
                    sm.lse2[s][t] = lse_t;
                    sm.dsum[s][t] = ds_t;
                }
                x.store(sm.qh[s], sm.ql[s], sm.gh[s], sm.gl[s], t);
                fence_async_smem();
                mbar_arrive(&sm.full[s]);
                cl.next(p, c, G);
                if (cl.valid()) prefetch();
            }
            if (n >= 2) {
                if (!cq.valid()) break;
                const int m = n - 2;
                if (!mbar_wait_warp(&sm.bar_d[m & 1], (m >> 1) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const Item it = make_item(p, cq.w);
                const long hd = static_cast<long>(p.H) * D;
                float* dqg = DET ? p.dq_part + (static_cast<long>(it.k0 / BK) * p.B + it.b) * p.T * hd + it.h * D
                                 : p.dq + static_cast<long>(it.b) * p.T * p.ld_d + it.h * D;
                dq_epilogue<DET, D>(p, tm, m & 1, qd, lane, (cq.it0 + cq.n) * BQ, dqg, DET ? hd : p.ld_d,
                            &sm.dq_free[m & 1]);
                cq.next(p, c, G);
            }
        }
    } else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            Descs d;
            make_descs(sm, d);
            // sdp(n) needs tile n loaded, for n >= 2 grads(n-2) issued (TMEM
            // buffer n&1; the tensor core runs this thread's MMAs in order)
            // and, for an item's first tile, the item's K / V staged.
            // grads(n) needs P / dS of tile n written and, for n >= 2, dQ
            // buffer n&1 read out.  An item's last dQ product commits kv_free.
            Cursor cs, cg;
            cs.start(p, c, G);
            cg.start(p, c, G);
            int ns = 0, ng = 0, kv_round = -1;
            uint64_t t_idle = 0;
            while (cg.valid() && !failed) {
                bool progressed = false;
                if (cs.valid() && ns < ng + 2) {
                    bool kv_ok = kv_round >= cs.r;
                    if (!kv_ok && mbar_test_wait(&sm.kv_full, cs.r & 1)) {
                        kv_round = cs.r;
                        kv_ok = true;
                    }
                    if (kv_ok && mbar_test_wait(&sm.full[ns % STAGES], (ns / STAGES) & 1)) {
                        tc_fence_after();
                        issue_sdp<D>(d, tm, ns % STAGES, ns & 1);
                        mma_commit(&sm.bar_s[ns & 1]);
                        ++ns;
                        cs.next(p, c, G);
                        progressed = true;
                    }
                }
                if (ng < ns && mbar_test_wait(&sm.pds[ng & 1], (ng >> 1) & 1) &&
                    (ng < 2 || mbar_test_wait(&sm.dq_free[ng & 1], ((ng - 2) >> 1) & 1))) {
                    tc_fence_after();
                    issue_dq<D>(d, tm, ng & 1);
                    if (cg.n == cg.n_it - 1) mma_commit(&sm.kv_free);
                    issue_dkv<D>(d, tm, ng % STAGES, ng & 1, cg.n == 0);
                    mma_commit(&sm.bar_d[ng & 1]);  // one commit: back-to-back commits stall the MMA pipe
                    ++ng;
                    cg.next(p, c, G);
                    progressed = true;
                }
                if (progressed) {
                    t_idle = 0;
                } else {
                    const uint64_t now = globaltimer_ns();
                    if (t_idle == 0) t_idle = now;
                    else if (now - t_idle > p.wait_ns) failed = true;
                    __nanosleep(20);
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ elementwise
        const int qd = warp & 3;          // TMEM lane quadrant: key rows 32*qd..
        const int hf = warp >> 2;         // query columns 32*hf..+31 (two 16-column chunks)
        const int row = qd * 32 + lane;   // key row inside the tile
        const uint32_t lb = static_cast<uint32_t>(qd * 32) << 16;
        // Offset from sh[0] of this thread's key row in the stacked-dS atom hf
        // of buffer 0 (sl[0] is 2*BK*128 bytes after sh[0]; buffer 1 is BK*128
        // bytes further).
        const uint32_t ds_off = (hf ? 2 * BK * 128 : 0) + row * 128;
        const uint32_t ds_sw = static_cast<uint32_t>(row & 7);
        int w = item_id(c, 0, G);
        Item it = make_item(p, w);
        {
            const long base = static_cast<long>(it.b) * p.T;
            tc::stage_rows2<BK, NELEM, V8, D>(sm.kh, sm.kl, p.k + base * p.ld_qkv + it.h * D, p.ld_qkv, sm.vh, sm.vl,
                                       p.v + base * p.ld_qkv + it.h * D, p.ld_qkv, it.k0, p.T, tid);
        }
        fence_async_smem();
        mbar_arrive(&sm.kv_full);

        int g = 0;  // the CTA's query-tile sequence number
        for (int r = 0; !failed; ++r) {
            const int j = it.k0 + row;
            for (int n = 0; n < it.n_it; ++n, ++g) {
                const int s = g % STAGES;  // ring stage of this query tile
                const int buf = g & 1;     // TMEM / dS buffer
                const int q0 = (it.it0 + n) * BQ;
                // full[s]: the loaders' lse / D writes for this tile are visible.
                if (!mbar_wait_warp(&sm.bar_s[buf], (g >> 1) & 1, p.wait_ns) ||
                    !mbar_wait_warp(&sm.full[s], (g / STAGES) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                if (g >= 2 && !mbar_wait_warp(&sm.bar_d[buf], ((g - 2) >> 1) & 1, p.wait_ns)) {
                    failed = true;  // dS buffer `buf` is read by tile g-2's dQ product
                    break;
                }
                tc_fence_after();
                const bool need_mask =
                    (p.causal && q0 < it.k0 + BK - 1) || q0 + BQ > p.T || it.k0 + BK > p.T;
                // Valid query columns of this key row in this warp's 32: bit i set when
                // query q0 + 32*hf + i attends to key j (causal: q >= j), both below T.
                uint32_t vmask = 0xffffffffu;
                if (need_mask) {
                    const int c0 = q0 + 32 * hf;
                    const int lo = p.causal ? max(0, j - c0) : 0;
                    const int hi = (j < p.T) ? min(32, p.T - c0) : 0;
                    vmask = (lo >= hi) ? 0u
                                       : ((hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u)) &
                                          ~((lo >= 32) ? 0xffffffffu : ((1u << lo) - 1u)));
                }
                const uint32_t cs = lb + tm + col_s(buf) + 32 * hf, cp = lb + tm + col_dp(buf) + 32 * hf;
                float sv[32], dp[32];
                tmem_ld32(cs, sv);
                tmem_ld32(cp, dp);
                tmem_wait_ld();
                const float4* l4 = reinterpret_cast<const float4*>(&sm.lse2[s][32 * hf]);
                const float4* d4 = reinterpret_cast<const float4*>(&sm.dsum[s][32 * hf]);
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {  // 16-column chunk: packed hi at +0, lo at +8
                    uint32_t ph[8], pl[8], gh[8], gl[8];
#pragma unroll
                    for (int i4 = 0; i4 < 4; ++i4) {
                        const float4 lv = l4[4 * cc + i4], dv = d4[4 * cc + i4];
                        const float lse_[4] = {lv.x, lv.y, lv.z, lv.w};
                        const float ds_[4] = {dv.x, dv.y, dv.z, dv.w};
                        float pr[4], gr[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int i = 16 * cc + 4 * i4 + u;
                            float pv = ex2(fmaf(sv[i], p.scale_log2, -lse_[u]));
                            pv = ((vmask >> i) & 1u) ? pv : 0.f;
                            pr[u] = pv;
                            gr[u] = pv * (dp[i] - ds_[u]);
                        }
                        split2(pr[0], pr[1], ph[2 * i4], pl[2 * i4]);
                        split2(pr[2], pr[3], ph[2 * i4 + 1], pl[2 * i4 + 1]);
                        split2(gr[0], gr[1], gh[2 * i4], gl[2 * i4]);
                        split2(gr[2], gr[3], gh[2 * i4 + 1], gl[2 * i4 + 1]);
                    }
                    // P and dS packed over the columns just read (see the header).
                    tmem_st8(cs + 16 * cc, ph);
                    tmem_st8(cs + 16 * cc + 8, pl);
                    tmem_st8(cp + 16 * cc, gh);
                    tmem_st8(cp + 16 * cc + 8, gl);
                    // Key row of the stacked dS operand of the dQ product
                    // (see the header): queries 32*hf + 16*cc.. go to
                    // atom hf (sh[buf] or sl[buf]), hi in chunks 4*cc, +1 and
                    // lo in chunks 4*cc + 2, +3.
                    uint8_t* const dsr = sm.sh[0] + ds_off + buf * (BK * 128);
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        *reinterpret_cast<uint4*>(dsr + (((4 * cc + u) ^ ds_sw) << 4)) =
                            make_uint4(gh[4 * u], gh[4 * u + 1], gh[4 * u + 2], gh[4 * u + 3]);
                        *reinterpret_cast<uint4*>(dsr + (((4 * cc + 2 + u) ^ ds_sw) << 4)) =
                            make_uint4(gl[4 * u], gl[4 * u + 1], gl[4 * u + 2], gl[4 * u + 3]);
                    }
                }
                tmem_wait_st();
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(&sm.pds[buf]);
            }
            if (failed) break;

            // Item end.  The next item's K / V rows go into registers now and
            // into shared memory once this item's last dQ product is done.
            const int wn = item_id(c, r + 1, G);
            const bool has_next = wn < p.n_work;
            Item nx = it;
            if (has_next) {
                nx = make_item(p, wn);
                const long base = static_cast<long>(nx.b) * p.T;
                tc::Rows2<BK, NELEM, D> kv;
                kv.template load<V8>(p.k + base * p.ld_qkv + nx.h * D, p.ld_qkv, p.v + base * p.ld_qkv + nx.h * D,
                                     p.ld_qkv, nx.k0, p.T, tid);
                if (!mbar_wait_warp(&sm.kv_free, r & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                kv.store(sm.kh, sm.kl, sm.vh, sm.vl, tid);
                fence_async_smem();
                mbar_arrive(&sm.kv_full);
            }
            const int gl_ = g - 1;  // this item's last tile
            if (!mbar_wait_warp(&sm.bar_d[gl_ & 1], (gl_ >> 1) & 1, p.wait_ns)) {
                failed = true;
                break;
            }
            tc_fence_after();
            if (!store_dkv(p, sm, tm, it, lb, row, hf, tid, r)) {
                failed = true;
                break;
            }
            if (!has_next) break;
            it = nx;
        }
    }

    if (failed) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, TMEM_COLS);
}

template <bool DET, bool V8>
__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_tc64(const Params p) {
    bwd_body<DET, V8, 64>(p);
}
template <bool DET, bool V8>
__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_tc32(const Params p) {
    bwd_body<DET, V8, 32>(p);
}

}  // namespace

bool bwd_tc_supported(const BwdArgs& a) { return a.d == 64 || a.d == 32; }

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
    p.dq_part = a.dq_part;
    p.dk = a.dk;
    p.dv = a.dv;
    p.ld_d = a.ld_d;
    p.status = status;
    p.wait_ns = a.wait_ns;
    p.B = a.B;
    p.T = a.T;
    p.H = a.H;
    p.scale = a.scale;
    p.scale_log2 = a.scale * kLog2e;
    p.causal = a.causal;
    p.n_ktiles = (a.T + BK - 1) / BK;
    p.n_qtiles = (a.T + BQ - 1) / BQ;
    const long n_work = static_cast<long>(p.n_ktiles) * a.B * a.H;
    if (n_work <= 0 || n_work > INT32_MAX) return cudaErrorInvalidValue;
    p.n_work = static_cast<int>(n_work);
    const bool d32 = a.d == 32;
    const size_t smem = (d32 ? sizeof(Smem<32>) : sizeof(Smem<64>)) + 1024;
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    // 256-bit row loads when every row of q, k, v and dout starts on a
    // 32-byte boundary (the per-head column offsets, 256 bytes, keep it).
    auto a32 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 31) == 0; };
    const bool v8 = a32(a.q) && a32(a.k) && a32(a.v) && a32(a.dout) && a.ld_qkv % 8 == 0 && a.ld_o % 8 == 0;
    static std::atomic<uint64_t> attr_done{0};  // one bit per device and variant: the attribute is per device
    const uint64_t bit = 1ull << ((8 * dev + (d32 ? 4 : 0) + (p.dq_part ? 2 : 0) + (v8 ? 1 : 0)) & 63);
    auto kernel = d32 ? (p.dq_part ? (v8 ? attn_bwd_tc32<true, true> : attn_bwd_tc32<true, false>)
                                   : (v8 ? attn_bwd_tc32<false, true> : attn_bwd_tc32<false, false>))
                      : (p.dq_part ? (v8 ? attn_bwd_tc64<true, true> : attn_bwd_tc64<true, false>)
                                   : (v8 ? attn_bwd_tc64<false, true> : attn_bwd_tc64<false, false>));
    if (!(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    // Persistent: one CTA per SM (the shared-memory footprint allows no more).
    const int grid = static_cast<int>(n_work < num_sms ? n_work : num_sms);
    e = launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(NTHREADS), smem, stream, p);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
