// Causal self-attention backward on the 5th-generation tensor cores
// (sm_100a), head_dim 64.  Replaces ComputeBackend::attention_backward
// (src/backend.rs:223-231; CPU src/backward.rs:464-514; WGSL
// attn_backward_scores / attn_backward_dkv), recomputing the probabilities
// from the forward's log-sum-exp instead of reading a cached [H][T][T] P.
//
// Two launches: attn_bwd_zero_dq clears dq (dQ is accumulated with vector
// reductions), then attn_bwd_tc64 does everything else, including
// D = rowsum(dO * O) (the reference's sum_j att[j] * d_att[j],
// src/backward.rs:501), which it forms while it converts each dO tile.
//
// Work item = one 128-row key tile of one (batch, head) slab: K, V and the
// dK, dV accumulators stay resident while the item walks the 64-row query
// tiles on or below the diagonal.  The kernel is persistent (one CTA per SM):
// CTA c takes items c, 2G-1-c, 2G+c, ... of the list ordered longest first
// (a snake order, which evens out the tile counts per CTA), and its query
// tiles form one pipeline across item boundaries.  Products (bf16x3:
// hi*hi + hi*lo + lo*hi, f32 accumulation):
//   S^T  = K Q^T      M=128 (keys) N=64 (queries)   SS, both K-major
//   dP^T = V dO^T     M=128 N=64                    SS, both K-major
//   P = exp2(S^T * scale*log2e - lse*log2e),  dS = P * (dP^T - D)   (threads)
//   dV  += P^T dO     M=128 N=64 K=64    TS: P from TMEM, dO MN-major
//   dK  += dS^T Q     M=128 N=64 K=64    TS: dS from TMEM, Q MN-major
//   dQ_i = dS K       M=64  N=64 K=128   SS: dS^T (shared) read MN-major, K MN-major;
//                     added into global dq with vector reductions.
//
// Loads are TMA copies of raw f32 tiles (3-D tensor maps over
// [B][T][columns]; rows past T read zeros), converted in place into bf16
// hi / lo halves in the 128B-swizzled UMMA layout: an item's K and V by the
// elementwise warps, each query tile's Q and dO by the stage warps.
//
// Warp roles (448 threads, one CTA per SM):
//   warps 0-7   elementwise.  Warp w reads TMEM lanes 32*(w%4).. (key rows)
//               and query columns 32*(w/4)..+31 of each 64-column tile and
//               writes P and dS.  At an item's start they convert its K / V.
//   warps 8-11  stage warps: per query tile, convert Q and dO, form D from
//               dO and O (O read from global, one tile ahead), and stage lse;
//               then add tile n-1's finished dQ into dq; at an item's end
//               they store its dK / dV straight from TMEM, so the elementwise
//               warps go on with the next item meanwhile.
//   warp 12     one lane issues every tcgen05.mma and commit, in whichever
//               order its inputs become ready.
//   warp 13     one lane issues every TMA copy as soon as its buffer is free.
// Everything a query tile touches is double-buffered (S^T / dP^T in TMEM,
// dS^T in shared memory, the dQ accumulator in TMEM), so the tensor core runs
// tile i's gradient products while the elementwise warps work on tile i+1.
// P and dS are packed over their own S^T / dP^T columns: for query columns
// 16c..16c+15, bf16 hi goes to columns 16c..16c+7 and lo to 16c+8..16c+15,
// which the owning warp has already read; the tensor core runs one thread's
// MMAs in issue order, so the next S^T lands only after dV / dK read them.
//
// Every wait is bounded (p.wait_ns of wall time) and every hand-off inside a
// warp group is an mbarrier, never a named barrier, so a role whose wait runs
// out can leave its loop without stranding the others: they run out at their
// next wait.  Copies and MMAs in flight are drained (bounded) before the
// tensor memory is freed, and the device status word is set.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"
#include "tc_tiles.cuh"
#include "tma_map.h"

namespace kattn {
using namespace sm100;

namespace {

constexpr int BK = 128;  // key rows per item
constexpr int BQ = 64;   // query rows per tile
constexpr int D = 64;
constexpr int NELEM = 256;  // elementwise threads (warps 0-7)
constexpr int NSTG = 128;   // stage threads (warps 8-11)
constexpr int MMA_WARP = (NELEM + NSTG) / 32;
constexpr int TMA_WARP = MMA_WARP + 1;
constexpr int NTHREADS = NELEM + NSTG + 64;
constexpr int STAGES = 3;  // query-tile ring depth (Q, dO, lse, D)
constexpr unsigned long long DRAIN_NS = 10000000ull;  // drain waits after a failure

// TMEM columns (512 allocated).  Buffer b: S^T (then P packed) at col_s(b),
// dP^T (then dS packed) at col_dp(b), dQ tile (M=64 layout) at col_dq(b).
__device__ __forceinline__ uint32_t col_s(int b) { return b ? 128u : 0u; }
__device__ __forceinline__ uint32_t col_dp(int b) { return b ? 192u : 64u; }
__device__ __forceinline__ uint32_t col_dq(int b) { return b ? 320u : 256u; }
constexpr uint32_t COL_DV = 384;
constexpr uint32_t COL_DK = 448;
constexpr uint32_t TMEM_COLS = 512;

constexpr uint32_t KV_BYTES = BK * 256;  // one raw f32 K or V tile; later hi (first half) | lo
constexpr uint32_t QT_BYTES = BQ * 256;  // one raw f32 Q or dO tile; later hi | lo
constexpr uint32_t STAGE_BYTES = 2 * QT_BYTES;

struct alignas(1024) Smem {
    uint8_t k[KV_BYTES];
    uint8_t v[KV_BYTES];
    uint8_t qg[STAGES][STAGE_BYTES];  // ring stage: Q tile, then dO tile
    uint8_t sh[2][BK * 128];          // dS^T [key][64 queries], per TMEM buffer
    uint8_t sl[2][BK * 128];
    float lse2[STAGES][BQ];  // lse * log2(e), +inf beyond T
    float dsum[STAGES][BQ];  // D, 0 beyond T
    uint64_t kv_full;    // K / V of the CTA's item r landed (phase r&1)
    uint64_t kv_read;    // every elementwise thread holds its share of the raw K, then of V (phases 2r, 2r+1)
    uint64_t kv_ready;   // K / V of item r converted
    uint64_t kv_free;    // item r's last dQ product done: K / V may be replaced
    uint64_t q_full[STAGES];   // Q / dO of a tile landed
    uint64_t q_read[STAGES];   // every stage thread holds its share of the raw Q / dO
    uint64_t q_ready[STAGES];  // Q / dO converted, lse and D staged
    uint64_t empty[STAGES];    // gradient products of the tile in the stage done
    uint64_t bar_s[2];    // S^T / dP^T of the tile in TMEM buffer b done
    uint64_t pds[2];      // P / dS of the tile in buffer b written
    uint64_t bar_d[2];    // gradient products of the tile in buffer b done
    uint64_t dq_free[2];  // dQ accumulator b read out by the stage warps
    uint64_t dkv_free;    // dK / dV of item r stored (phase r&1)
    uint64_t drain;       // MMAs drained after a failure
    uint32_t tmem_slot;
};

static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory (plus alignment slack) exceeds 227 KB");

struct alignas(64) Params {
    CUtensorMap tq, tk, tv, tdo;  // {H*64 columns, T rows, B} f32; boxes {64, BQ, 1} (q, dO), {64, BK, 1} (k, v)
    const float* o;
    long ld_o;
    const float* lse;
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
    __device__ __forceinline__ bool last_of_item() const { return n + 1 == n_it; }
};

// Shared-memory descriptors, built once by the issuing thread.  A K-major
// k-step advances 32 bytes inside the swizzled row; an MN-major k-step
// advances 16 rows (2048 bytes).  The K-major and MN-major descriptors of one
// tile differ only in the leading-byte offset.
struct Descs {
    uint64_t kh, kl, vh, vl;      // K / V, K-major (S^T, dP^T A operands)
    uint64_t kh_mn, kl_mn;        // K, MN-major (dQ B operand)
    uint64_t qh, ql, gh, gl;      // Q / dO of ring stage 0, K-major; stage s is STAGE_BYTES * s further
    uint64_t s0h, s0l, s1h, s1l;  // dS^T buffer 0 / 1, MN-major (dQ A)
};

constexpr uint32_t MN_LBO_Q = BQ * 128;  // leading-byte offset of a 64-row MN-major tile
constexpr uint32_t MN_LBO_K = BK * 128;

__device__ __forceinline__ uint64_t as_mn(uint64_t kdesc, uint32_t lbo) {
    return (kdesc & ~(static_cast<uint64_t>(0x3FFFu) << 16)) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16);
}

__device__ __forceinline__ void make_descs(const Smem& sm, Descs& d) {
    d.kh = smem_desc(smem_u32(sm.k), 16, 1024);
    d.kl = smem_desc(smem_u32(sm.k + BK * 128), 16, 1024);
    d.vh = smem_desc(smem_u32(sm.v), 16, 1024);
    d.vl = smem_desc(smem_u32(sm.v + BK * 128), 16, 1024);
    d.kh_mn = as_mn(d.kh, MN_LBO_K);
    d.kl_mn = as_mn(d.kl, MN_LBO_K);
    d.qh = smem_desc(smem_u32(sm.qg[0]), 16, 1024);
    d.ql = smem_desc(smem_u32(sm.qg[0] + BQ * 128), 16, 1024);
    d.gh = smem_desc(smem_u32(sm.qg[0] + QT_BYTES), 16, 1024);
    d.gl = smem_desc(smem_u32(sm.qg[0] + QT_BYTES + BQ * 128), 16, 1024);
    d.s0h = smem_desc(smem_u32(sm.sh[0]), MN_LBO_K, 1024);
    d.s0l = smem_desc(smem_u32(sm.sl[0]), MN_LBO_K, 1024);
    d.s1h = smem_desc(smem_u32(sm.sh[1]), MN_LBO_K, 1024);
    d.s1l = smem_desc(smem_u32(sm.sl[1]), MN_LBO_K, 1024);
}

// S^T and dP^T of the query tile in ring stage s into TMEM buffer b.
__device__ __forceinline__ void issue_sdp(const Descs& d, uint32_t tm, int s, int b) {
    constexpr uint32_t idesc = idesc_bf16(BK, BQ, 0, 0);
    const uint32_t cs = tm + col_s(b), cp = tm + col_dp(b);
    const uint32_t so = s * STAGE_BYTES;
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

// dQ_b = dS K (dS^T of buffer b from shared memory, K MN-major).
__device__ __forceinline__ void issue_dq(const Descs& d, uint32_t tm, int b) {
    constexpr uint32_t idesc_q = idesc_bf16(BQ, D, 1, 1);
    const uint32_t cq = tm + col_dq(b);
    const uint64_t sh = b ? d.s1h : d.s0h, sl = b ? d.s1l : d.s0l;
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
        const uint32_t o = ks * 2048;
        mma_ss(cq, desc_add(sh, o), desc_add(d.kh_mn, o), idesc_q, ks > 0);
        mma_ss(cq, desc_add(sh, o), desc_add(d.kl_mn, o), idesc_q, 1);
        mma_ss(cq, desc_add(sl, o), desc_add(d.kh_mn, o), idesc_q, 1);
    }
}

// dV += P^T dO, dK += dS^T Q (P, dS from TMEM buffer b; dO, Q of ring stage s).
__device__ __forceinline__ void issue_dkv(const Descs& d, uint32_t tm, int s, int b, bool first) {
    constexpr uint32_t idesc_kv = idesc_bf16(BK, D, 0, 1);
    const uint32_t so = s * STAGE_BYTES;
    const uint64_t qh = as_mn(desc_add(d.qh, so), MN_LBO_Q), ql = as_mn(desc_add(d.ql, so), MN_LBO_Q);
    const uint64_t gh = as_mn(desc_add(d.gh, so), MN_LBO_Q), gl = as_mn(desc_add(d.gl, so), MN_LBO_Q);
#pragma unroll
    for (int ks = 0; ks < BQ / 16; ++ks) {
        const uint32_t acc = (first && ks == 0) ? 0u : 1u;
        const uint32_t o = ks * 2048;
        const uint32_t ph = tm + col_s(b) + 16 * ks, gph = tm + col_dp(b) + 16 * ks;  // hi; lo is 8 further
        mma_ts(tm + COL_DV, ph, desc_add(gh, o), idesc_kv, acc);
        mma_ts(tm + COL_DV, ph, desc_add(gl, o), idesc_kv, 1);
        mma_ts(tm + COL_DV, ph + 8, desc_add(gh, o), idesc_kv, 1);
        mma_ts(tm + COL_DK, gph, desc_add(qh, o), idesc_kv, acc);
        mma_ts(tm + COL_DK, gph, desc_add(ql, o), idesc_kv, 1);
        mma_ts(tm + COL_DK, gph + 8, desc_add(qh, o), idesc_kv, 1);
    }
}

// A dQ tile (M=64 accumulator: query row 16*qd + l sits in lane 32*qd + l,
// l < 16), scaled and added into dq by the stage warp of lane quadrant qd,
// 32 columns at a time.  The TMEM loads run on every lane (warp-collective).
__device__ __forceinline__ void dq_epilogue(const Params& p, uint32_t tm, int b, int qd, int lane, int q0,
                                            float* dqg) {
    const uint32_t ta = (static_cast<uint32_t>(qd * 32) << 16) + tm + col_dq(b);
    const int r = q0 + qd * 16 + lane;
    float* dst = dqg + static_cast<long>(r) * p.ld_d;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float v[32];
        tmem_ld32(ta + 32 * h, v);
        tmem_wait_ld();
        if (lane < 16 && r < p.T) {
#pragma unroll
            for (int c = 0; c < 32; c += 4)
                red_add_v4(dst + 32 * h + c, v[c] * p.scale, v[c + 1] * p.scale, v[c + 2] * p.scale,
                           v[c + 3] * p.scale);
        }
    }
}

// dK, dV of an item -> global, by the stage warp of lane quadrant qd: key row
// k0 + 32*qd + lane, 32 columns per TMEM load (warp-collective), stored as
// that row's float4s.
__device__ __forceinline__ void store_dkv(const Params& p, uint32_t tm, const Item& it, int qd, int lane) {
    const uint32_t lb = static_cast<uint32_t>(qd * 32) << 16;
    const int row = it.k0 + qd * 32 + lane;
    const long g = (static_cast<long>(it.b) * p.T + row) * p.ld_d + it.h * D;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const uint32_t col = t ? COL_DK : COL_DV;
        float* dst = (t ? p.dk : p.dv) + g;
        const float mul = t ? p.scale : 1.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float a[32];
            tmem_ld32(lb + tm + col + 32 * h, a);
            tmem_wait_ld();
            if (row < p.T) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    *reinterpret_cast<float4*>(dst + 32 * h + 4 * i) =
                        make_float4(a[4 * i] * mul, a[4 * i + 1] * mul, a[4 * i + 2] * mul, a[4 * i + 3] * mul);
            }
        }
    }
}

__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_tc64(const __grid_constant__ Params p) {
    // Launched behind attn_bwd_zero_dq, which waited for every earlier grid
    // before letting this one launch: all inputs are final.  Only the dq
    // reductions wait for the clearing.
    pdl_launch();
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

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
        mbar_init(&sm.kv_full, 1);
        mbar_init(&sm.kv_read, NELEM);
        mbar_init(&sm.kv_ready, NELEM);
        mbar_init(&sm.kv_free, 1);
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&sm.q_full[i], 1);
            mbar_init(&sm.q_read[i], NSTG);
            mbar_init(&sm.q_ready[i], NSTG);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.bar_s[i], 1);
            mbar_init(&sm.pds[i], NELEM);
            mbar_init(&sm.bar_d[i], 1);
            mbar_init(&sm.dq_free[i], NSTG);
        }
        mbar_init(&sm.dkv_free, NSTG);
        mbar_init(&sm.drain, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = sm.tmem_slot;
    bool failed = false;

    if (warp == TMA_WARP) {
        // ------------------------------------------------------------ TMA issuer
        //   K / V of item r     once item r-1's last dQ product is done (kv_free)
        //   Q / dO of tile n    once tile n-STAGES's gradient products are done (empty)
        // Each probe is unambiguous: a barrier's next phase can complete only
        // after the copy this thread issues in response to the one probed.
        if (lane == 0) {
            prefetch_tensormap(&p.tq);
            prefetch_tensormap(&p.tk);
            prefetch_tensormap(&p.tv);
            prefetch_tensormap(&p.tdo);
            Cursor cq;
            cq.start(p, c, G);
            int n_items = 0;  // this CTA's items
            while (item_id(c, n_items, G) < p.n_work) ++n_items;
            int nq = 0, rkv = 0;  // query tiles / items whose copies were issued
            uint64_t t_idle = 0;
            while (!failed && (cq.valid() || rkv < n_items)) {
                bool progressed = false;
                // The next item's K / V (items are loaded in order, never
                // ahead of the item whose query tiles are being loaded).
                if (rkv < n_items && (!cq.valid() || rkv <= cq.r) &&
                    (rkv == 0 || mbar_test_wait(&sm.kv_free, (rkv - 1) & 1))) {
                    const Item it = make_item(p, item_id(c, rkv, G));
                    mbar_arrive_expect_tx(&sm.kv_full, 2 * KV_BYTES);
                    tma_load_3d(sm.k, &p.tk, it.h * D, it.k0, it.b, &sm.kv_full);
                    tma_load_3d(sm.v, &p.tv, it.h * D, it.k0, it.b, &sm.kv_full);
                    ++rkv;
                    progressed = true;
                }
                const int s = nq % STAGES;
                if (cq.valid() && (nq < STAGES || mbar_test_wait(&sm.empty[s], ((nq - STAGES) / STAGES) & 1))) {
                    const Item it = make_item(p, cq.w);
                    const int q0 = (cq.it0 + cq.n) * BQ;
                    mbar_arrive_expect_tx(&sm.q_full[s], 2 * QT_BYTES);
                    tma_load_3d(sm.qg[s], &p.tq, it.h * D, q0, it.b, &sm.q_full[s]);
                    tma_load_3d(sm.qg[s] + QT_BYTES, &p.tdo, it.h * D, q0, it.b, &sm.q_full[s]);
                    ++nq;
                    cq.next(p, c, G);
                    progressed = true;
                }
                if (progressed) {
                    t_idle = 0;
                } else {
                    const uint64_t now = globaltimer_ns();
                    if (t_idle == 0) t_idle = now;
                    else if (now - t_idle > p.wait_ns) failed = true;
                    __nanosleep(64);
                }
            }
            if (failed) {
                // Copies still landing complete before the shared memory is
                // released (bounded waits).  Earlier copies into a buffer were
                // consumed before it was reloaded.
                if (rkv > 0) mbar_wait(&sm.kv_full, (rkv - 1) & 1, DRAIN_NS);
                for (int t = max(0, nq - STAGES); t < nq; ++t)
                    mbar_wait(&sm.q_full[t % STAGES], (t / STAGES) & 1, DRAIN_NS);
            }
        }
        __syncwarp();
    } else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        // sdp(n) needs tile n converted, for n >= 2 grads(n-2) issued (TMEM
        // buffer n&1; the tensor core runs this thread's MMAs in order) and
        // the item's K / V converted.  grads(n) needs P / dS of tile n
        // written, for n >= 2 dQ buffer n&1 read out, and for an item's first
        // tile the previous item's dK / dV stored.  An item's last dQ product
        // commits kv_free.
        if (lane == 0) {
            Descs d;
            make_descs(sm, d);
            Cursor cs, cg;
            cs.start(p, c, G);
            cg.start(p, c, G);
            int ns = 0, ng = 0, kv_round = -1;
            uint64_t t_idle = 0;
            while (cg.valid() && !failed) {
                bool progressed = false;
                if (cs.valid() && ns < ng + 2) {
                    bool kv_ok = kv_round >= cs.r;
                    if (!kv_ok && mbar_test_wait(&sm.kv_ready, cs.r & 1)) {
                        kv_round = cs.r;
                        kv_ok = true;
                    }
                    if (kv_ok && mbar_test_wait(&sm.q_ready[ns % STAGES], (ns / STAGES) & 1)) {
                        tc_fence_after();
                        issue_sdp(d, tm, ns % STAGES, ns & 1);
                        mma_commit(&sm.bar_s[ns & 1]);
                        ++ns;
                        cs.next(p, c, G);
                        progressed = true;
                    }
                }
                if (ng < ns && mbar_test_wait(&sm.pds[ng & 1], (ng >> 1) & 1) &&
                    (ng < 2 || mbar_test_wait(&sm.dq_free[ng & 1], ((ng - 2) >> 1) & 1)) &&
                    (cg.n != 0 || cg.r == 0 || mbar_test_wait(&sm.dkv_free, (cg.r - 1) & 1))) {
                    tc_fence_after();
                    issue_dq(d, tm, ng & 1);
                    if (cg.last_of_item()) mma_commit(&sm.kv_free);
                    issue_dkv(d, tm, ng % STAGES, ng & 1, cg.n == 0);
                    mma_commit(&sm.empty[ng % STAGES]);
                    mma_commit(&sm.bar_d[ng & 1]);
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
            if (failed) {
                // MMAs still in flight complete before the columns are freed.
                mma_commit(&sm.drain);
                mbar_wait(&sm.drain, 0, DRAIN_NS);
            }
        }
        __syncwarp();
    } else if (warp >= NELEM / 32) {
        // ------------------------------------------------------------ stage warps
        // Iteration n: convert query tile n (Q, dO; D = rowsum(dO * O) with O
        // read from global one tile ahead; lse), then add tile n-1's dQ into
        // dq and, if tile n-1 ended its item, store that item's dK / dV.
        const int t = tid - NELEM;
        const int qd = warp & 3;
        Cursor cl, ce;  // tile to convert, tile whose dQ is added
        cl.start(p, c, G);
        ce.start(p, c, G);
        constexpr int QI = BQ * 16 / NSTG;  // float4s of a 64x64 tile per thread
        float4 ov[QI];
        float lse_t = 0.f;
        auto prefetch = [&]() {  // O rows and lse of the tile at cl
            const Item it = make_item(p, cl.w);
            const int q0 = (cl.it0 + cl.n) * BQ;
            const float* og = p.o + static_cast<long>(it.b) * p.T * p.ld_o + it.h * D;
#pragma unroll
            for (int i = 0; i < QI; ++i) {
                const int f = t + i * NSTG;  // row f >> 4, columns 4 (f & 15) ..
                const int r = q0 + (f >> 4);
                ov[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (r < p.T)
                    ov[i] = __ldg(reinterpret_cast<const float4*>(og + static_cast<long>(r) * p.ld_o + 4 * (f & 15)));
            }
            if (t < BQ) {
                const long bh = (static_cast<long>(it.b) * p.H + it.h) * p.T;
                lse_t = (q0 + t < p.T) ? p.lse[bh + q0 + t] * kLog2e : INFINITY;
            }
        };
        bool dq_cleared = false;
        if (cl.valid()) prefetch();
        for (int n = 0; !failed; ++n) {
            if (cl.valid()) {
                const int s = n % STAGES;
                uint8_t* qt = sm.qg[s];
                uint8_t* gt = sm.qg[s] + QT_BYTES;
                if (!mbar_wait_warp(&sm.q_full[s], (n / STAGES) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                // D of this thread's rows (t >> 4) + 8 i from the raw dO in
                // shared memory and the O registers: the 16 threads of a
                // half-warp hold one row between them.  Done before the raw
                // tiles are read for conversion, so O and the tiles are not
                // live in registers at once.
#pragma unroll
                for (int i = 0; i < QI; ++i) {
                    const float4 g = reinterpret_cast<const float4*>(gt)[t + i * NSTG];
                    float dv = g.x * ov[i].x + g.y * ov[i].y + g.z * ov[i].z + g.w * ov[i].w;
#pragma unroll
                    for (int off = 8; off > 0; off >>= 1) dv += __shfl_xor_sync(0xffffffffu, dv, off);
                    if ((t & 15) == 0) sm.dsum[s][(t >> 4) + 8 * i] = dv;
                }
                if (t < BQ) sm.lse2[s][t] = lse_t;
                tc::RawTile<BQ, NSTG> qr, gr;
                qr.read(qt, t);
                gr.read(gt, t);
                // Converted in place: every thread has read its share first.
                mbar_arrive(&sm.q_read[s]);
                if (!mbar_wait_warp(&sm.q_read[s], (n / STAGES) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                qr.write(qt, 1.f, t);
                gr.write(gt, 1.f, t);
                fence_async_smem();
                mbar_arrive(&sm.q_ready[s]);
                cl.next(p, c, G);
                if (cl.valid()) prefetch();
            }
            if (n >= 1) {
                if (!ce.valid()) break;
                const int m = n - 1;
                if (!mbar_wait_warp(&sm.bar_d[m & 1], (m >> 1) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                if (!dq_cleared) {
                    pdl_wait();  // attn_bwd_zero_dq has finished
                    dq_cleared = true;
                }
                const Item it = make_item(p, ce.w);
                float* dqg = p.dq + static_cast<long>(it.b) * p.T * p.ld_d + it.h * D;
                dq_epilogue(p, tm, m & 1, qd, lane, (ce.it0 + ce.n) * BQ, dqg);
                const bool item_end = ce.last_of_item();
                if (item_end) store_dkv(p, tm, it, qd, lane);
                tc_fence_before();
                mbar_arrive(&sm.dq_free[m & 1]);
                if (item_end) mbar_arrive(&sm.dkv_free);
                ce.next(p, c, G);
            }
        }
    } else {
        // ------------------------------------------------------------ elementwise
        const int qd = warp & 3;          // TMEM lane quadrant: key rows 32*qd..
        const int hf = warp >> 2;         // query columns 32*hf..+31 (two 16-column chunks)
        const int row = qd * 32 + lane;   // key row inside the tile
        const uint32_t lb = static_cast<uint32_t>(qd * 32) << 16;
        int g = 0;  // the CTA's query-tile sequence number
        for (int r = 0; !failed; ++r) {
            const int w = item_id(c, r, G);
            if (w >= p.n_work) break;
            const Item it = make_item(p, w);
            // The item's K / V: raw tiles converted in place (every thread
            // reads its share before any thread writes).
            {
                if (!mbar_wait_warp(&sm.kv_full, r & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                // K, then V: kv_read completes twice per item (phases 2r, 2r+1).
                bool ok = true;
#pragma unroll 1
                for (int u = 0; u < 2 && ok; ++u) {
                    uint8_t* tile = u ? sm.v : sm.k;
                    tc::RawTile<BK, NELEM> kr;
                    kr.read(tile, tid);
                    mbar_arrive(&sm.kv_read);
                    ok = mbar_wait_warp(&sm.kv_read, u, p.wait_ns);
                    if (ok) kr.write(tile, 1.f, tid);
                }
                if (!ok) {
                    failed = true;
                    break;
                }
                fence_async_smem();
                mbar_arrive(&sm.kv_ready);
            }
            const int j = it.k0 + row;
            for (int n = 0; n < it.n_it; ++n, ++g) {
                const int s = g % STAGES;  // ring stage of this query tile
                const int buf = g & 1;     // TMEM / dS buffer
                const int q0 = (it.it0 + n) * BQ;
                // q_ready[s]: this tile's lse / D are staged.
                if (!mbar_wait_warp(&sm.bar_s[buf], (g >> 1) & 1, p.wait_ns) ||
                    !mbar_wait_warp(&sm.q_ready[s], (g / STAGES) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                if (g >= 2 && !mbar_wait_warp(&sm.bar_d[buf], ((g - 2) >> 1) & 1, p.wait_ns)) {
                    failed = true;  // dS^T buffer `buf` is read by tile g-2's dQ product
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
                    // dS^T row for the dQ product: query chunks 4*hf + 2*cc, +1.
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t off = sw128(row, 4 * hf + 2 * cc + u);
                        *reinterpret_cast<uint4*>(sm.sh[buf] + off) =
                            make_uint4(gh[4 * u], gh[4 * u + 1], gh[4 * u + 2], gh[4 * u + 3]);
                        *reinterpret_cast<uint4*>(sm.sl[buf] + off) =
                            make_uint4(gl[4 * u], gl[4 * u + 1], gl[4 * u + 2], gl[4 * u + 3]);
                    }
                }
                tmem_wait_st();
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(&sm.pds[buf]);
            }
        }
    }

    if (__syncthreads_or(failed) && tid == 0) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, TMEM_COLS);
}

// dq = 0 over the H*64 columns of every row of a strided [rows][ld] buffer.
// It waits for the grid before it first (dq may be that grid's input), so the
// backward behind it launches only once every earlier grid has finished.
__global__ void __launch_bounds__(256) attn_bwd_zero_dq(float* dq, long ld, long rows, int c4) {
    pdl_wait();
    pdl_launch();
    const long n = rows * c4;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / c4;
        const int q = static_cast<int>(i - r * c4);
        *reinterpret_cast<float4*>(dq + r * ld + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

}  // namespace

bool bwd_tc_supported(const BwdArgs& a) { return a.d == 64; }

cudaError_t launch_bwd_tc(const BwdArgs& a, int num_sms, int* status, cudaStream_t stream, int* launches) {
    Params p;
    if (!encode_rows(&p.tq, a.q, a.ld_qkv, a.B, a.T, a.H, D, BQ, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_rows(&p.tk, a.k, a.ld_qkv, a.B, a.T, a.H, D, BK, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_rows(&p.tv, a.v, a.ld_qkv, a.B, a.T, a.H, D, BK, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_rows(&p.tdo, a.dout, a.ld_o, a.B, a.T, a.H, D, BQ, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    p.o = a.o;
    p.ld_o = a.ld_o;
    p.lse = a.lse;
    p.dq = a.dq;
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

    const long rows = static_cast<long>(a.B) * a.T;
    const int c4 = a.H * D / 4;
    const long n4 = rows * c4;
    const long zgrid = std::min<long>((n4 + 255) / 256, 4L * (num_sms > 0 ? num_sms : 148));
    cudaError_t e = launch_pdl(attn_bwd_zero_dq, dim3(static_cast<unsigned>(zgrid)), dim3(256), 0, stream, a.dq,
                               a.ld_d, rows, c4);
    if (e != cudaSuccess) return e;
    *launches += 1;

    const size_t smem = sizeof(Smem) + 1024;
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_done{0};  // one bit per device: the attribute is per device
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(attn_bwd_tc64, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    // Persistent: one CTA per SM (the shared-memory footprint allows no more).
    const int grid = static_cast<int>(n_work < num_sms ? n_work : num_sms);
    e = launch_pdl(attn_bwd_tc64, dim3(static_cast<unsigned>(grid)), dim3(NTHREADS), smem, stream, p);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
