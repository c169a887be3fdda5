// Causal self-attention forward on the 5th-generation tensor cores (sm_100a),
// head_dim 64 and 32 (one kernel body, templated on the head dimension D; the
// notes below give the D = 64 sizes).  Replaces the scalar head loop of
// src/pipeline.rs:305-347.
//
// Numerics: every f32 operand x is split into bf16 hi = bf16(x) and
// lo = bf16(x - hi); each product A*B is formed as hi*hi + hi*lo + lo*hi with
// f32 accumulation in tensor memory (relative error ~1e-5, inside the 1e-4
// forward tolerance; a single bf16 or tf32 product is not).
//
// Work item = 128 query rows of one (batch, head) slab.  The kernel is
// persistent: two CTAs per SM, CTA c taking items c, 2G-1-c, 2G+c, ... of the
// list ordered longest first (a snake order: at the 768-dim shape 192 CTAs
// run one long item, 88 run two short ones; block b acts as CTA G-1-b, so
// the two-item CTAs launch first).  g numbers the CTA's 64-row key
// tiles across its items; tile g uses K stage g&1, V stage g&1 and TMEM
// buffers g&1.
//
// Warp roles (320 threads):
//   warps 0-7  two threads per query row: warp w handles TMEM lanes
//              32*(w%4).. (rows) and key columns 32*(w/4).. of each tile.
//              They convert the landed tiles and run the online softmax
//              (log2 domain), exchanging half-row maxima through shared
//              memory.
//   warp 8     one lane issues every tcgen05.mma as soon as its operands are
//              ready, so that no softmax thread blocks on the MMA queue.
//   warp 9     one lane issues every TMA copy as soon as its buffer is free
//              (a copy instruction can wait for the SM's copy engine).
// Loads are TMA copies of raw f32 tiles (3-D tensor maps over [B][T][columns],
// so rows past T read zeros) straight into the operand buffers, ahead of use:
// K_{g+2} once S_g is done, V_{g+2} once PV_g is done, an item's Q once the
// previous item's Q is in TMEM.  The softmax threads convert each landed K / V
// tile in place into bf16 hi / lo halves in the 128B-swizzled UMMA layout, and
// an item's Q into TMEM (hi / lo), where it is the A operand of S.
// Per key tile g the softmax threads
//   convert K_{g+1}                  -> S_{g+1} = Q K_{g+1}^T (TS, 12 MMAs)
//   softmax of S_g, P_g hi/lo over S_g
//   convert V_g                      -> O += P_g V_g (TS, P from TMEM, 12 MMAs)
// so S_{g+1} runs during the softmax of S_g.  O accumulates in TMEM; the
// running row maximum is raised lazily (only when a tile exceeds it by more
// than 2^8), and only then is O rescaled.  O is staged through the item's last
// V stage (64 rows at a time) for coalesced stores.  ~99 KB of shared memory
// and 256 TMEM columns per CTA: two CTAs share an SM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <type_traits>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"
#include "tc_tiles.cuh"
#include "tma_map.h"

namespace kattn {
using namespace sm100;

namespace {

constexpr int BM = 128;  // query rows per item
constexpr int BN = 64;   // key rows per tile
constexpr int NSM = 256;  // softmax / convert threads (warps 0-7), two per query row
constexpr int MMA_WARP = NSM / 32;
constexpr int TMA_WARP = MMA_WARP + 1;
constexpr int NTHREADS = NSM + 64;
constexpr unsigned IDLE_NS = 64;  // back-off of an idle issuer loop

// TMEM columns.  Buffer b: S at col_s(b) (64 f32 columns; P packed over it:
// for key columns 32c..32c+31, bf16 hi in columns 32c..32c+15 and lo in
// 32c+16..32c+31); the O accumulator of the current item at COL_O.
__device__ __forceinline__ uint32_t col_s(int b) { return b ? 64u : 0u; }
constexpr uint32_t COL_O = 128;
// O takes D columns.  Q of the current item as the A operand of S = Q K^T:
// d pair (2i, 2i+1) of a row packed in column i, hi at Q_HI, lo at Q_LO (D/2
// columns each).
constexpr uint32_t Q_HI = 192;
constexpr uint32_t Q_LO = 224;
// mu may trail the true row maximum by up to this much (log2 units).
constexpr float RESCALE_LOG2 = 8.f;
constexpr uint32_t TMEM_COLS = 256;

// Head dimension D = 64 or 32.  A K / V buffer holds a raw f32 tile (rows x
// 4D bytes) as TMA lands it, then the converted bf16 hi half (rows x 2D
// bytes) followed by the lo half, 128B-swizzled at D = 64 and 64B-swizzled at
// D = 32.  The Q buffer holds the raw tile only, as D/32 128B-swizzled boxes
// of 32 columns (each thread then reads its own row without bank conflicts).
template <int D>
struct Cfg {
    static_assert(D == 64 || D == 32, "head_dim 64 or 32");
    static constexpr uint32_t Q_BYTES = BM * D * 4;
    static constexpr uint32_t Q_BOX_BYTES = BM * 128;
    static constexpr uint32_t KV_BYTES = BN * D * 4;
    static constexpr uint32_t HALF = BN * D * 2;      // one converted bf16 half of a K / V tile
    static constexpr uint32_t ROW = D * 2;            // bytes of a converted row
    static constexpr uint32_t SBO = 8 * ROW;          // 8-row swizzle atom
};

template <int D>
struct alignas(1024) Smem {
    uint8_t q[Cfg<D>::Q_BYTES];
    uint8_t k[2][Cfg<D>::KV_BYTES];
    uint8_t v[2][Cfg<D>::KV_BYTES];
    uint64_t q_full;       // raw Q of the CTA's item r landed (phase r&1)
    uint64_t q_ready;      // Q of item r in TMEM; its shared-memory buffer is free (phase r&1)
    uint64_t k_full[2];    // raw K tile g landed in stage g&1 (phase (g>>1)&1)
    uint64_t k_ready[2];   // K tile g converted
    uint64_t v_full[2];    // raw V tile g landed in stage g&1
    uint64_t pv_ready[2];  // P_g written to TMEM and V_g converted
    uint64_t bar_s[2];     // S_g done (TMEM buffer g&1, phase (g>>1)&1)
    uint64_t bar_o[2];     // PV_g done
    uint64_t stg_free;     // item r's O staging read out of its last V stage (phase r&1)
    uint64_t drain;        // MMAs drained after a failure
    float red[2][2][BM];   // row max (per tile, buffer g&1) / row sum of each half-row
    uint32_t tmem_slot;
};

struct alignas(64) Params {
    CUtensorMap tq, tk, tv;  // {H*D columns, T rows, B} f32; boxes {32, BM, 1} (128B swizzle) for q, {D, BN, 1} for k, v
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
    unsigned long long wait_ns;  // wall-time limit of every bounded wait
    int withhold_first_key_load;  // diagnostic: no copy of the first key tile is issued
};

// Item round r of CTA c: item w = r*G + (r odd ? G-1-c : c) of the list
// ordered longest first, its slab (b, h), first query row q0 and key-tile
// count n_kv.
struct Seq {
    int r, j, w, b, h, q0, n_kv;
    __device__ __forceinline__ void set_item(const Params& p, int c, int G) {
        j = 0;
        w = r * G + ((r & 1) ? G - 1 - c : c);
        if (w >= p.n_work) {
            w = -1;
            return;
        }
        const int nslab = p.B * p.H;
        const int slab = w % nslab;
        b = slab / p.H;
        h = slab - b * p.H;
        q0 = (p.n_qtiles - 1 - w / nslab) * BM;
        n_kv = p.causal ? min(p.n_ktiles, (q0 + BM + BN - 1) / BN) : p.n_ktiles;
    }
    __device__ __forceinline__ bool valid() const { return w >= 0; }
};

// Thread 0's next tile to load (item round r, key tile j; w < 0: none
// left), with only what the walk needs kept in registers.
struct Ahead {
    int r, j, w, n_kv;
    __device__ __forceinline__ void set(const Params& p, int c, int G) {
        j = 0;
        w = r * G + ((r & 1) ? G - 1 - c : c);
        if (w >= p.n_work) {
            w = -1;
            return;
        }
        const int q0 = (p.n_qtiles - 1 - w / (p.B * p.H)) * BM;
        n_kv = p.causal ? min(p.n_ktiles, (q0 + BM + BN - 1) / BN) : p.n_ktiles;
    }
    __device__ __forceinline__ void next(const Params& p, int c, int G) {
        if (++j == n_kv) {
            ++r;
            set(p, c, G);
        }
    }
    __device__ __forceinline__ bool valid() const { return w >= 0; }
    __device__ __forceinline__ int slab(const Params& p) const { return w % (p.B * p.H); }
};

// Shared-memory descriptors of K / V stage 0 (stage 1 is KV_BYTES further),
// rebuilt by the issuing thread at each issue (a few integer operations)
// rather than held in registers by every thread.  K is the K-major B operand
// of S; V the MN-major B operand of P V (one N atom, so the leading-byte
// offset is unused).  D = 32 rows are 64 bytes, in the 64B-swizzled layout.
struct Descs {
    uint64_t kh, kl, vh, vl;
};

template <int D>
__device__ __forceinline__ uint64_t k_desc(uint32_t addr) {
    if constexpr (D == 64) return smem_desc(addr, 16, Cfg<D>::SBO);
    else return smem_desc_sw64(addr, Cfg<D>::SBO);
}
template <int D>
__device__ __forceinline__ uint64_t v_desc(uint32_t addr) {
    if constexpr (D == 64) return smem_desc(addr, BN * 128, Cfg<D>::SBO);
    else return smem_desc_sw64(addr, Cfg<D>::SBO);
}

template <int D>
__device__ __forceinline__ Descs make_descs(const Smem<D>& sm) {
    Descs d;
    d.kh = k_desc<D>(smem_u32(sm.k[0]));
    d.kl = k_desc<D>(smem_u32(sm.k[0] + Cfg<D>::HALF));
    d.vh = v_desc<D>(smem_u32(sm.v[0]));
    d.vl = v_desc<D>(smem_u32(sm.v[0] + Cfg<D>::HALF));
    return d;
}

// S = Q K^T of the key tile in stage `stage` into TMEM buffer b (TS: Q from
// TMEM, so only K is read from shared memory).
template <int D>
__device__ __forceinline__ void issue_s(const Descs& d, uint32_t tm, int stage, int b) {
    constexpr uint32_t idesc = idesc_bf16(BM, BN, 0, 0);
    const uint32_t so = stage * Cfg<D>::KV_BYTES;
    const uint64_t kh = desc_add(d.kh, so), kl = desc_add(d.kl, so);
#pragma unroll
    for (int s = 0; s < D / 16; ++s) {
        const uint32_t o = s * 32;
        mma_ts(tm + col_s(b), tm + Q_HI + 8 * s, desc_add(kh, o), idesc, s > 0);
        mma_ts(tm + col_s(b), tm + Q_HI + 8 * s, desc_add(kl, o), idesc, 1);
        mma_ts(tm + col_s(b), tm + Q_LO + 8 * s, desc_add(kh, o), idesc, 1);
    }
}

// O (+)= P V of the key tile in stage `stage`, P packed over S buffer b;
// `first`: the item's first tile (O is overwritten).
template <int D>
__device__ __forceinline__ void issue_pv(const Descs& d, uint32_t tm, int stage, int b, bool first) {
    constexpr uint32_t idesc = idesc_bf16(BM, D, 0, 1);
    const uint32_t so = stage * Cfg<D>::KV_BYTES;
    const uint64_t vh = desc_add(d.vh, so), vl = desc_add(d.vl, so);
#pragma unroll
    for (int s = 0; s < BN / 16; ++s) {
        const uint32_t o = s * 16 * Cfg<D>::ROW;  // 16 keys
        const uint32_t ph = tm + col_s(b) + 32 * (s >> 1) + 8 * (s & 1);
        mma_ts(tm + COL_O, ph, desc_add(vh, o), idesc, (first && s == 0) ? 0u : 1u);
        mma_ts(tm + COL_O, ph, desc_add(vl, o), idesc, 1);
        mma_ts(tm + COL_O, ph + 16, desc_add(vh, o), idesc, 1);
    }
}

// TMA of one raw tile: `rows` rows of slab (b, h) from row `row0`.
template <int D>
__device__ __forceinline__ void load_tile(const CUtensorMap& map, void* dst, uint64_t* bar, uint32_t bytes, int h,
                                          int row0, int b) {
    mbar_arrive_expect_tx(bar, bytes);
    tma_load_3d(dst, &map, h * D, row0, b, bar);
}

template <int D>
__device__ __forceinline__ void fwd_body(const Params& p) {
    // The next grid may launch at once (it waits for this one before it
    // touches memory); this grid's setup below touches no global memory, so
    // it runs while the grid before still drains, and every thread waits
    // for that grid (griddepcontrol.wait) before its first global access.
    pdl_launch();
    extern __shared__ uint8_t smem_raw[];
    Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using C = Cfg<D>;
    // A raw K / V tile, converted in place: 128B-swizzled rows at D = 64,
    // 64B-swizzled at D = 32.
    using Tile = std::conditional_t<D == 64, tc::RawTile<BN, NSM>, tc::RawTile32<BN, NSM>>;

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    // Block b walks the item list as CTA G-1-b, so the CTAs with two short
    // items have the lowest block indices.  Of two CTAs sharing an SM, the
    // warp scheduler favours the one launched first: with the two-item CTAs
    // launched second, their first item ran at ~1.4 us per tile against
    // ~0.8 us, and the kernel ended on their lone second item.
    const int cta = static_cast<int>(gridDim.x - 1 - blockIdx.x);
    const int G = static_cast<int>(gridDim.x);

    if (warp == 0) {
        tmem_alloc(&sm.tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.bar_s[i], 1);
            mbar_init(&sm.bar_o[i], 1);
            mbar_init(&sm.k_full[i], 1);
            mbar_init(&sm.v_full[i], 1);
            mbar_init(&sm.k_ready[i], NSM);
            mbar_init(&sm.pv_ready[i], NSM);
        }
        mbar_init(&sm.q_full, 1);
        mbar_init(&sm.q_ready, NSM);
        mbar_init(&sm.stg_free, NSM);
        mbar_init(&sm.drain, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_wait();
    const uint32_t tm = sm.tmem_slot;
    bool failed = false;

    if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        // One lane issues every tcgen05.mma, in whichever order the
        // conditions are met (non-blocking probes of the barriers):
        //   S_ns   once K_ns is converted (and, for an item's first tile, its
        //          Q), PV_{ns-2} issued (S_ns overwrites P_{ns-2}; the tensor
        //          core runs one thread's MMAs in order)
        //   PV_np  once P_np is written, O rescaled and V_np converted
        // Each probe is unambiguous: the previous phase of the probed barrier
        // completed before the MMA that needed it was issued.
        if ((tid & 31) == 0) {
            Ahead sq, pq;
            sq.r = 0;
            sq.set(p, cta, G);
            pq = sq;
            int ns = 0, np = 0;
            uint64_t t_idle = 0;
            while (!failed && (sq.valid() || np < ns)) {
                bool progressed = false;
                if (np < ns && mbar_test_wait(&sm.pv_ready[np & 1], (np >> 1) & 1)) {
                    tc_fence_after();
                    issue_pv<D>(make_descs<D>(sm), tm, np & 1, np & 1, pq.j == 0);
                    mma_commit(&sm.bar_o[np & 1]);
                    ++np;
                    pq.next(p, cta, G);
                    progressed = true;
                }
                if (sq.valid() && np >= ns - 1 && mbar_test_wait(&sm.k_ready[ns & 1], (ns >> 1) & 1) &&
                    (sq.j != 0 || mbar_test_wait(&sm.q_ready, sq.r & 1))) {
                    tc_fence_after();
                    issue_s<D>(make_descs<D>(sm), tm, ns & 1, ns & 1);
                    mma_commit(&sm.bar_s[ns & 1]);
                    ++ns;
                    sq.next(p, cta, G);
                    progressed = true;
                }
                if (progressed) {
                    t_idle = 0;
                } else {
                    // Idle: back off so the poll leaves the sub-partition's
                    // issue slots to the softmax warps.
                    const uint64_t now = globaltimer_ns();
                    if (t_idle == 0) t_idle = now;
                    else if (now - t_idle > p.wait_ns) failed = true;
                    __nanosleep(IDLE_NS);
                }
            }
            if (failed) {
                // MMAs still in flight complete before the columns are freed.
                mma_commit(&sm.drain);
                mbar_wait(&sm.drain, 0, 10000000ull);
            }
        }
        __syncwarp();
    } else if (warp == TMA_WARP) {
        // ------------------------------------------------------------ TMA issuer
        // One lane issues every copy as soon as its buffer is free.  A copy
        // instruction can wait for the SM's copy engine, which is why this
        // is not the lane that issues the MMAs.
        //   K_gk -> stage gk&1      once S_{gk-2} is done
        //   V_gv -> stage gv&1      once PV_{gv-2} is done and, if tile gv-2
        //                           ended an item, that item's O staging in
        //                           the stage is read out (stg_free)
        //   Q of item qr            once item qr-1's Q is in TMEM (q_ready)
        // Probes are unambiguous by induction: the copy into a buffer one
        // use earlier waited for the phase before the one probed now.
        if ((tid & 31) == 0) {
            prefetch_tensormap(&p.tq);
            prefetch_tensormap(&p.tk);
            prefetch_tensormap(&p.tv);
            Ahead kq, vq, qq;
            kq.r = 0;
            kq.set(p, cta, G);
            vq = kq;
            qq = kq;
            int gk = 0, gv = 0;
            int stg_item[2] = {-1, -1};  // item whose O staging occupies V stage s
            uint64_t t_idle = 0;
            while (!failed && (kq.valid() || vq.valid() || qq.valid())) {
                bool progressed = false;
                // Q first: an item's first S needs Q and K_0, and at kernel
                // start every CTA's copies queue up at once.
                if (qq.valid() && (qq.r == 0 || mbar_test_wait(&sm.q_ready, (qq.r - 1) & 1))) {
                    const int sl = qq.slab(p);
                    const int q0 = (p.n_qtiles - 1 - qq.w / (p.B * p.H)) * BM;
                    mbar_arrive_expect_tx(&sm.q_full, C::Q_BYTES);
#pragma unroll
                    for (int bx = 0; bx < D / 32; ++bx)
                        tma_load_3d(sm.q + bx * C::Q_BOX_BYTES, &p.tq, (sl % p.H) * D + 32 * bx, q0, sl / p.H,
                                    &sm.q_full);
                    ++qq.r;
                    qq.set(p, cta, G);
                    progressed = true;
                }
                if (kq.valid() && (gk < 2 || mbar_test_wait(&sm.bar_s[gk & 1], ((gk - 2) >> 1) & 1))) {
                    const int sl = kq.slab(p);
                    if (gk != 0 || !p.withhold_first_key_load)
                        load_tile<D>(p.tk, sm.k[gk & 1], &sm.k_full[gk & 1], C::KV_BYTES, sl % p.H, kq.j * BN, sl / p.H);
                    ++gk;
                    kq.next(p, cta, G);
                    progressed = true;
                }
                if (vq.valid() && (gv < 2 || (mbar_test_wait(&sm.bar_o[gv & 1], ((gv - 2) >> 1) & 1) &&
                                              (stg_item[gv & 1] < 0 ||
                                               mbar_test_wait(&sm.stg_free, stg_item[gv & 1] & 1))))) {
                    stg_item[gv & 1] = -1;
                    if (vq.j + 1 == vq.n_kv) stg_item[gv & 1] = vq.r;
                    const int sl = vq.slab(p);
                    load_tile<D>(p.tv, sm.v[gv & 1], &sm.v_full[gv & 1], C::KV_BYTES, sl % p.H, vq.j * BN, sl / p.H);
                    ++gv;
                    vq.next(p, cta, G);
                    progressed = true;
                }
                if (progressed) {
                    t_idle = 0;
                } else {
                    // Idle: back off so the poll leaves the sub-partition's
                    // issue slots to the softmax warps.
                    const uint64_t now = globaltimer_ns();
                    if (t_idle == 0) t_idle = now;
                    else if (now - t_idle > p.wait_ns) failed = true;
                    __nanosleep(IDLE_NS);
                }
            }
            if (failed) {
                // Copies still landing complete before the CTA's shared memory
                // is released (bounded waits: 10 ms each).  Earlier copies into
                // a stage were consumed before the stage was reloaded.
                for (int t = max(0, gk - 2); t < gk; ++t) mbar_wait(&sm.k_full[t & 1], (t >> 1) & 1, 10000000ull);
                for (int t = max(0, gv - 2); t < gv; ++t) mbar_wait(&sm.v_full[t & 1], (t >> 1) & 1, 10000000ull);
                if (qq.r > 0) mbar_wait(&sm.q_full, (qq.r - 1) & 1, 10000000ull);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ softmax
        // Two threads per query row: warp w handles TMEM lanes 32*(w%4).. (rows)
        // and key columns 32*hf..32*hf+31 of each tile, hf = w/4 (the other
        // half of the row is warp w^4).  The halves exchange their row max
        // through shared memory once per tile and their row sums once per
        // item.  Waits are bounded; a failed one is reported at the next
        // barrier of the eight warps (named barrier 1), after which all of
        // them stop together.
        //
        // O accumulates in TMEM across an item's tiles (PV_g adds onto it).
        // The probabilities are exp2(s - mu) with mu a running row maximum
        // that is raised only when a tile's maximum exceeds it by more than
        // RESCALE_LOG2 (then O and l are scaled by exp2(mu_old - mu_new)
        // before PV_g), so P <= 2^RESCALE_LOG2 and O is rarely touched.
        const int hf = warp >> 2;
        const int rl = (warp & 3) * 32 + (tid & 31);  // row in the item's tile, TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        bool bad = false;
        // Columns (D/2)*hf.. of row rl of item rq's Q (scaled by
        // scale*log2(e)), from swizzled box hf (D = 64) or half hf of the one
        // box (D = 32), into TMEM lane rl.  Every S of the item before has
        // completed (the caller waited for the last one).
        auto load_q = [&](int rq) {
            bad |= !mbar_wait(&sm.q_full, rq & 1, p.wait_ns);
            constexpr int NC = D / 8;  // float4 chunks of this thread's half row
            const uint8_t* box = sm.q + (D == 64 ? hf * C::Q_BOX_BYTES : 0) + rl * 128;
            const int c0 = D == 64 ? 0 : 4 * hf;
            uint32_t qh[2 * NC], ql[2 * NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float4 x = *reinterpret_cast<const float4*>(box + (((c0 + c) ^ (rl & 7)) << 4));
                split2_x2(x.x * p.scale_log2, x.y * p.scale_log2, qh[2 * c], ql[2 * c]);
                split2_x2(x.z * p.scale_log2, x.w * p.scale_log2, qh[2 * c + 1], ql[2 * c + 1]);
            }
            if constexpr (D == 64) {
                tmem_st16(lane_base + tm + Q_HI + 16 * hf, qh);
                tmem_st16(lane_base + tm + Q_LO + 16 * hf, ql);
            } else {
                tmem_st8(lane_base + tm + Q_HI + 8 * hf, qh);
                tmem_st8(lane_base + tm + Q_LO + 8 * hf, ql);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&sm.q_ready);
        };
        int g = 0;  // the CTA's tile sequence number
        Seq it;
        it.r = 0;
        it.set_item(p, cta, G);
        for (int r = 0; it.valid(); ++r) {
            const int n_kv = it.n_kv;
            const int row = it.q0 + rl;
            Seq nx = it;
            ++nx.r;
            nx.set_item(p, cta, G);
            const bool has_next = nx.valid();

            // Item start (the CTA's first item only): convert K_0 and move
            // Q into TMEM.  Later items' K_0 and Q are converted during the
            // previous item's last tile, so their first S runs meanwhile.
            if (g == 0) {
                Tile kr;
                bad |= !mbar_wait(&sm.k_full[0], 0, p.wait_ns);
                kr.read(sm.k[0], tid);
                if (named_sync_or(1, NSM, bad)) {
                    failed = true;
                    break;
                }
                kr.write(sm.k[0], 1.f, tid);
                fence_async_smem();
                mbar_arrive(&sm.k_ready[0]);
                load_q(0);
            }

            float mu = -INFINITY, l = 0.f;  // l: this half's share of the row sum
            for (int j = 0; j < n_kv; ++j, ++g) {
                const int bf = g & 1;  // TMEM S buffer and K / V stages of tile g
                const int k0 = j * BN;

                // (1) Convert K_{g+1} (this item's next tile or the next
                // item's first), so S_{g+1} can run during this softmax.
                if (j + 1 < n_kv || has_next) {
                    const int gn = g + 1;
                    Tile kr;
                    bad |= !mbar_wait(&sm.k_full[gn & 1], (gn >> 1) & 1, p.wait_ns);
                    kr.read(sm.k[gn & 1], tid);
                    if (named_sync_or(1, NSM, bad)) {
                        failed = true;
                        break;
                    }
                    kr.write(sm.k[gn & 1], 1.f, tid);
                    fence_async_smem();
                    mbar_arrive(&sm.k_ready[gn & 1]);
                }

                // (2) Softmax of this half of S_g: row max (masked columns to
                // -inf, three-input maxima), combined with the other
                // half's; then the probabilities, packed bf16 hi / lo over the
                // 32 S columns just read (hi in the first 16, lo in the next).
                bad |= !mbar_wait(&sm.bar_s[bf], (g >> 1) & 1, p.wait_ns);
                tc_fence_after();
                // The item's last S is done, so its Q columns are free: move
                // the next item's Q in now (its first S then runs during this
                // softmax and the epilogue).
                if (j + 1 == n_kv && has_next) load_q(r + 1);
                const int kb = k0 + 32 * hf;  // first key of this half
                const bool need_mask = (p.causal && kb + 31 > it.q0) || kb + 32 > p.T;
                const uint32_t cs = lane_base + tm + col_s(bf) + 32 * hf;
                float sv[32];
                tmem_ld32(cs, sv);
                tmem_wait_ld();
                if (need_mask) {
                    const int nv = min(p.T - kb, p.causal ? row - kb + 1 : 32);
#pragma unroll
                    for (int i = 0; i < 32; ++i) sv[i] = (i < nv) ? sv[i] : -INFINITY;
                }
                float mx[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) mx[u] = max3(sv[u], sv[u + 8], sv[u + 16]);
#pragma unroll
                for (int u = 0; u < 4; ++u) mx[u] = max3(mx[u], mx[u + 4], sv[u + 24]);
                mx[0] = max3(mx[0], sv[28], sv[29]);
                mx[1] = max3(mx[1], sv[30], sv[31]);
                sm.red[bf][hf][rl] = fmaxf(max3(mx[0], mx[1], mx[2]), mx[3]);
                if (named_sync_or(1, NSM, bad)) {
                    failed = true;
                    break;
                }
                const float tmax = fmaxf(sm.red[bf][0][rl], sm.red[bf][1][rl]);
                // Raise mu on the item's first tile, or when this tile's max is
                // more than 2^RESCALE_LOG2 above it (both halves decide alike).
                float alpha = 1.f;
                if (j == 0 || tmax > mu + RESCALE_LOG2) {
                    const float mn = fmaxf(mu, tmax);
                    alpha = (j == 0 || mu == -INFINITY) ? 0.f : ex2(mu - mn);
                    mu = mn;
                }
                const float ms = (mu == -INFINITY) ? 0.f : mu;
                // Four packed partial sums (eight lanes); arguments and sums as
                // packed f32x2 operations.
                uint64_t acc2[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) acc2[u] = f2_pack(0.f, 0.f);
                {
                    const uint64_t ms2 = f2_pack(ms, ms);
                    uint32_t ph[16], pl[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float d0, d1;
                        f2_unpack(f2_sub(f2_pack(sv[i], sv[i + 1]), ms2), d0, d1);
                        const float e0 = ex2(d0), e1 = ex2(d1);
                        acc2[(i >> 1) & 3] = f2_add(acc2[(i >> 1) & 3], f2_pack(e0, e1));
                        split2_x2(e0, e1, ph[i / 2], pl[i / 2]);
                    }
                    tmem_st16(cs, ph);
                    tmem_st16(cs + 16, pl);
                }
                float r0, r1;
                f2_unpack(f2_add(f2_add(acc2[0], acc2[1]), f2_add(acc2[2], acc2[3])), r0, r1);
                const float rs = r0 + r1;
                l = (j == 0) ? rs : l * alpha + rs;

                // (3) Rescale this half of O if a row of this warp raised mu
                // (after PV_{g-1} has added onto it); convert V_g; then P_g, O
                // and V_g are ready for PV_g.
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    const int gp = g - 1;
                    bad |= !mbar_wait(&sm.bar_o[gp & 1], (gp >> 1) & 1, p.wait_ns);
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < D / 2; c += 16) {
                        float ov[16];
                        uint32_t ow[16];
                        tmem_ld16(lane_base + tm + COL_O + (D / 2) * hf + c, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) ow[i] = __float_as_uint(ov[i] * alpha);
                        tmem_st16(lane_base + tm + COL_O + (D / 2) * hf + c, ow);
                    }
                }
                tmem_wait_st();
                {
                    Tile vr;
                    bad |= !mbar_wait(&sm.v_full[bf], (g >> 1) & 1, p.wait_ns);
                    vr.read(sm.v[bf], tid);
                    if (named_sync_or(1, NSM, bad)) {
                        failed = true;
                        break;
                    }
                    vr.write(sm.v[bf], 1.f, tid);
                }
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(&sm.pv_ready[bf]);
            }
            if (failed) break;

            // The item's last P V; the row sum of both halves; normalise and
            // store O, staged through the last tile's V stage (its P V is
            // done; the producer reloads the stage only after stg_free), 64
            // rows at a time, float4 chunks XOR-swizzled by row, so that the
            // global stores are whole 256-byte rows.
            const int gl = g - 1;
            bad |= !mbar_wait(&sm.bar_o[gl & 1], (gl >> 1) & 1, p.wait_ns);
            tc_fence_after();
            sm.red[0][hf][rl] = l;
            if (named_sync_or(1, NSM, bad)) {
                failed = true;
                break;
            }
            const float lt = sm.red[0][0][rl] + sm.red[0][1][rl];
            const float inv = 1.f / lt;
            if (hf == 0 && row < p.T) p.lse[(static_cast<long>(it.b) * p.H + it.h) * p.T + row] = (mu + log2f(lt)) * kLn2;
            constexpr int NCH = D / 4;  // float4 chunks of an O row
            float4* stg = reinterpret_cast<float4*>(sm.v[gl & 1]);  // 64 rows x NCH float4 (the stage)
            float* og = p.o + static_cast<long>(it.b) * p.T * p.ld_o + it.h * D;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                // TMEM loads are warp-collective: every warp loads, the warps
                // of the rows in this half stage.
                {
                    float ov[D / 2];
                    if constexpr (D == 64) tmem_ld32(lane_base + tm + COL_O + 32 * hf, ov);
                    else tmem_ld16(lane_base + tm + COL_O + 16 * hf, ov);
                    tmem_wait_ld();
                    if ((rl >> 6) == half) {
                        const int rr = rl & 63;
#pragma unroll
                        for (int i = 0; i < D / 8; ++i) {
                            const int c4 = (D / 8) * hf + i;
                            stg[rr * NCH + (c4 ^ (rr & (NCH - 1)))] =
                                make_float4(ov[4 * i] * inv, ov[4 * i + 1] * inv, ov[4 * i + 2] * inv, ov[4 * i + 3] * inv);
                        }
                    }
                }
                named_sync(1, NSM);
#pragma unroll
                for (int k = 0; k < 64 * NCH / NSM; ++k) {
                    const int i = tid + k * NSM;
                    const int rr = i / NCH;
                    const int c4 = i % NCH;
                    const int qrow = it.q0 + 64 * half + rr;
                    if (qrow < p.T)
                        *reinterpret_cast<float4*>(og + static_cast<long>(qrow) * p.ld_o + c4 * 4) =
                            stg[rr * NCH + (c4 ^ (rr & (NCH - 1)))];
                }
                named_sync(1, NSM);
            }
            fence_async_smem();
            tc_fence_before();  // the next item's first P V overwrites the O columns just read
            mbar_arrive(&sm.stg_free);
            it = nx;
        }
    }

    if (__syncthreads_or(failed) && tid == 0) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, TMEM_COLS);
}

__global__ void __launch_bounds__(NTHREADS, 2) attn_fwd_tc64(const __grid_constant__ Params p) { fwd_body<64>(p); }
__global__ void __launch_bounds__(NTHREADS, 2) attn_fwd_tc32(const __grid_constant__ Params p) { fwd_body<32>(p); }

}  // namespace

namespace {

using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link-time dependency on the driver library).
EncodeTiled encode_tiled() {
    static const EncodeTiled fn = []() -> EncodeTiled {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiled>(f);
    }();
    return fn;
}

}  // namespace

bool encode_rows(CUtensorMap* map, const float* base, long ld, int B, int T, int H, int d, int box_cols, int box_rows,
                 CUtensorMapSwizzle swizzle) {
    const EncodeTiled fn = encode_tiled();
    if (fn == nullptr) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(H) * d, static_cast<cuuint64_t>(T),
                                static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(ld) * 4 * T};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_2d(CUtensorMap* map, const float* base, long cols, long rows, long ld, int box_cols, int box_rows) {
    const EncodeTiled fn = encode_tiled();
    if (fn == nullptr || cols <= 0 || rows <= 0) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_2d_bf16(CUtensorMap* map, const uint16_t* base, long cols, long rows, long ld, int box_cols, int box_rows,
                    CUtensorMapSwizzle swizzle) {
    const EncodeTiled fn = encode_tiled();
    if (fn == nullptr || cols <= 0 || rows <= 0) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t elem[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool fwd_tc_supported(const FwdArgs& a) { return a.d == 64 || a.d == 32; }

cudaError_t launch_fwd_tc(const FwdArgs& a, int num_sms, int* status, cudaStream_t stream, int* launches) {
    if (!fwd_tc_supported(a)) return cudaErrorInvalidValue;
    const int D = a.d;
    Params p;
    if (!encode_rows(&p.tq, a.q, a.ld_qkv, a.B, a.T, a.H, D, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_rows(&p.tk, a.k, a.ld_qkv, a.B, a.T, a.H, D, D, BN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_rows(&p.tv, a.v, a.ld_qkv, a.B, a.T, a.H, D, D, BN, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    p.o = a.o;
    p.ld_o = a.ld_o;
    p.lse = a.lse;
    p.status = status;
    p.wait_ns = a.wait_ns;
    p.withhold_first_key_load = a.withhold_first_key_load;
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
    const size_t smem = (D == 64 ? sizeof(Smem<64>) : sizeof(Smem<32>)) + 1024;
    auto kernel = D == 64 ? attn_fwd_tc64 : attn_fwd_tc32;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_done{0};  // one bit per device and head_dim: the attribute is per device
    const uint64_t bit = 1ull << ((2 * dev + (D == 32 ? 1 : 0)) & 63);
    if (!(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    // Persistent: two CTAs per SM (shared memory and TMEM allow two), each
    // walking its items in the snake order.
    const long slots = 2L * (num_sms > 0 ? num_sms : 148);
    const int grid = static_cast<int>(n_work < slots ? n_work : slots);
    e = launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(NTHREADS), smem, stream, p);
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
