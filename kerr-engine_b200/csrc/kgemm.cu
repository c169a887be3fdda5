// Dense f32 GEMM on the 5th-generation tensor cores (sm_100a) for the
// attention projections c_attn / c_proj (kproj.cu): C (+)= A B^T with
// A(m, k) and B(n, k) read from row-major f32 buffers in either orientation.
//
// Numerics: every f32 operand element x is split into bf16 hi = bf16(x) and
// lo = bf16(x - hi); each k-step accumulates hi*hi + hi*lo + lo*hi in f32 in
// tensor memory (relative error ~1e-5 against an f32 loop, where a single
// bf16 or tf32 product gives ~1e-3).
//
// Operand paths (the three products of a k-step read B from shared memory
// only, so the tensor core's shared-memory reads stay at 2/3 of an SS MMA's):
//   B  split once per call by gemm_split_planes into a bf16 hi plane and a
//      lo plane (the weight W, or x for the dW product), which TMA copies
//      straight into the 128B-swizzled UMMA layout (K-major tiles: 64 bf16
//      per row; MN-major ones: 64-column atoms).
//   A  read as f32 from global memory by the A warps, split in registers and
//      stored into tensor memory with tcgen05.st, where the MMAs read it
//      (A from TMEM: row m in lane m, two bf16 per column).
// An operand is "K-major" when K runs along the memory rows (x, W of the
// forward, dy of the dx product) and "MN-major" when M or N does (W of the
// dx product, dy and x of the dW product).
//
// Tiles: 128 (M) x 192 (N) per unit, K in 64-wide stages (12 MMAs per
// stage: the issuing thread waits on one barrier per 12 MMAs, since every
// barrier wait between MMAs leaves the tensor pipe idle).  Tensor memory: two
// 192-column accumulators (the epilogue drains one while the next unit
// accumulates into the other) and two 64-column A stages (32 columns hi, 32
// lo) beside them; four B stages in shared memory.  Units are (tile, K split); with fewer tiles than
// SMs the K range is split and the partial tiles are summed in a fixed order
// by gemm_split_sum, so results do not depend on scheduling.
//
// Warp roles (448 threads, one CTA per SM, persistent over units):
//   warps 0-7   A warps: warp w fills TMEM lanes 32*(w%4).. of each stage
//               (K-major A through the 16x256b store shape, so that four
//               lanes share a row and the loads are 64-byte row segments),
//               loads issued one stage ahead; they arrive on the stage's
//               barrier once its B copy has landed too
//   warps 8-11  epilogue: accumulator b (TMEM) -> C, through a per-warp
//               shared staging area so that stores are whole rows
//   warp 12     one lane issues the MMAs (12 per stage) and commits
//   warp 13     one lane issues the TMA copies of B
// Every wait is bounded (wait_ns of wall time); a role whose wait runs out
// leaves its loop, copies and MMAs in flight are drained, the status word set.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "kattn_common.cuh"
#include "kattn_launch.h"
#include "sm100.cuh"
#include "tma_map.h"

namespace kattn {
using namespace sm100;

namespace {

constexpr int GM = 128;  // tile rows (MMA M)
constexpr int GN = 192;  // tile columns (MMA N)
constexpr int GK = 64;   // K per stage
constexpr int NA = 256;  // A threads
constexpr int NEPI = 128;
constexpr int G_MMA_WARP = (NA + NEPI) / 32;
constexpr int G_TMA_WARP = G_MMA_WARP + 1;
constexpr int G_THREADS = NA + NEPI + 64;
constexpr int A_STAGES = 2;                 // A stages in TMEM (64 columns each)
constexpr int B_STAGES = 4;                 // B stages in shared memory
constexpr uint32_t B_HALF = GN * GK * 2;    // one plane's tile: 24 KB
constexpr uint32_t B_BYTES = 2 * B_HALF;    // hi | lo
constexpr uint32_t MN_BOX = 64 * GK * 2;    // MN-major box: 64 columns x GK rows of bf16 (8 KB)
constexpr int EPI_PITCH = 36;               // floats per staged row (conflict-free float4 access)
constexpr uint32_t G_TMEM_COLS = 512;
constexpr unsigned long long G_DRAIN_NS = 10000000ull;

static_assert(GN % 64 == 0 && GN <= 256 && GN % 16 == 0, "tile width");

// TMEM columns: accumulator b at 256*b (GN wide); A stage s at a_col(s)
// (hi k 0..63 in 32 columns at +0, lo at +32), in the 64 columns each
// accumulator leaves free.
__host__ __device__ constexpr uint32_t acc_col(int b) { return 256u * static_cast<uint32_t>(b); }
__host__ __device__ constexpr uint32_t a_col(int s) { return 256u * static_cast<uint32_t>(s) + GN; }
static_assert(GN + GK <= 256 && A_STAGES == 2, "an A stage fits beside each accumulator");

struct alignas(1024) GSmem {
    uint8_t b[B_STAGES][B_BYTES];
    float epi[NEPI / 32][32 * EPI_PITCH];  // per epilogue warp: 32 rows x 32 columns
    uint64_t b_full[B_STAGES];  // B stage landed
    uint64_t done[B_STAGES];    // stage g's MMAs complete (ring slot g % B_STAGES)
    uint64_t a_full[A_STAGES];  // A stage stored in TMEM and its B landed
    uint64_t acc_full[2];       // accumulator b complete
    uint64_t acc_free[2];       // accumulator b read out
    uint64_t drain;
    uint32_t tmem_slot;
};

static_assert(sizeof(GSmem) + 1024 <= 232448, "shared memory (plus alignment slack) exceeds 227 KB");

struct alignas(64) GParams {
    CUtensorMap tb_hi, tb_lo;  // B planes: K-major {K, N} box {32, GN}; MN-major {N, K} box {64, 32}
    const float* a;            // A: K-major a[m * lda + k]; MN-major a[k * lda + m]
    long lda;
    float* c;
    long ldc;
    const float* bias;  // [N] or null (added when the unit writes C)
    float* part;        // split partials [splits][M][N] (row stride N), or null
    int M, N, K;
    int m_tiles, n_tiles, splits, stages_per_split, k_stages, n_units;
    int accumulate;  // C += result (splits == 1 only)
    int* status;
    unsigned long long wait_ns;
};

// Unit u: tile (u / splits) in row-major tile order, K split (u % splits).
struct Unit {
    int m0, n0, s, st0, n_st;
};

__device__ __forceinline__ Unit make_unit(const GParams& p, int u) {
    Unit x;
    const int t = u / p.splits;
    x.s = u - t * p.splits;
    const int mt = t / p.n_tiles;
    x.m0 = mt * GM;
    x.n0 = (t - mt * p.n_tiles) * GN;
    x.st0 = x.s * p.stages_per_split;
    x.n_st = min(p.stages_per_split, p.k_stages - x.st0);
    return x;
}

// Walks this CTA's stages in order: unit u (c, c+G, ...), stage j of it.
struct StageCursor {
    int u, j;
    Unit x;
    __device__ __forceinline__ void start(const GParams& p, int c) {
        u = c;
        j = 0;
        if (u < p.n_units) x = make_unit(p, u);
    }
    __device__ __forceinline__ bool valid(const GParams& p) const { return u < p.n_units; }
    __device__ __forceinline__ void next(const GParams& p, int G) {
        if (++j >= x.n_st) {
            j = 0;
            u += G;
            if (u < p.n_units) x = make_unit(p, u);
        }
    }
};

// tcgen05.st.16x256b.x2: 16 TMEM lanes x 16 columns; thread t supplies
// lanes t/4 (registers 0-1, 4-5) and t/4 + 8 (2-3, 6-7), columns 2(t%4),
// 2(t%4)+1 (registers 0-3) and those + 8 (4-7).
__device__ __forceinline__ void tmem_st_16x256b_x2(uint32_t ta, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(ta), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

// This thread's 32 A elements of a stage (zeros outside M x K; K-major rows
// have K a multiple of 4, so a float4 is wholly in or out).
//   K-major: warp (q, h) owns the 16 tile rows 32q + 16h ..; lane t loads
//     rows a = +t/4 and b = +t/4+8 at k = 4(t%4) + 16j, j = 0..3 (eight
//     float4: each load instruction reads 64 contiguous bytes of 8 rows), in
//     16x256b fragment order: float4 i is row (i&1 ? b : a), k-chunk i>>1,
//     so that r[0..15] fill columns 0..15 (k 0..31) and r[16..31] columns
//     16..31 (k 32..63) of each plane.
//   MN-major: lane t owns tile row 32q + t (consecutive lanes read
//     consecutive addresses) and k = 32h .. 32h+31, for tcgen05.st.32x32b.
template <bool A_MN>
__device__ __forceinline__ void load_a(const GParams& p, int m0, int q, int h, int lane, int k0, float (&r)[32]) {
    if (A_MN) {
        const int m = m0 + 32 * q + lane;
        const bool in_m = m < p.M;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int k = k0 + 32 * h + i;
            r[i] = (in_m && k < p.K) ? __ldg(p.a + static_cast<long>(k) * p.lda + m) : 0.f;
        }
    } else {
        const int ma = m0 + 32 * q + 16 * h + (lane >> 2);
        const int kc = k0 + 4 * (lane & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = ma + 8 * (i & 1);
            const int k = kc + 16 * (i >> 1);
            const float4 v = (m < p.M && k < p.K)
                                 ? __ldg(reinterpret_cast<const float4*>(p.a + static_cast<long>(m) * p.lda + k))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            r[4 * i] = v.x;
            r[4 * i + 1] = v.y;
            r[4 * i + 2] = v.z;
            r[4 * i + 3] = v.w;
        }
    }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(G_THREADS, 1) gemm_bf16x3(const __grid_constant__ GParams p) {
    // The next grid may launch at once (it waits for this one before it
    // touches memory); this grid's setup below touches no global memory, so
    // it runs while the grid before still drains, and every thread waits
    // for that grid (griddepcontrol.wait) before its first global access.
    pdl_launch();
    extern __shared__ uint8_t smem_raw[];
    GSmem& sm = *reinterpret_cast<GSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int c = static_cast<int>(blockIdx.x);
    const int G = static_cast<int>(gridDim.x);

    if (warp == 0) {
        tmem_alloc(&sm.tmem_slot, G_TMEM_COLS);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < B_STAGES; ++i) {
            mbar_init(&sm.b_full[i], 1);
            mbar_init(&sm.done[i], 1);
        }
        for (int i = 0; i < A_STAGES; ++i) mbar_init(&sm.a_full[i], NA);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.acc_full[i], 1);
            mbar_init(&sm.acc_free[i], NEPI);
        }
        mbar_init(&sm.drain, 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_wait();
    const uint32_t tm = sm.tmem_slot;
    bool failed = false;

    if (warp == G_TMA_WARP) {
        // ------------------------------------------------------------ TMA issuer (B)
        if (lane == 0) {
            prefetch_tensormap(&p.tb_hi);
            prefetch_tensormap(&p.tb_lo);
            StageCursor cur;
            cur.start(p, c);
            int g = 0;
            for (; cur.valid(p) && !failed; ++g, cur.next(p, G)) {
                const int s = g % B_STAGES;
                if (g >= B_STAGES && !mbar_wait(&sm.done[s], ((g - B_STAGES) / B_STAGES) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                const int k0 = (cur.x.st0 + cur.j) * GK;
                const int n0 = cur.x.n0;
                mbar_arrive_expect_tx(&sm.b_full[s], B_BYTES);
                if (B_MN) {
#pragma unroll
                    for (int a = 0; a < GN / 64; ++a) {
                        tma_load_2d(sm.b[s] + a * MN_BOX, &p.tb_hi, n0 + 64 * a, k0, &sm.b_full[s]);
                        tma_load_2d(sm.b[s] + B_HALF + a * MN_BOX, &p.tb_lo, n0 + 64 * a, k0, &sm.b_full[s]);
                    }
                } else {
                    tma_load_2d(sm.b[s], &p.tb_hi, k0, n0, &sm.b_full[s]);
                    tma_load_2d(sm.b[s] + B_HALF, &p.tb_lo, k0, n0, &sm.b_full[s]);
                }
            }
            if (failed)  // copies still landing complete before the shared memory is released
                for (int t = max(0, g - B_STAGES); t < g; ++t)
                    mbar_wait(&sm.b_full[t % B_STAGES], (t / B_STAGES) & 1, G_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == G_MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(GM, GN, 0, B_MN ? 1 : 0);
            // K-major B: 128-byte rows (128B swizzle, 1024-byte atoms), k-step
            // 32 bytes; MN-major: 64-column atoms GK rows apart (lbo), k-step
            // 16 rows (2048 bytes).  One barrier per stage: the A warps arrive
            // on a_full only after the stage's B has landed.
            constexpr uint32_t B_KSTEP = B_MN ? 2048 : 32;
            int g = 0, i = 0;
            for (int u = c; u < p.n_units && !failed; u += G, ++i) {
                const Unit x = make_unit(p, u);
                const int b = i & 1;
                if (i >= 2 && !mbar_wait(&sm.acc_free[b], ((i - 2) >> 1) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tm + acc_col(b);
                for (int j = 0; j < x.n_st; ++j, ++g) {
                    const int sa = g % A_STAGES, s = g % B_STAGES;
                    if (!mbar_wait(&sm.a_full[sa], (g / A_STAGES) & 1, p.wait_ns)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sb = smem_u32(sm.b[s]);
                    const uint64_t bh = B_MN ? smem_desc(sb, MN_BOX, 1024) : smem_desc(sb, 16, 1024);
                    const uint64_t bl = B_MN ? smem_desc(sb + B_HALF, MN_BOX, 1024) : smem_desc(sb + B_HALF, 16, 1024);
                    const uint32_t ah = tm + a_col(sa), al = ah + GK / 2;
#pragma unroll
                    for (int ks = 0; ks < GK / 16; ++ks) {
                        const uint32_t ob = ks * B_KSTEP;
                        mma_ts(acc, ah + 8 * ks, desc_add(bh, ob), idesc, (j > 0 || ks > 0) ? 1u : 0u);
                        mma_ts(acc, ah + 8 * ks, desc_add(bl, ob), idesc, 1);
                        mma_ts(acc, al + 8 * ks, desc_add(bh, ob), idesc, 1);
                    }
                    mma_commit(&sm.done[s]);  // one commit per stage: back-to-back commits stall the MMA pipe
                }
                if (failed) break;
                mma_commit(&sm.acc_full[b]);
            }
            if (failed) {
                mma_commit(&sm.drain);
                mbar_wait(&sm.drain, 0, G_DRAIN_NS);
            }
        }
        __syncwarp();
    } else if (warp >= NA / 32) {
        // ------------------------------------------------------------ epilogue
        // Warp e (lane quadrant e) owns tile rows 32e..32e+31.  Per 32-column
        // chunk: TMEM -> registers -> the warp's staging rows -> whole-row
        // float4 stores (8 lanes per 128-byte row segment).
        const int e = warp - NA / 32;
        const uint32_t lb = static_cast<uint32_t>(e * 32) << 16;
        float* stg = sm.epi[e];
        int i = 0;
        for (int u = c; u < p.n_units && !failed; u += G, ++i) {
            const Unit x = make_unit(p, u);
            const int b = i & 1;
            if (!mbar_wait_warp(&sm.acc_full[b], (i >> 1) & 1, p.wait_ns)) {
                failed = true;
                break;
            }
            tc_fence_after();
            const bool direct = p.splits == 1;
            float* dst = direct ? p.c : p.part + static_cast<long>(x.s) * p.M * p.N;
            const long ld = direct ? p.ldc : p.N;
            for (int ch = 0; ch < GN / 32; ++ch) {
                const int n_base = x.n0 + 32 * ch;
                if (n_base >= p.N) break;  // warp-uniform
                float v[32];
                tmem_ld32(lb + tm + acc_col(b) + 32 * ch, v);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    *reinterpret_cast<float4*>(stg + lane * EPI_PITCH + 4 * q) =
                        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                __syncwarp();
                const int n = n_base + 4 * (lane & 7);
                float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
                if (direct && p.bias && n < p.N)  // 4-byte aligned only: scalar loads
                    bb = make_float4(p.bias[n], p.bias[n + 1], p.bias[n + 2], p.bias[n + 3]);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int rr = 4 * q + (lane >> 3);
                    const int m = x.m0 + 32 * e + rr;
                    if (m < p.M && n < p.N) {
                        float4 r = *reinterpret_cast<const float4*>(stg + rr * EPI_PITCH + 4 * (lane & 7));
                        float* o = dst + static_cast<long>(m) * ld + n;
                        if (direct) {
                            r.x += bb.x;
                            r.y += bb.y;
                            r.z += bb.z;
                            r.w += bb.w;
                            if (p.accumulate) {
                                const float4 old = *reinterpret_cast<const float4*>(o);
                                r.x += old.x;
                                r.y += old.y;
                                r.z += old.z;
                                r.w += old.w;
                            }
                        }
                        *reinterpret_cast<float4*>(o) = r;
                    }
                }
                __syncwarp();
            }
            tc_fence_before();
            mbar_arrive(&sm.acc_free[b]);
        }
    } else {
        // ------------------------------------------------------------ A warps
        // Warp w: TMEM lane quadrant q = w%4, half h = w/4 (the 16-lane group
        // 32q + 16h of K-major A; k 32h .. 32h+31 of MN-major A, see load_a).
        // Loads run one stage ahead of the stage being stored; a stage's TMEM
        // columns are stored once the MMAs that read them last have
        // completed.
        const int q = warp & 3, h = warp >> 2;
        const uint32_t lb = static_cast<uint32_t>(32 * q) << 16;
        float r0[32], r1[32];
        StageCursor ld_cur, st_cur;
        ld_cur.start(p, c);
        st_cur.start(p, c);
        auto load_next = [&](float (&r)[32]) {
            if (ld_cur.valid(p)) {
                load_a<A_MN>(p, ld_cur.x.m0, q, h, lane, (ld_cur.x.st0 + ld_cur.j) * GK, r);
                ld_cur.next(p, G);
            }
        };
        int g = 0;
        // Stage g from `cur` (loaded one stage earlier); stage g + 1 loaded
        // into `nxt`.  False when the CTA's stages are done or a wait failed.
        auto step = [&](float (&cur)[32], float (&nxt)[32]) -> bool {
            if (!st_cur.valid(p) || failed) return false;
            load_next(nxt);
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) split2(cur[2 * i], cur[2 * i + 1], hi[i], lo[i]);
            // A stage s was last read by the MMAs of stage g - A_STAGES (done
            // slot (g - A_STAGES) % B_STAGES), which cannot complete again
            // before stage g's A is stored.
            const int s = g % A_STAGES;
            const int gp = g - A_STAGES;
            if (g >= A_STAGES && !mbar_wait_warp(&sm.done[gp % B_STAGES], (gp / B_STAGES) & 1, p.wait_ns)) {
                failed = true;
                return false;
            }
            tc_fence_after();
            if (A_MN) {
                const uint32_t col = lb + tm + a_col(s) + 16 * h;
                tmem_st16(col, *reinterpret_cast<const uint32_t(*)[16]>(hi));
                tmem_st16(col + GK / 2, *reinterpret_cast<const uint32_t(*)[16]>(lo));
            } else {
                const uint32_t col = lb + (static_cast<uint32_t>(16 * h) << 16) + tm + a_col(s);
                tmem_st_16x256b_x2(col, *reinterpret_cast<const uint32_t(*)[8]>(hi));
                tmem_st_16x256b_x2(col + 16, *reinterpret_cast<const uint32_t(*)[8]>(hi + 8));
                tmem_st_16x256b_x2(col + GK / 2, *reinterpret_cast<const uint32_t(*)[8]>(lo));
                tmem_st_16x256b_x2(col + GK / 2 + 16, *reinterpret_cast<const uint32_t(*)[8]>(lo + 8));
            }
            tmem_wait_st();
            // One thread also waits for the stage's B copy, so that a_full
            // completing implies both operands are in place.
            if (tid == 0 && !mbar_wait(&sm.b_full[g % B_STAGES], (g / B_STAGES) & 1, p.wait_ns)) failed = true;
            if (__any_sync(0xffffffffu, failed)) {
                failed = true;
                return false;
            }
            tc_fence_before();
            mbar_arrive(&sm.a_full[s]);
            ++g;
            st_cur.next(p, G);
            return true;
        };
        load_next(r0);
        while (step(r0, r1) && step(r1, r0)) {
        }
    }

    if (__syncthreads_or(failed) && tid == 0) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, G_TMEM_COLS);
}

// Splits a row-major f32 matrix [rows][cols] (row stride ld, cols and ld
// multiples of 4) into bf16 planes hi = bf16(x), lo = bf16(x - hi), each
// [rows][pitch] (pitch a multiple of 8 >= cols).
__global__ void __launch_bounds__(256) gemm_split_planes(const float* x, long ld, long rows, int cols, int pitch,
                                                         uint2* hi, uint2* lo) {
    pdl_enter();
    const int c4 = cols / 4;
    const long total = rows * c4;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / c4;
        const int k = 4 * static_cast<int>(i - r * c4);
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + r * ld + k));
        uint2 h, l;
        split2(v.x, v.y, h.x, l.x);
        split2(v.z, v.w, h.y, l.y);
        const long o = (r * pitch + k) / 4;
        hi[o] = h;
        lo[o] = l;
    }
}

// C[m][n] = (accumulate ? C[m][n] : 0) + bias[n] + sum_s part[s][m][n], the
// split partials added in split order (deterministic).  float4 per thread.
__global__ void __launch_bounds__(256) gemm_split_sum(float* c, long ldc, const float* part, const float* bias, int M,
                                                      int N, int splits, int accumulate) {
    pdl_enter();
    const int n4 = N / 4;
    const long total = static_cast<long>(M) * n4;
    const long plane = static_cast<long>(M) * N;
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long m = i / n4;
        const int n = 4 * static_cast<int>(i - m * n4);
        float4 r = bias ? make_float4(bias[n], bias[n + 1], bias[n + 2], bias[n + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (accumulate) {
            const float4 o = *reinterpret_cast<const float4*>(c + m * ldc + n);
            r.x += o.x;
            r.y += o.y;
            r.z += o.z;
            r.w += o.w;
        }
        for (int s = 0; s < splits; ++s) {
            const float4 q = *reinterpret_cast<const float4*>(part + s * plane + m * N + n);
            r.x += q.x;
            r.y += q.y;
            r.z += q.z;
            r.w += q.w;
        }
        *reinterpret_cast<float4*>(c + m * ldc + n) = r;
    }
}

template <bool A_MN, bool B_MN>
cudaError_t launch_gemm_t(const GParams& p, int grid, cudaStream_t s) {
    static std::atomic<uint64_t> attr_done{0};  // one bit per device: the attribute is per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t smem = sizeof(GSmem) + 1024;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(gemm_bf16x3<A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    return launch_pdl(gemm_bf16x3<A_MN, B_MN>, dim3(static_cast<unsigned>(grid)), dim3(G_THREADS), smem, s, p);
}

}  // namespace

ProjStatus gemm_tc(cudaStream_t s, cudaMemPool_t pool, int num_sms, const float* a, long lda, bool a_mn,
                   const float* b, long ldb, bool b_mn, float* c, long ldc, const float* bias, int M, int N, int K,
                   int accumulate, int* status, unsigned long long wait_ns, int* launches) {
    ProjStatus st;
    auto fail = [&](cudaError_t e, const char* what) {
        st.cuda = e;
        st.what = what;
        return st;
    };
    // float4 access: C rows and B rows (N or K wide) and K-major A rows.
    if (M <= 0 || N <= 0 || K <= 0 || N % 4 != 0 || (b_mn ? N : K) % 4 != 0 || (!a_mn && K % 4 != 0))
        return fail(cudaErrorInvalidValue, "GEMM shape");
    const int sms = num_sms > 0 ? num_sms : 148;
    GParams p;
    p.a = a;
    p.lda = lda;
    p.c = c;
    p.ldc = ldc;
    p.bias = bias;
    p.M = M;
    p.N = N;
    p.K = K;
    p.m_tiles = (M + GM - 1) / GM;
    p.n_tiles = (N + GN - 1) / GN;
    p.k_stages = (K + GK - 1) / GK;
    const long tiles = static_cast<long>(p.m_tiles) * p.n_tiles;
    // Split K while the tiles alone leave at least half the SMs idle (the
    // partial sums cost a write and a read of splits x M x N floats), keeping
    // >= 4 stages (256 of K) per split so that the ring fills.
    int splits = 1;
    if (2 * tiles <= sms) splits = static_cast<int>(std::min<long>((sms + tiles - 1) / tiles, std::max(1, p.k_stages / 4)));
    splits = std::min(splits, 8);
    p.stages_per_split = (p.k_stages + splits - 1) / splits;
    p.splits = (p.k_stages + p.stages_per_split - 1) / p.stages_per_split;
    const long n_units = tiles * p.splits;
    if (n_units > INT32_MAX) return fail(cudaErrorInvalidValue, "GEMM too large");
    p.n_units = static_cast<int>(n_units);
    p.accumulate = accumulate;
    p.status = status;
    p.wait_ns = wait_ns;
    p.part = nullptr;

    // B as a row-major matrix: K-major b[n * ldb + k] is [N][K], MN-major
    // b[k * ldb + n] is [K][N]; its planes have the same shape at a pitch
    // that is a multiple of 8 bf16 (16-byte TMA row strides).
    const long b_rows = b_mn ? K : N, b_cols = b_mn ? N : K;
    const long pitch = (b_cols + 7) / 8 * 8;
    const size_t plane = sizeof(uint16_t) * static_cast<size_t>(b_rows) * pitch;
    uint16_t* planes = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&planes), 2 * plane, pool, s);
    if (e != cudaSuccess) return fail(e, "GEMM operand planes");
    uint16_t* hi = planes;
    uint16_t* lo = planes + plane / sizeof(uint16_t);
    const bool ok = b_mn ? encode_2d_bf16(&p.tb_hi, hi, b_cols, b_rows, pitch, 64, GK, CU_TENSOR_MAP_SWIZZLE_128B) &&
                               encode_2d_bf16(&p.tb_lo, lo, b_cols, b_rows, pitch, 64, GK, CU_TENSOR_MAP_SWIZZLE_128B)
                         : encode_2d_bf16(&p.tb_hi, hi, b_cols, b_rows, pitch, GK, GN, CU_TENSOR_MAP_SWIZZLE_128B) &&
                               encode_2d_bf16(&p.tb_lo, lo, b_cols, b_rows, pitch, GK, GN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) e = cudaErrorInvalidValue;
    const char* what = ok ? "GEMM launch" : "GEMM tensor maps";
    if (e == cudaSuccess && p.splits > 1) {
        e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&p.part), sizeof(float) * static_cast<size_t>(p.splits) * M * N,
                                    pool, s);
        if (e != cudaSuccess) what = "GEMM split workspace";
    }
    if (e == cudaSuccess) {
        const long n4 = b_rows * (b_cols / 4);
        const int pgrid = static_cast<int>(std::min<long>((n4 + 255) / 256, 8L * sms));
        e = launch_pdl(gemm_split_planes, dim3(static_cast<unsigned>(pgrid)), dim3(256), 0, s, b, ldb, b_rows,
                       static_cast<int>(b_cols), static_cast<int>(pitch), reinterpret_cast<uint2*>(hi),
                       reinterpret_cast<uint2*>(lo));
        if (e == cudaSuccess) *launches += 1;
    }
    if (e == cudaSuccess) {
        const int grid = static_cast<int>(std::min<long>(n_units, sms));
        if (a_mn && b_mn) e = launch_gemm_t<true, true>(p, grid, s);
        else if (a_mn) e = launch_gemm_t<true, false>(p, grid, s);
        else if (b_mn) e = launch_gemm_t<false, true>(p, grid, s);
        else e = launch_gemm_t<false, false>(p, grid, s);
        if (e == cudaSuccess) *launches += 1;
    }
    if (e == cudaSuccess && p.splits > 1) {
        const long n4 = static_cast<long>(M) * (N / 4);
        const int sgrid = static_cast<int>(std::min<long>((n4 + 255) / 256, 8L * sms));
        e = launch_pdl(gemm_split_sum, dim3(static_cast<unsigned>(sgrid)), dim3(256), 0, s, c, ldc,
                       static_cast<const float*>(p.part), bias, M, N, p.splits, accumulate);
        if (e == cudaSuccess) *launches += 1;
    }
    if (p.part) {
        const cudaError_t ef = cudaFreeAsync(p.part, s);
        if (e == cudaSuccess) e = ef;
    }
    {
        const cudaError_t ef = cudaFreeAsync(planes, s);
        if (e == cudaSuccess) e = ef;
    }
    if (e != cudaSuccess) return fail(e, what);
    return st;
}

}  // namespace kattn
