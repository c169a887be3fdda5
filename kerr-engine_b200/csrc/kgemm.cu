// Dense f32 GEMM on the 5th-generation tensor cores (sm_100a) for the
// attention projections c_attn / c_proj (kproj.cu): C (+)= A B^T with
// A(m, k) and B(n, k) read from row-major f32 buffers in either orientation.
//
// Numerics: every f32 operand element x is split into bf16 hi = bf16(x) and
// lo = bf16(x - hi); each k-step accumulates hi*hi + hi*lo + lo*hi in f32 in
// tensor memory (relative error ~1e-5 against an f32 loop, where a single
// bf16 or tf32 product gives ~1e-3).  The split happens on chip: TMA copies
// raw f32 tiles into shared memory and the converter warps rewrite them in
// place as bf16 hi / lo halves in the 128B-swizzled UMMA layout, so no split
// copy of an operand goes through HBM.
//
// Tiles: 128 (M) x 256 (N) per unit, K in 32-wide stages (A 16 KB + B 32 KB
// raw per stage, four stages, so that a stage's copy and conversion overlap
// the MMAs of the three before it).  K-major operands are converted into the
// 64B-swizzled layout (32 bf16 per row), MN-major ones into 128B-swizzled
// atoms of 64 columns.  An operand is "K-major" when K runs along the
// memory rows (x, W of the forward, dy of the dx product) and "MN-major" when
// M or N does (W of the dx product, dy and x of the dW product); the two
// orientations differ in the TMA box, the in-place rewrite and the MMA
// descriptor, not in the pipeline.  Units are (tile, K split); with fewer
// tiles than SMs the K range is split and the partial tiles are summed in a
// fixed order by gemm_split_sum, so results do not depend on scheduling.
//
// Warp roles (448 threads, one CTA per SM, persistent over units):
//   warps 0-7   converters: f32 stage -> bf16 hi / lo in place
//   warps 8-11  epilogue: accumulator b (TMEM, double-buffered) -> C, through
//               a per-warp shared staging area so that stores are whole rows
//   warp 12     one lane issues the MMAs (12 per stage) and commits
//   warp 13     one lane issues the TMA copies
// Every wait is bounded (wait_ns of wall time); a role whose wait runs out
// leaves its loop, copies and MMAs in flight are drained, the status word set.
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

constexpr int GM = 128;  // tile rows (MMA M)
constexpr int GN = 256;  // tile columns (MMA N)
constexpr int GK = 32;   // K per stage
constexpr int NCONV = 256;
constexpr int NEPI = 128;
constexpr int G_MMA_WARP = (NCONV + NEPI) / 32;
constexpr int G_TMA_WARP = G_MMA_WARP + 1;
constexpr int G_THREADS = NCONV + NEPI + 64;
constexpr int G_STAGES = 4;
constexpr uint32_t A_BYTES = GM * GK * 4;  // raw f32 A stage; later hi (8 KB) | lo
constexpr uint32_t B_BYTES = GN * GK * 4;  // raw f32 B stage; later hi (16 KB) | lo
constexpr int EPI_PITCH = 36;              // floats per staged row (conflict-free float4 access)
constexpr uint32_t G_TMEM_COLS = 512;      // two 256-column accumulators
constexpr unsigned long long G_DRAIN_NS = 10000000ull;

struct alignas(1024) GSmem {
    uint8_t a[G_STAGES][A_BYTES];
    uint8_t b[G_STAGES][B_BYTES];
    float epi[NEPI / 32][32 * EPI_PITCH];  // per epilogue warp: 32 rows x 32 columns
    uint64_t full[G_STAGES];    // stage landed
    uint64_t read_a[G_STAGES];  // every converter thread holds its share of the raw A tile
    uint64_t read_b[G_STAGES];  // ... of the raw B tile
    uint64_t ready[G_STAGES];   // stage converted
    uint64_t empty[G_STAGES];   // stage's MMAs done
    uint64_t acc_full[2];       // accumulator b complete
    uint64_t acc_free[2];       // accumulator b read out
    uint64_t drain;
    uint32_t tmem_slot;
};

static_assert(sizeof(GSmem) + 1024 <= 232448, "shared memory (plus alignment slack) exceeds 227 KB");

struct alignas(64) GParams {
    CUtensorMap ta, tb;  // A: K-major {K, M} box {32, 128} or MN-major {M, K} box {128, 32}; B likewise with N, 256
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

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(G_THREADS, 1) gemm_bf16x3(const __grid_constant__ GParams p) {
    pdl_enter();
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
        for (int i = 0; i < G_STAGES; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.read_a[i], NCONV);
            mbar_init(&sm.read_b[i], NCONV);
            mbar_init(&sm.ready[i], NCONV);
            mbar_init(&sm.empty[i], 1);
        }
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
    const uint32_t tm = sm.tmem_slot;
    bool failed = false;

    if (warp == G_TMA_WARP) {
        // ------------------------------------------------------------ TMA issuer
        if (lane == 0) {
            prefetch_tensormap(&p.ta);
            prefetch_tensormap(&p.tb);
            int g = 0;  // the CTA's stage sequence number
            for (int u = c; u < p.n_units && !failed; u += G) {
                const Unit x = make_unit(p, u);
                for (int j = 0; j < x.n_st; ++j, ++g) {
                    const int s = g % G_STAGES;
                    if (g >= G_STAGES && !mbar_wait(&sm.empty[s], ((g - G_STAGES) / G_STAGES) & 1, p.wait_ns)) {
                        failed = true;
                        break;
                    }
                    const int k0 = (x.st0 + j) * GK;
                    mbar_arrive_expect_tx(&sm.full[s], A_BYTES + B_BYTES);
                    if (A_MN) tma_load_2d(sm.a[s], &p.ta, x.m0, k0, &sm.full[s]);
                    else tma_load_2d(sm.a[s], &p.ta, k0, x.m0, &sm.full[s]);
                    if (B_MN) tma_load_2d(sm.b[s], &p.tb, x.n0, k0, &sm.full[s]);
                    else tma_load_2d(sm.b[s], &p.tb, k0, x.n0, &sm.full[s]);
                }
            }
            if (failed)
                for (int t = max(0, g - G_STAGES); t < g; ++t)
                    mbar_wait(&sm.full[t % G_STAGES], (t / G_STAGES) & 1, G_DRAIN_NS);
        }
        __syncwarp();
    } else if (warp == G_MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(GM, GN, A_MN ? 1 : 0, B_MN ? 1 : 0);
            // K-major: 64-byte rows (64B swizzle, 512-byte atoms), k-step 32
            // bytes; MN-major: 64-column atoms GK rows apart (lbo), k-step 16
            // rows (2048 bytes).
            constexpr uint32_t A_KSTEP = A_MN ? 2048 : 32, B_KSTEP = B_MN ? 2048 : 32;
            auto desc = [](uint32_t addr, bool mn) -> uint64_t {
                return mn ? smem_desc(addr, GK * 128, 1024) : smem_desc_sw64(addr, 512);
            };
            int g = 0, i = 0;
            for (int u = c; u < p.n_units && !failed; u += G, ++i) {
                const Unit x = make_unit(p, u);
                const int b = i & 1;
                if (i >= 2 && !mbar_wait(&sm.acc_free[b], ((i - 2) >> 1) & 1, p.wait_ns)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tm + b * GN;
                for (int j = 0; j < x.n_st; ++j, ++g) {
                    const int s = g % G_STAGES;
                    if (!mbar_wait(&sm.ready[s], (g / G_STAGES) & 1, p.wait_ns)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ah = desc(smem_u32(sm.a[s]), A_MN);
                    const uint64_t al = desc(smem_u32(sm.a[s] + A_BYTES / 2), A_MN);
                    const uint64_t bh = desc(smem_u32(sm.b[s]), B_MN);
                    const uint64_t bl = desc(smem_u32(sm.b[s] + B_BYTES / 2), B_MN);
#pragma unroll
                    for (int ks = 0; ks < GK / 16; ++ks) {
                        const uint32_t oa = ks * A_KSTEP, ob = ks * B_KSTEP;
                        mma_ss(acc, desc_add(ah, oa), desc_add(bh, ob), idesc, (j > 0 || ks > 0) ? 1u : 0u);
                        mma_ss(acc, desc_add(ah, oa), desc_add(bl, ob), idesc, 1);
                        mma_ss(acc, desc_add(al, oa), desc_add(bh, ob), idesc, 1);
                    }
                    mma_commit(&sm.empty[s]);
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
    } else if (warp >= NCONV / 32) {
        // ------------------------------------------------------------ epilogue
        // Warp e (lane quadrant e) owns tile rows 32e..32e+31.  Per 32-column
        // chunk: TMEM -> registers -> the warp's staging rows -> whole-row
        // float4 stores (8 lanes per 128-byte row segment).
        const int e = warp - NCONV / 32;
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
                tmem_ld32(lb + tm + b * GN + 32 * ch, v);
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
        // ------------------------------------------------------------ converters
        int g = 0;
        for (int u = c; u < p.n_units && !failed; u += G) {
            const Unit x = make_unit(p, u);
            for (int j = 0; j < x.n_st; ++j, ++g) {
                const int s = g % G_STAGES;
                const uint32_t ph = (g / G_STAGES) & 1;
                if (!mbar_wait_warp(&sm.full[s], ph, p.wait_ns)) {
                    failed = true;
                    break;
                }
                // A: [128][32] K-major or [32][128] MN-major; B: [256][32] or
                // [32][256].  Each tile is rewritten in place once every
                // thread has read its share of it; A first, then B, so that
                // only one tile's share is live in registers at a time.
                using ATile = typename std::conditional<A_MN, tc::RawTileMN<GK, GM, NCONV>, tc::RawTile32<GM, NCONV>>::type;
                using BTile = typename std::conditional<B_MN, tc::RawTileMN<GK, GN, NCONV>, tc::RawTile32<GN, NCONV>>::type;
                {
                    ATile ta;
                    ta.read(sm.a[s], tid);
                    mbar_arrive(&sm.read_a[s]);
                    if (!mbar_wait_warp(&sm.read_a[s], ph, p.wait_ns)) {
                        failed = true;
                        break;
                    }
                    ta.write(sm.a[s], tid);
                }
                {
                    BTile tb;
                    tb.read(sm.b[s], tid);
                    mbar_arrive(&sm.read_b[s]);
                    if (!mbar_wait_warp(&sm.read_b[s], ph, p.wait_ns)) {
                        failed = true;
                        break;
                    }
                    tb.write(sm.b[s], tid);
                }
                fence_async_smem();
                mbar_arrive(&sm.ready[s]);
            }
        }
    }

    if (__syncthreads_or(failed) && tid == 0) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, G_TMEM_COLS);
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
    if (M <= 0 || N <= 0 || K <= 0) {
        st.cuda = cudaErrorInvalidValue;
        st.what = "GEMM shape";
        return st;
    }
    GParams p;
    // A(m, k): K-major = a[m * lda + k] ({K, M}); MN-major = a[k * lda + m] ({M, K}).
    const bool ok_a = a_mn ? encode_2d(&p.ta, a, M, K, lda, GM, GK) : encode_2d(&p.ta, a, K, M, lda, GK, GM);
    const bool ok_b = b_mn ? encode_2d(&p.tb, b, N, K, ldb, GN, GK) : encode_2d(&p.tb, b, K, N, ldb, GK, GN);
    if (!ok_a || !ok_b) {
        st.cuda = cudaErrorInvalidValue;
        st.what = "GEMM tensor maps";
        return st;
    }
    const int sms = num_sms > 0 ? num_sms : 148;
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
    // Split K while the tiles alone leave SMs idle, keeping >= 8 stages
    // (256 of K) per split so that the four-stage ring fills.
    int splits = 1;
    if (tiles < sms) splits = static_cast<int>(std::min<long>((sms + tiles - 1) / tiles, std::max(1, p.k_stages / 8)));
    splits = std::min(splits, 8);
    p.stages_per_split = (p.k_stages + splits - 1) / splits;
    p.splits = (p.k_stages + p.stages_per_split - 1) / p.stages_per_split;
    const long n_units = tiles * p.splits;
    if (n_units > INT32_MAX) {
        st.cuda = cudaErrorInvalidValue;
        st.what = "GEMM too large";
        return st;
    }
    p.n_units = static_cast<int>(n_units);
    p.accumulate = accumulate;
    p.status = status;
    p.wait_ns = wait_ns;
    p.part = nullptr;
    cudaError_t e = cudaSuccess;
    if (p.splits > 1) {
        e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&p.part),
                                    sizeof(float) * static_cast<size_t>(p.splits) * M * N, pool, s);
        if (e != cudaSuccess) {
            st.cuda = e;
            st.what = "GEMM split workspace";
            return st;
        }
    }
    const int grid = static_cast<int>(std::min<long>(n_units, sms));
    if (a_mn && b_mn) e = launch_gemm_t<true, true>(p, grid, s);
    else if (a_mn) e = launch_gemm_t<true, false>(p, grid, s);
    else if (b_mn) e = launch_gemm_t<false, true>(p, grid, s);
    else e = launch_gemm_t<false, false>(p, grid, s);
    if (e == cudaSuccess) {
        *launches += 1;
        if (p.splits > 1) {
            const long n4 = static_cast<long>(M) * (N / 4);
            const int sgrid = static_cast<int>(std::min<long>((n4 + 255) / 256, 8L * sms));
            e = launch_pdl(gemm_split_sum, dim3(static_cast<unsigned>(sgrid)), dim3(256), 0, s, c, ldc,
                           static_cast<const float*>(p.part), bias, M, N, p.splits, accumulate);
            if (e == cudaSuccess) *launches += 1;
        }
    }
    if (p.part) {
        const cudaError_t ef = cudaFreeAsync(p.part, s);
        if (e == cudaSuccess) e = ef;
    }
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "GEMM launch";
    }
    return st;
}

}  // namespace kattn
