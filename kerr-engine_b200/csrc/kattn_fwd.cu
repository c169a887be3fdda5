// Causal self-attention forward, f32 on the FFMA pipe (sm_100a).
//
// Replaces the scalar head loop of src/pipeline.rs:305-347: one CTA owns a
// 64-row query tile of one (batch, head) slab, streams the slab's 64-row key /
// value tiles through shared memory (cp.async double buffer), keeps the running
// row max / row sum of an online softmax in registers and writes the normalised
// output plus the row log-sum-exp.  Only tiles on or below the diagonal are
// visited when causal.
//
// Thread layout (256 threads): tx = tid % 16, ty = tid / 16.  A thread owns
// score rows ty + 16a and key columns tx + 16b (a, b < 4) of the 64x64 tile,
// and output rows ty + 16a, columns tx*DC .. tx*DC + DC-1 (DC = d / 16).
#include "kattn_common.cuh"
#include "kattn_launch.h"

namespace kattn {

constexpr int FWD_BM = 64;
constexpr int FWD_BN = 64;
constexpr int FWD_NT = 256;

template <int D>
struct FwdSmem {
    static constexpr int LDD = D + 4;       // pitch of q/k/v tiles: conflict-free float4 columns
    static constexpr int LDP = FWD_BN + 16;  // pitch of the probability tile
    float q[FWD_BM * LDD];
    float k[2][FWD_BN * LDD];
    float v[2][FWD_BN * LDD];
    float p[FWD_BM * LDP];
};

struct FwdParams {
    const float* q;
    const float* k;
    const float* v;
    long ld_qkv;
    float* o;
    long ld_o;
    float* lse;
    int B, T, H;
    float scale_log2;  // scale * log2(e): scores are kept in log2 units
    int causal;
    int n_tiles;
};

template <int D>
__global__ void __launch_bounds__(FWD_NT, (D <= 64 ? 2 : 1)) attn_fwd_f32(const FwdParams p) {
    pdl_enter();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    FwdSmem<D>& sm = *reinterpret_cast<FwdSmem<D>*>(smem_raw);
    constexpr int LDD = FwdSmem<D>::LDD;
    constexpr int LDP = FwdSmem<D>::LDP;
    constexpr int DC = D / 16;  // output columns per thread
    constexpr int C4 = D / 4;   // float4 per tile row

    const int nslab = p.B * p.H;
    // Diagonal-heavy query tiles (most key tiles under the causal mask) first.
    const int qt = p.n_tiles - 1 - static_cast<int>(blockIdx.x / nslab);
    const int slab = static_cast<int>(blockIdx.x % nslab);
    const int b = slab / p.H;
    const int h = slab % p.H;
    const int tid = threadIdx.x;
    const int tx = tid & 15;
    const int ty = tid >> 4;
    const int q0 = qt * FWD_BM;

    const long row0 = static_cast<long>(b) * p.T;
    const float* qg = p.q + row0 * p.ld_qkv + h * D;
    const float* kg = p.k + row0 * p.ld_qkv + h * D;
    const float* vg = p.v + row0 * p.ld_qkv + h * D;

    auto load_kv = [&](int j, int buf) {
        const int k0 = j * FWD_BN;
#pragma unroll
        for (int i = tid; i < FWD_BN * C4; i += FWD_NT) {
            const int r = i / C4;
            const int c = (i % C4) * 4;
            const bool ok = k0 + r < p.T;
            const long off = static_cast<long>(ok ? k0 + r : 0) * p.ld_qkv + c;
            cp_async16(&sm.k[buf][r * LDD + c], kg + off, ok ? 16 : 0);
            cp_async16(&sm.v[buf][r * LDD + c], vg + off, ok ? 16 : 0);
        }
        cp_async_commit();
    };

    const int n_kv = p.causal ? qt + 1 : p.n_tiles;
    load_kv(0, 0);

    // Query tile, pre-scaled so that q.k lands in log2 units.
#pragma unroll
    for (int i = tid; i < FWD_BM * C4; i += FWD_NT) {
        const int r = i / C4;
        const int c = (i % C4) * 4;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < p.T) x = *reinterpret_cast<const float4*>(qg + static_cast<long>(q0 + r) * p.ld_qkv + c);
        x.x *= p.scale_log2;
        x.y *= p.scale_log2;
        x.z *= p.scale_log2;
        x.w *= p.scale_log2;
        *reinterpret_cast<float4*>(&sm.q[r * LDD + c]) = x;
    }

    float acc[4][DC];
    float m[4], l[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -INFINITY;
        l[a] = 0.f;
#pragma unroll
        for (int c = 0; c < DC; ++c) acc[a][c] = 0.f;
    }

    for (int j = 0; j < n_kv; ++j) {
        const int buf = j & 1;
        if (j + 1 < n_kv) {
            load_kv(j + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();

        // S = Q K^T on this thread's 4x4 fragment.
        float s[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) s[a][c] = 0.f;
        const float* ks = sm.k[buf];
#pragma unroll 4
        for (int kk = 0; kk < D; kk += 4) {
            float4 qa[4], kb[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(&sm.q[(ty + 16 * a) * LDD + kk]);
#pragma unroll
            for (int c = 0; c < 4; ++c) kb[c] = *reinterpret_cast<const float4*>(&ks[(tx + 16 * c) * LDD + kk]);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    s[a][c] = fmaf(qa[a].x, kb[c].x, s[a][c]);
                    s[a][c] = fmaf(qa[a].y, kb[c].y, s[a][c]);
                    s[a][c] = fmaf(qa[a].z, kb[c].z, s[a][c]);
                    s[a][c] = fmaf(qa[a].w, kb[c].w, s[a][c]);
                }
        }

        const int k0 = j * FWD_BN;
        if ((p.causal && j == qt) || k0 + FWD_BN > p.T) {
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int r = q0 + ty + 16 * a;
                    const int col = k0 + tx + 16 * c;
                    if ((p.causal && col > r) || col >= p.T) s[a][c] = -INFINITY;
                }
        }

        // Online softmax update (log2 domain).
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float mt = fmaxf(fmaxf(s[a][0], s[a][1]), fmaxf(s[a][2], s[a][3]));
            mt = max16(mt);
            const float mn = fmaxf(m[a], mt);
            const float ms = (mn == -INFINITY) ? 0.f : mn;  // fully masked so far
            const float alpha = ex2(m[a] - ms);
            m[a] = mn;
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float e = ex2(s[a][c] - ms);
                s[a][c] = e;
                rs += e;
            }
            l[a] = l[a] * alpha + rs;
#pragma unroll
            for (int c = 0; c < DC; ++c) acc[a][c] *= alpha;
        }

#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) sm.p[(ty + 16 * a) * LDP + tx + 16 * c] = s[a][c];
        __syncthreads();

        // O += P V.
        const float* vs = sm.v[buf];
#pragma unroll 2
        for (int kk = 0; kk < FWD_BN; kk += 4) {
            float4 pa[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) pa[a] = *reinterpret_cast<const float4*>(&sm.p[(ty + 16 * a) * LDP + kk]);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                Frag<DC> vr;
                vr.load(&vs[(kk + u) * LDD + tx * DC]);
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float pv = u == 0 ? pa[a].x : u == 1 ? pa[a].y : u == 2 ? pa[a].z : pa[a].w;
#pragma unroll
                    for (int c = 0; c < DC; ++c) acc[a][c] = fmaf(pv, vr.x[c], acc[a][c]);
                }
            }
        }
        __syncthreads();  // P and K/V buffer `buf` are rewritten next iteration
    }

    float* og = p.o + row0 * p.ld_o + h * D;
    float* lseg = p.lse + (static_cast<long>(b) * p.H + h) * p.T;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int r = q0 + ty + 16 * a;
        const float lt = sum16(l[a]);
        if (r < p.T) {
            const float inv = 1.f / lt;
            Frag<DC> f;
#pragma unroll
            for (int c = 0; c < DC; ++c) f.x[c] = acc[a][c] * inv;
            f.store(og + static_cast<long>(r) * p.ld_o + tx * DC);
            if (tx == 0) lseg[r] = (m[a] + log2f(lt)) * kLn2;
        }
    }
}

template <int D>
static cudaError_t launch_fwd_d(const FwdArgs& a, cudaStream_t stream) {
    FwdParams p;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.ld_qkv = a.ld_qkv;
    p.o = a.o;
    p.ld_o = a.ld_o;
    p.lse = a.lse;
    p.B = a.B;
    p.T = a.T;
    p.H = a.H;
    p.scale_log2 = a.scale * kLog2e;
    p.causal = a.causal;
    p.n_tiles = (a.T + FWD_BM - 1) / FWD_BM;
    const size_t smem = sizeof(FwdSmem<D>);
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_f32<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const long nblocks = static_cast<long>(p.n_tiles) * a.B * a.H;
    return launch_pdl(attn_fwd_f32<D>, dim3(static_cast<unsigned>(nblocks)), dim3(FWD_NT), smem, stream, p);
}

cudaError_t launch_fwd(const FwdArgs& a, int /*num_sms*/, cudaStream_t stream, int* launches) {
    cudaError_t e = cudaErrorInvalidValue;
    switch (a.d) {
        case 32: e = launch_fwd_d<32>(a, stream); break;
        case 64: e = launch_fwd_d<64>(a, stream); break;
        case 128: e = launch_fwd_d<128>(a, stream); break;
        default: return cudaErrorInvalidValue;
    }
    if (e == cudaSuccess) *launches += 1;
    return e;
}

}  // namespace kattn
