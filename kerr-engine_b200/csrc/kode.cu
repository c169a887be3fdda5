// Kerr-ODE forward and backward (sm_100a), the ODE core of kerr-engine's FFN
// (KerrMaestroAdd / KerrDualMaestro).  Replaces ComputeBackend::kerr_ode_batch
// (src/backend.rs:109-111; CPU kerr_ode_cpu :387-417; wgpu
// gpu_kerr_ode_batch_fused, src/gpu_ops_forward.rs:405) and
// kerr_ode_backward_batch (src/backend.rs:147-176; CPU kerr_ode_backward,
// src/backward.rs:382-458; wgpu src/gpu_ops_backward.rs:84), called at
// src/pipeline.rs:504, :626, :1003, :1022, :1067, :1107.
//
// Per position, n_embd = 2 nb floats hold nb bands interleaved (r_k, s_k).
// gamma = softplus(gamma_raw); n_steps RK4 steps of dt = 1/n_steps of
//   mag_k = r_k^2 + s_k^2,  ns_k = mag_{k-2} + mag_{k-1} + mag_{k+1} + mag_{k+2}
//   phi_k = omega_k + alpha mag_k + beta ns_k
//   dr_k = -gamma_k r_k - phi_k s_k,   ds_k = -gamma_k s_k + phi_k r_k
// (src/model.rs:778-843).  The backward recomputes the states and runs each
// RK4 step's adjoint from the last step to the first (src/backward.rs:
// 184-379); the parameter gradients are summed over all positions.
//
// Layout: one CTA is one position group; thread t owns NB consecutive bands
// [NB t, NB t + NB) in registers (2 NB consecutive floats of the row: one or
// two 16-byte loads, coalesced across the CTA).  The only coupling between
// bands is the +-2 stencil of ns (and its transpose in the backward): each
// derivative evaluation writes the thread's NB values to shared memory, one
// __syncthreads, and reads the two values on either side from the
// neighbouring threads' slots.  Two exchange buffers alternate, so one
// barrier per exchange suffices.  Bands past nb (padding up to a whole warp)
// hold zeros, which the ODE keeps at zero and which add nothing to their
// neighbours' stencils, so no band needs a bounds test.  CTAs are persistent:
// each walks positions blockIdx.x, + gridDim.x, ...
//
// The backward keeps the n_steps states of the current position in shared
// memory (each thread its own slots; 2 n_steps NB floats per thread) and the
// four evaluations of the step being differentiated in registers.  Each CTA
// sums its positions' d_gamma / d_omega per band in registers and d_alpha /
// d_beta per thread, writes one partial row per CTA, and a second kernel sums
// the partial rows in CTA order (no atomics: the same inputs give the same
// bits) and applies softplus' derivative.
//
// Bound: FP32 issue, not HBM.  Per band and position the forward executes
// about 25 floating-point instructions per derivative evaluation (4 per RK4
// step, n_steps steps) against 16 bytes of HBM traffic, and the backward
// about three times that.
#include <cuda_runtime.h>

#include "kattn_common.cuh"
#include "kattn_launch.h"

namespace kattn {

namespace {

template <int NB>
__device__ __forceinline__ void store_nb(float* p, const float (&v)[NB]) {
    if constexpr (NB == 2)
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    else
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

template <int NB>
__device__ __forceinline__ void load_nb(const float* p, float (&v)[NB]) {
    if constexpr (NB == 2) {
        const float2 a = *reinterpret_cast<const float2*>(p);
        v[0] = a.x;
        v[1] = a.y;
    } else {
        const float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x;
        v[1] = a.y;
        v[2] = a.z;
        v[3] = a.w;
    }
}

// One position's 2 NB interleaved floats (r_0, s_0, r_1, s_1, ...) of this
// thread's bands.
template <int NB>
__device__ __forceinline__ void load_bands(const float* row, float (&r)[NB], float (&s)[NB]) {
#pragma unroll
    for (int i = 0; i < NB; i += 2) {
        const float4 a = *reinterpret_cast<const float4*>(row + 2 * i);
        r[i] = a.x;
        s[i] = a.y;
        r[i + 1] = a.z;
        s[i + 1] = a.w;
    }
}

template <int NB>
__device__ __forceinline__ void store_bands(float* row, const float (&r)[NB], const float (&s)[NB]) {
#pragma unroll
    for (int i = 0; i < NB; i += 2)
        *reinterpret_cast<float4*>(row + 2 * i) = make_float4(r[i], s[i], r[i + 1], s[i + 1]);
}

// Stencil sums of the exchanged values v: out_i = v_{i-2} + v_{i-1} + v_{i+1}
// + v_{i+2} over the band axis, in that order (the reference's order).  This
// thread's own values are `own`; its neighbours' come from `ex`, where every
// thread of the CTA has just stored its NB values at ex[NB t].
template <int NB>
__device__ __forceinline__ void stencil(float* ex, const float (&own)[NB], float (&out)[NB], int t, int nthreads) {
    store_nb<NB>(ex + NB * t, own);
    __syncthreads();
    float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
    if (t > 0) lo = *reinterpret_cast<const float2*>(ex + NB * t - 2);
    if (t + 1 < nthreads) hi = *reinterpret_cast<const float2*>(ex + NB * t + NB);
    float e[NB + 4];
    e[0] = lo.x;
    e[1] = lo.y;
#pragma unroll
    for (int i = 0; i < NB; ++i) e[i + 2] = own[i];
    e[NB + 2] = hi.x;
    e[NB + 3] = hi.y;
#pragma unroll
    for (int i = 0; i < NB; ++i) out[i] = ((e[i] + e[i + 1]) + e[i + 3]) + e[i + 4];
}

template <int NB>
struct Bands {
    float gamma[NB];
    float omega[NB];
};

// Kerr derivative of (r, s) into (dr, ds); ns (the stencil sums of mag) is
// returned for the backward's cache.
template <int NB>
__device__ __forceinline__ void derivative(const float (&r)[NB], const float (&s)[NB], float (&dr)[NB],
                                           float (&ds)[NB], float (&ns)[NB], const Bands<NB>& p, float alpha,
                                           float beta, float* ex, int t, int nthreads) {
    float m[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) m[i] = r[i] * r[i] + s[i] * s[i];
    stencil<NB>(ex, m, ns, t, nthreads);
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        const float phi = p.omega[i] + alpha * m[i] + beta * ns[i];
        dr[i] = -p.gamma[i] * r[i] - phi * s[i];
        ds[i] = -p.gamma[i] * s[i] + phi * r[i];
    }
}

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : logf(1.f + expf(x)); }

template <int NB>
__device__ __forceinline__ void load_params(Bands<NB>& p, const float* gamma_raw, const float* omega, int nb, int t) {
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        const int k = NB * t + i;
        p.gamma[i] = k < nb ? softplus(gamma_raw[k]) : 0.f;
        p.omega[i] = k < nb ? omega[k] : 0.f;
    }
}

struct OdeArgs {
    const float* x;
    long ld_x;
    float* y;  // forward output
    long ld_y;
    const float* dy;  // backward input
    long ld_dy;
    float* dx;
    long ld_dx;
    const float* gamma_raw;
    const float* omega;
    const float* alpha_beta;
    float* part;  // backward: [gridDim.x][kode_part_width(nb)] partial parameter sums
    int M, nb, n_steps;
};

template <int NB>
__global__ void __launch_bounds__(KODE_MAX_THREADS) kode_fwd(const OdeArgs a) {
    extern __shared__ float kode_smem[];
    const int t = threadIdx.x, nthreads = blockDim.x;
    float* ex0 = kode_smem;
    float* ex1 = kode_smem + NB * nthreads;
    pdl_enter();
    Bands<NB> p;
    load_params<NB>(p, a.gamma_raw, a.omega, a.nb, t);
    const float alpha = a.alpha_beta[0], beta = a.alpha_beta[1];
    const float dt = 1.f / static_cast<float>(a.n_steps);
    const float hdt = 0.5f * dt, dt6 = dt / 6.f;
    const bool live = NB * t < a.nb;
    for (int m = blockIdx.x; m < a.M; m += gridDim.x) {
        float r[NB], s[NB];
        if (live) {
            load_bands<NB>(a.x + static_cast<long>(m) * a.ld_x + 2 * NB * t, r, s);
        } else {
#pragma unroll
            for (int i = 0; i < NB; ++i) r[i] = s[i] = 0.f;
        }
        for (int st = 0; st < a.n_steps; ++st) {
            float kr[NB], ks[NB], ar[NB], as[NB], ri[NB], si[NB], ns[NB];
            derivative<NB>(r, s, kr, ks, ns, p, alpha, beta, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                ar[i] = kr[i];
                as[i] = ks[i];
                ri[i] = r[i] + hdt * kr[i];
                si[i] = s[i] + hdt * ks[i];
            }
            derivative<NB>(ri, si, kr, ks, ns, p, alpha, beta, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                ar[i] += 2.f * kr[i];
                as[i] += 2.f * ks[i];
                ri[i] = r[i] + hdt * kr[i];
                si[i] = s[i] + hdt * ks[i];
            }
            derivative<NB>(ri, si, kr, ks, ns, p, alpha, beta, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                ar[i] += 2.f * kr[i];
                as[i] += 2.f * ks[i];
                ri[i] = r[i] + dt * kr[i];
                si[i] = s[i] + dt * ks[i];
            }
            derivative<NB>(ri, si, kr, ks, ns, p, alpha, beta, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                r[i] += dt6 * (ar[i] + kr[i]);
                s[i] += dt6 * (as[i] + ks[i]);
            }
        }
        if (live) store_bands<NB>(a.y + static_cast<long>(m) * a.ld_y + 2 * NB * t, r, s);
    }
}

// Adjoint of one derivative evaluation at (r, s) with stencil sums ns, for
// incoming (ddr, dds) = dL/d(dr, ds): writes (gr, gs) = dL/d(r, s) and adds the
// parameter terms into dg, dom (per band) and da, db.
template <int NB>
__device__ __forceinline__ void derivative_adjoint(const float (&r)[NB], const float (&s)[NB], const float (&ns)[NB],
                                                   const float (&ddr)[NB], const float (&dds)[NB], float (&gr)[NB],
                                                   float (&gs)[NB], const Bands<NB>& p, float alpha, float beta,
                                                   float (&dg)[NB], float (&dom)[NB], float& da, float& db, float* ex,
                                                   int t, int nthreads) {
    float dphi[NB], dns[NB], nsum[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        dphi[i] = ddr[i] * (-s[i]) + dds[i] * r[i];
        dns[i] = dphi[i] * beta;
    }
    stencil<NB>(ex, dns, nsum, t, nthreads);
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        const float m = r[i] * r[i] + s[i] * s[i];
        const float phi = p.omega[i] + alpha * m + beta * ns[i];
        dg[i] += ddr[i] * (-r[i]) + dds[i] * (-s[i]);
        dom[i] += dphi[i];
        da += dphi[i] * m;
        db += dphi[i] * ns[i];
        const float dm2 = 2.f * (dphi[i] * alpha + nsum[i]);
        gr[i] = ddr[i] * (-p.gamma[i]) + dds[i] * phi + dm2 * r[i];
        gs[i] = ddr[i] * (-phi) + dds[i] * (-p.gamma[i]) + dm2 * s[i];
    }
}

template <int NB>
__global__ void __launch_bounds__(KODE_MAX_THREADS) kode_bwd(const OdeArgs a) {
    extern __shared__ float kode_smem[];
    const int t = threadIdx.x, nthreads = blockDim.x;
    float* ex0 = kode_smem;
    float* ex1 = kode_smem + NB * nthreads;
    float* states = kode_smem + 2 * NB * nthreads;  // [n_steps][2][nthreads][NB]
    pdl_enter();
    Bands<NB> p;
    load_params<NB>(p, a.gamma_raw, a.omega, a.nb, t);
    const float alpha = a.alpha_beta[0], beta = a.alpha_beta[1];
    const float dt = 1.f / static_cast<float>(a.n_steps);
    const float hdt = 0.5f * dt, dt6 = dt / 6.f, dt3 = 2.f * dt6;
    const bool live = NB * t < a.nb;
    float dg[NB], dom[NB], da = 0.f, db = 0.f;
#pragma unroll
    for (int i = 0; i < NB; ++i) dg[i] = dom[i] = 0.f;

    for (int m = blockIdx.x; m < a.M; m += gridDim.x) {
        float r[NB], s[NB], gr[NB], gs[NB];
        if (live) {
            load_bands<NB>(a.x + static_cast<long>(m) * a.ld_x + 2 * NB * t, r, s);
            load_bands<NB>(a.dy + static_cast<long>(m) * a.ld_dy + 2 * NB * t, gr, gs);
        } else {
#pragma unroll
            for (int i = 0; i < NB; ++i) r[i] = s[i] = gr[i] = gs[i] = 0.f;
        }
        // Forward: keep the state entering every step.
        for (int st = 0; st < a.n_steps; ++st) {
            float* slot = states + (static_cast<long>(st) * 2 * nthreads + t) * NB;
            store_nb<NB>(slot, r);
            store_nb<NB>(slot + NB * nthreads, s);
            float kr[NB], ks[NB], ar[NB], as[NB], ri[NB], si[NB], ns[NB];
            derivative<NB>(r, s, kr, ks, ns, p, alpha, beta, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                ar[i] = kr[i];
                as[i] = ks[i];
                ri[i] = r[i] + hdt * kr[i];
                si[i] = s[i] + hdt * ks[i];
            }
            derivative<NB>(ri, si, kr, ks, ns, p, alpha, beta, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                ar[i] += 2.f * kr[i];
                as[i] += 2.f * ks[i];
                ri[i] = r[i] + hdt * kr[i];
                si[i] = s[i] + hdt * ks[i];
            }
            derivative<NB>(ri, si, kr, ks, ns, p, alpha, beta, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                ar[i] += 2.f * kr[i];
                as[i] += 2.f * ks[i];
                ri[i] = r[i] + dt * kr[i];
                si[i] = s[i] + dt * ks[i];
            }
            derivative<NB>(ri, si, kr, ks, ns, p, alpha, beta, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                r[i] += dt6 * (ar[i] + kr[i]);
                s[i] += dt6 * (as[i] + ks[i]);
            }
        }
        // Adjoint, last step first.  (gr, gs) = dL/d(state after the step).
        for (int st = a.n_steps - 1; st >= 0; --st) {
            const float* slot = states + (static_cast<long>(st) * 2 * nthreads + t) * NB;
            float r1[NB], s1[NB], r2[NB], s2[NB], r3[NB], s3[NB], r4[NB], s4[NB];
            float ns1[NB], ns2[NB], ns3[NB], ns4[NB], kr[NB], ks[NB];
            load_nb<NB>(slot, r1);
            load_nb<NB>(slot + NB * nthreads, s1);
            derivative<NB>(r1, s1, kr, ks, ns1, p, alpha, beta, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                r2[i] = r1[i] + hdt * kr[i];
                s2[i] = s1[i] + hdt * ks[i];
            }
            derivative<NB>(r2, s2, kr, ks, ns2, p, alpha, beta, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                r3[i] = r1[i] + hdt * kr[i];
                s3[i] = s1[i] + hdt * ks[i];
            }
            derivative<NB>(r3, s3, kr, ks, ns3, p, alpha, beta, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                r4[i] = r1[i] + dt * kr[i];
                s4[i] = s1[i] + dt * ks[i];
            }
            // The fourth evaluation's stencil sums (its derivative is not needed).
            {
                float m[NB];
#pragma unroll
                for (int i = 0; i < NB; ++i) m[i] = r4[i] * r4[i] + s4[i] * s4[i];
                stencil<NB>(ex1, m, ns4, t, nthreads);
            }
            // r_new = r + dt/6 (k1 + 2 k2 + 2 k3 + k4), k_{i+1} evaluated at
            // r + c_i dt k_i (c = 1/2, 1/2, 1).
            float on_r[NB], on_s[NB], ddr[NB], dds[NB], er[NB], es[NB];
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                on_r[i] = gr[i];
                on_s[i] = gs[i];
                ddr[i] = on_r[i] * dt6;
                dds[i] = on_s[i] * dt6;
            }
            derivative_adjoint<NB>(r4, s4, ns4, ddr, dds, er, es, p, alpha, beta, dg, dom, da, db, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                gr[i] += er[i];
                gs[i] += es[i];
                ddr[i] = er[i] * dt + on_r[i] * dt3;
                dds[i] = es[i] * dt + on_s[i] * dt3;
            }
            derivative_adjoint<NB>(r3, s3, ns3, ddr, dds, er, es, p, alpha, beta, dg, dom, da, db, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                gr[i] += er[i];
                gs[i] += es[i];
                ddr[i] = er[i] * hdt + on_r[i] * dt3;
                dds[i] = es[i] * hdt + on_s[i] * dt3;
            }
            derivative_adjoint<NB>(r2, s2, ns2, ddr, dds, er, es, p, alpha, beta, dg, dom, da, db, ex0, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                gr[i] += er[i];
                gs[i] += es[i];
                ddr[i] = er[i] * hdt + on_r[i] * dt6;
                dds[i] = es[i] * hdt + on_s[i] * dt6;
            }
            derivative_adjoint<NB>(r1, s1, ns1, ddr, dds, er, es, p, alpha, beta, dg, dom, da, db, ex1, t, nthreads);
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                gr[i] += er[i];
                gs[i] += es[i];
            }
        }
        if (live) store_bands<NB>(a.dx + static_cast<long>(m) * a.ld_dx + 2 * NB * t, gr, gs);
    }

    // This CTA's partial row: d_gamma, d_omega per band, then d_alpha, d_beta
    // summed over the CTA's threads in a fixed order.
    float* row = a.part + static_cast<long>(blockIdx.x) * kode_part_width(a.nb);
    if (live) {
        store_nb<NB>(row + NB * t, dg);
        store_nb<NB>(row + a.nb + NB * t, dom);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        da += __shfl_xor_sync(0xffffffffu, da, o);
        db += __shfl_xor_sync(0xffffffffu, db, o);
    }
    __syncthreads();  // the exchange buffers are free: reuse ex0 for the warp sums
    const int lane = t & 31, wid = t >> 5, nwarps = nthreads >> 5;
    if (lane == 0) {
        ex0[2 * wid] = da;
        ex0[2 * wid + 1] = db;
    }
    __syncthreads();
    if (t == 0) {
        float sa = 0.f, sb = 0.f;
        for (int w = 0; w < nwarps; ++w) {
            sa += ex0[2 * w];
            sb += ex0[2 * w + 1];
        }
        row[2 * a.nb] = sa;
        row[2 * a.nb + 1] = sb;
    }
}

// out[i] (+)= sum over CTAs c of part[c][i] for the 2 nb + 2 parameter
// gradients (rows kode_part_width(nb) floats apart); d_gamma is chained
// through softplus' derivative sigmoid(gamma_raw) (src/backward.rs:150-153).
// A CTA of 32 x 32 threads takes 32 outputs: thread (x, y) sums rows y, y + 32,
// ... of output x (coalesced across x), then thread (x, 0) adds the 32 sums
// in order of y.  The order is fixed: the same partials give the same bits.
constexpr int KODE_FINAL_COLS = 32;
constexpr int KODE_FINAL_GROUPS = 32;

__global__ void __launch_bounds__(KODE_FINAL_COLS* KODE_FINAL_GROUPS)
    kode_param_final(const float* __restrict__ part, int P, int nb, const float* __restrict__ gamma_raw,
                     float* __restrict__ dgr, float* __restrict__ dom, float* __restrict__ dab, int accumulate) {
    __shared__ float sums[KODE_FINAL_GROUPS][KODE_FINAL_COLS + 1];
    pdl_enter();
    const int x = threadIdx.x, y = threadIdx.y;
    const int i = blockIdx.x * KODE_FINAL_COLS + x;
    const int width = kode_part_width(nb);
    const bool valid = i < 2 * nb + 2;
    float acc = 0.f;
    if (valid) {
        const float* col = part + i;
        int c = y;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        for (; c + 3 * KODE_FINAL_GROUPS < P; c += 4 * KODE_FINAL_GROUPS) {
            a0 += col[static_cast<long>(c) * width];
            a1 += col[static_cast<long>(c + KODE_FINAL_GROUPS) * width];
            a2 += col[static_cast<long>(c + 2 * KODE_FINAL_GROUPS) * width];
            a3 += col[static_cast<long>(c + 3 * KODE_FINAL_GROUPS) * width];
        }
        for (; c < P; c += KODE_FINAL_GROUPS) a0 += col[static_cast<long>(c) * width];
        acc = (a0 + a1) + (a2 + a3);
    }
    sums[y][x] = acc;
    __syncthreads();
    if (y != 0 || !valid) return;
    float sum = 0.f;
    for (int g = 0; g < KODE_FINAL_GROUPS; ++g) sum += sums[g][x];
    float* dst;
    if (i < nb) {
        const float g = gamma_raw[i];
        sum *= g > 20.f ? 1.f : expf(g) / (1.f + expf(g));
        dst = dgr + i;
    } else if (i < 2 * nb) {
        dst = dom + (i - nb);
    } else {
        dst = dab + (i - 2 * nb);
    }
    *dst = accumulate ? *dst + sum : sum;
}

int kode_nb(int nb) { return nb <= 64 ? 2 : 4; }

int kode_threads(int nb) {
    const int per = kode_nb(nb);
    const int t = (nb + per - 1) / per;
    return (t + 31) / 32 * 32;
}

template <int NB>
cudaError_t launch_ode(bool backward, const OdeArgs& a, int threads, size_t smem, int grid, cudaStream_t s) {
    auto k = backward ? kode_bwd<NB> : kode_fwd<NB>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_pdl(k, dim3(static_cast<unsigned>(grid)), dim3(static_cast<unsigned>(threads)), smem, s, a);
}

template <int NB>
cudaError_t ode_grid(bool backward, int threads, size_t smem, int num_sms, int M, int* grid) {
    auto k = backward ? kode_bwd<NB> : kode_fwd<NB>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const long cap = static_cast<long>(per_sm) * (num_sms > 0 ? num_sms : 148);
    *grid = static_cast<int>(M < cap ? M : cap);
    return cudaSuccess;
}

size_t fwd_smem(int threads, int NB) { return sizeof(float) * 2 * NB * static_cast<size_t>(threads); }
size_t bwd_smem(int threads, int NB, int n_steps) {
    return sizeof(float) * NB * static_cast<size_t>(threads) * (2 + 2 * static_cast<size_t>(n_steps));
}

}  // namespace

bool kode_supported(int nb, int n_steps) {
    if (nb <= 0 || nb % 4 != 0 || nb > KODE_MAX_BANDS || n_steps < 1) return false;
    const int threads = kode_threads(nb);
    return bwd_smem(threads, kode_nb(nb), n_steps) <= KODE_MAX_SMEM;
}

ProjStatus kode_forward(cudaStream_t s, int num_sms, const float* x, long ld_x, float* y, long ld_y,
                        const float* gamma_raw, const float* omega, const float* alpha_beta, int M, int nb,
                        int n_steps, int* launches) {
    ProjStatus st;
    if (M == 0) return st;
    OdeArgs a = {};
    a.x = x;
    a.ld_x = ld_x;
    a.y = y;
    a.ld_y = ld_y;
    a.gamma_raw = gamma_raw;
    a.omega = omega;
    a.alpha_beta = alpha_beta;
    a.M = M;
    a.nb = nb;
    a.n_steps = n_steps;
    const int NB = kode_nb(nb), threads = kode_threads(nb);
    const size_t smem = fwd_smem(threads, NB);
    int grid = 0;
    cudaError_t e = NB == 2 ? ode_grid<2>(false, threads, smem, num_sms, M, &grid)
                            : ode_grid<4>(false, threads, smem, num_sms, M, &grid);
    if (e == cudaSuccess)
        e = NB == 2 ? launch_ode<2>(false, a, threads, smem, grid, s) : launch_ode<4>(false, a, threads, smem, grid, s);
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "Kerr-ODE forward launch";
        return st;
    }
    *launches += 1;
    return st;
}

ProjStatus kode_backward_rows(cudaStream_t s, const float* dy, long ld_dy, const float* x, long ld_x,
                              const float* gamma_raw, const float* omega, const float* alpha_beta, float* dx,
                              long ld_dx, int M, int nb, int n_steps, float* part, int part_rows, int* launches) {
    ProjStatus st;
    if (M == 0) return st;
    OdeArgs a = {};
    a.x = x;
    a.ld_x = ld_x;
    a.dy = dy;
    a.ld_dy = ld_dy;
    a.dx = dx;
    a.ld_dx = ld_dx;
    a.gamma_raw = gamma_raw;
    a.omega = omega;
    a.alpha_beta = alpha_beta;
    a.part = part;
    a.M = M;
    a.nb = nb;
    a.n_steps = n_steps;
    const int NB = kode_nb(nb), threads = kode_threads(nb);
    const size_t smem = bwd_smem(threads, NB, n_steps);
    const cudaError_t e = NB == 2 ? launch_ode<2>(true, a, threads, smem, part_rows, s)
                                  : launch_ode<4>(true, a, threads, smem, part_rows, s);
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "Kerr-ODE backward launch";
        return st;
    }
    *launches += 1;
    return st;
}

ProjStatus kode_backward_final(cudaStream_t s, const float* part, int part_rows, int nb, const float* gamma_raw,
                               float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int accumulate,
                               int* launches) {
    ProjStatus st;
    const int outputs = 2 * nb + 2;
    const cudaError_t e =
        launch_pdl(kode_param_final, dim3(static_cast<unsigned>((outputs + KODE_FINAL_COLS - 1) / KODE_FINAL_COLS)),
                   dim3(KODE_FINAL_COLS, KODE_FINAL_GROUPS), 0, s, part, part_rows, nb, gamma_raw, d_gamma_raw,
                   d_omega, d_alpha_beta, accumulate);
    if (e != cudaSuccess) {
        st.cuda = e;
        st.what = "Kerr-ODE parameter-gradient launch";
        return st;
    }
    *launches += 1;
    return st;
}

ProjStatus kode_backward(cudaStream_t s, int num_sms, const float* dy, long ld_dy, const float* x, long ld_x,
                         const float* gamma_raw, const float* omega, const float* alpha_beta, float* dx, long ld_dx,
                         float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int M, int nb, int n_steps,
                         int accumulate, float* part, int part_rows, int* launches) {
    (void)num_sms;
    ProjStatus st = kode_backward_rows(s, dy, ld_dy, x, ld_x, gamma_raw, omega, alpha_beta, dx, ld_dx, M, nb,
                                       n_steps, part, part_rows, launches);
    if (!st.ok()) return st;
    return kode_backward_final(s, part, M > 0 ? part_rows : 0, nb, gamma_raw, d_gamma_raw, d_omega, d_alpha_beta,
                               accumulate, launches);
}

cudaError_t kode_backward_grid(int num_sms, int M, int nb, int n_steps, int* grid) {
    if (M == 0) {
        *grid = 0;
        return cudaSuccess;
    }
    const int NB = kode_nb(nb), threads = kode_threads(nb);
    const size_t smem = bwd_smem(threads, NB, n_steps);
    return NB == 2 ? ode_grid<2>(true, threads, smem, num_sms, M, grid)
                   : ode_grid<4>(true, threads, smem, num_sms, M, grid);
}

}  // namespace kattn
