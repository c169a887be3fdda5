// Device-resident block pipeline (include/kerr_attn.h, kattn_block_*): one
// transformer block of the reference's batched forward / backward
// (forward_backward_batch, src/pipeline.rs:764-1222; per block :236-360 and
// :670-750) as far as this library covers it, with every intermediate kept on
// the device between the forward and the backward:
//
//   x1 = LN1(h); qkv = c_attn(x1); o = attention(qkv); h1 = h + c_proj(o)
//   h_out = h1 + KerrODE(LN2(h1))      (the FFN's ODE core; optional)
//
// The calls below are this library's own entry points (LayerNorm, the
// tcgen05 GEMM, attention, Kerr-ODE) on one stream; c_proj's GEMM adds its
// product onto a copy of h in its epilogue, so the residual costs no pass of
// its own.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "kattn_common.cuh"
#include "kattn_internal.h"
#include "kattn_launch.h"
#include "kerr_attn.h"

using namespace kattn_abi;

struct kattn_block {
    kattn_ctx* ctx = nullptr;
    int B = 0, T = 0, C = 0, H = 0, d = 0, rk4 = 0;
    long M = 0;
    float* buf = nullptr;  // one allocation for everything below
    // forward state
    float* x1 = nullptr;   // LN1(h)           [M][C]
    float* qkv = nullptr;  // c_attn(x1)       [M][3C]
    float* o = nullptr;    // attention output [M][C]
    float* lse = nullptr;  // [B][H][T]
    float* h1 = nullptr;   // h + c_proj(o)    [M][C] (FFN only; else h_out)
    float* x2 = nullptr;   // LN2(h1)          [M][C] (FFN only)
    // backward temporaries
    float* t = nullptr;     // dx2, then dx1   [M][C]
    float* dh1 = nullptr;   // d(loss)/dh1     [M][C] (FFN only)
    float* d_o = nullptr;   // d(loss)/do, then LN1's dx [M][C]
    float* dqkv = nullptr;  // [M][3C]
    const float* h = nullptr;  // the forward's input (read again by LN1's backward)
    kattn_block_params p{};
    bool valid = false;  // a forward was enqueued
};

namespace {

// out = a + b over n floats (n a multiple of 4; 16-byte aligned; out may
// alias a or b).
__global__ void __launch_bounds__(256) block_add(float* out, const float* a, const float* b, long n4) {
    kattn::pdl_enter();
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const float4 x = reinterpret_cast<const float4*>(a)[i];
        const float4 y = reinterpret_cast<const float4*>(b)[i];
        reinterpret_cast<float4*>(out)[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
    }
}

cudaError_t add(const kattn_block* blk, float* out, const float* a, const float* b, cudaStream_t s, int* launches) {
    const long n4 = blk->M * blk->C / 4;
    const long grid = std::min<long>((n4 + 255) / 256, 8L * (blk->ctx->num_sms > 0 ? blk->ctx->num_sms : 148));
    const cudaError_t e = kattn::launch_pdl(block_add, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, out, a, b, n4);
    if (e == cudaSuccess) ++*launches;
    return e;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

// Runs one public entry point and adds the kernels it enqueued.
#define BLK_CALL(expr)                                 \
    do {                                               \
        const int _s = (expr);                         \
        if (_s != KATTN_OK) return _s;                 \
        launches += kattn_last_launch_count();         \
    } while (0)

int check_block(const kattn_ctx* ctx, const kattn_block* blk) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (!blk) return fail(KATTN_ERR_INVALID_ARGUMENT, "block is NULL");
    if (blk->ctx != ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "block belongs to another context");
    return KATTN_OK;
}

}  // namespace

extern "C" {
#pragma GCC visibility push(default)

int kattn_block_create(kattn_ctx* ctx, int B, int T, int C, int H, int rk4_n_steps, kattn_block** out) {
    if (!out) return fail(KATTN_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (B <= 0 || T <= 0 || C <= 0 || H <= 0)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "sizes must be positive (B=%d T=%d C=%d H=%d)", B, T, C, H);
    if (C % 8 != 0 || C % H != 0) return fail(KATTN_ERR_UNSUPPORTED, "C=%d must be a multiple of 8 and of H=%d", C, H);
    const int d = C / H;
    if (d != 32 && d != 64 && d != 128) return fail(KATTN_ERR_UNSUPPORTED, "head_dim %d unsupported (32, 64 or 128)", d);
    if (C > KATTN_LN_MAX_N) return fail(KATTN_ERR_UNSUPPORTED, "C=%d exceeds KATTN_LN_MAX_N", C);
    if (rk4_n_steps < 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "rk4_n_steps must be >= 0");
    if (rk4_n_steps > 0 && ((C / 2) % 4 != 0 || C / 2 > KATTN_KODE_MAX_BANDS))
        return fail(KATTN_ERR_UNSUPPORTED, "the FFN needs C/2 bands, a multiple of 4, at most %d", KATTN_KODE_MAX_BANDS);
    const long M = static_cast<long>(B) * T;
    if (M * 3 * C > (1L << 40)) return fail(KATTN_ERR_INVALID_ARGUMENT, "problem too large");
    kattn_block* blk = new kattn_block;
    blk->ctx = ctx;
    blk->B = B;
    blk->T = T;
    blk->C = C;
    blk->H = H;
    blk->d = d;
    blk->rk4 = rk4_n_steps;
    blk->M = M;
    const bool ffn = rk4_n_steps > 0;
    const size_t mc = static_cast<size_t>(M) * C;
    const size_t lse = (static_cast<size_t>(B) * H * T + 63) / 64 * 64;  // keeps the arrays after it 256-byte aligned
    const size_t floats = mc * (ffn ? 13 : 10) + lse;
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) {
        delete blk;
        return cuda_fail(scope.err, "cudaSetDevice");
    }
    const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&blk->buf), floats * sizeof(float));
    if (e != cudaSuccess) {
        delete blk;
        return cuda_fail(e, "block activations");
    }
    float* q = blk->buf;
    auto take = [&](size_t n) {
        float* r = q;
        q += n;
        return r;
    };
    blk->x1 = take(mc);
    blk->qkv = take(3 * mc);
    blk->o = take(mc);
    blk->lse = take(lse);
    blk->t = take(mc);
    blk->d_o = take(mc);
    blk->dqkv = take(3 * mc);
    if (ffn) {
        blk->h1 = take(mc);
        blk->x2 = take(mc);
        blk->dh1 = take(mc);
    }
    *out = blk;
    return KATTN_OK;
}

int kattn_block_destroy(kattn_block* blk) {
    if (!blk) return KATTN_OK;
    DeviceScope scope(blk->ctx->device);
    const cudaError_t e = blk->buf ? cudaFree(blk->buf) : cudaSuccess;
    delete blk;
    return e == cudaSuccess ? KATTN_OK : cuda_fail(e, "cudaFree(block activations)");
}

int kattn_block_fwd(kattn_ctx* ctx, kattn_block* blk, const kattn_block_params* params, const float* h,
                    float* h_out, void* stream) {
    {
        const int st = check_block(ctx, blk);
        if (st != KATTN_OK) return st;
    }
    if (!params) return fail(KATTN_ERR_INVALID_ARGUMENT, "params is NULL");
    const kattn_block_params& p = *params;
    const bool ffn = blk->rk4 > 0;
    if (!h || !h_out) return fail(KATTN_ERR_INVALID_ARGUMENT, "h / h_out is NULL");
    if (h == h_out) return fail(KATTN_ERR_INVALID_ARGUMENT, "h_out must not alias h");
    if (!aligned16(h) || !aligned16(h_out)) return fail(KATTN_ERR_MISALIGNED, "h / h_out not 16-byte aligned");
    if (!p.ln1_w || !p.ln1_b || !p.w_attn || !p.b_attn || !p.w_proj || !p.b_proj)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "a parameter of the attention sublayer is NULL");
    if (ffn && (!p.ln2_w || !p.ln2_b || !p.gamma_raw || !p.omega || !p.alpha_beta))
        return fail(KATTN_ERR_INVALID_ARGUMENT, "a parameter of the FFN is NULL");
    if (!aligned16(p.w_proj) || !aligned4(p.b_proj))
        return fail(KATTN_ERR_MISALIGNED, "w_proj not 16-byte or b_proj not 4-byte aligned");
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int M = static_cast<int>(blk->M), C = blk->C, H = blk->H, d = blk->d;
    const float scale = 1.0f / std::sqrt(static_cast<float>(d));
    int launches = 0;
    blk->valid = false;
    BLK_CALL(kattn_layernorm_fwd(ctx, h, C, p.ln1_w, p.ln1_b, blk->x1, C, M, C, stream));
    BLK_CALL(kattn_linear_fwd(ctx, blk->x1, C, p.w_attn, p.b_attn, blk->qkv, 3L * C, M, 3 * C, C, stream));
    BLK_CALL(kattn_fwd(ctx, blk->qkv, blk->qkv + C, blk->qkv + 2 * C, 3L * C, blk->o, C, blk->lse, blk->B, blk->T, H, d,
                       scale, 1, stream));
    // h1 = h + c_proj(o): the GEMM accumulates onto a copy of h.
    float* h1 = ffn ? blk->h1 : h_out;
    cudaError_t e = cudaMemcpyAsync(h1, h, sizeof(float) * blk->M * C, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "residual copy");
    const kattn::ProjStatus ps =
        kattn::gemm_tc(s, ctx->pool, ctx->num_sms, blk->o, C, false, p.w_proj, C, false, h1, C, p.b_proj, M, C, C, 1,
                       ctx->d_status, ctx->wait_ns.load(), &launches);
    if (ps.cuda != cudaSuccess) return cuda_fail(ps.cuda, ps.what);
    if (ffn) {
        BLK_CALL(kattn_layernorm_fwd(ctx, h1, C, p.ln2_w, p.ln2_b, blk->x2, C, M, C, stream));
        BLK_CALL(kattn_kerr_ode_fwd(ctx, blk->x2, C, h_out, C, p.gamma_raw, p.omega, p.alpha_beta, M, C / 2, blk->rk4,
                                    stream));
        e = add(blk, h_out, h_out, h1, s, &launches);
        if (e != cudaSuccess) return cuda_fail(e, "residual add");
    }
    blk->h = h;
    blk->p = p;
    blk->valid = true;
    return ok_with_launches(launches);
}

int kattn_block_bwd(kattn_ctx* ctx, kattn_block* blk, const float* dh_out, float* dh, const kattn_block_grads* grads,
                    int accumulate, void* stream) {
    {
        const int st = check_block(ctx, blk);
        if (st != KATTN_OK) return st;
    }
    if (!blk->valid) return fail(KATTN_ERR_INVALID_ARGUMENT, "no forward of this block to differentiate");
    if (!grads) return fail(KATTN_ERR_INVALID_ARGUMENT, "grads is NULL");
    if (!dh_out || !dh) return fail(KATTN_ERR_INVALID_ARGUMENT, "dh_out / dh is NULL");
    if (!aligned16(dh_out) || !aligned16(dh)) return fail(KATTN_ERR_MISALIGNED, "dh_out / dh not 16-byte aligned");
    const kattn_block_grads& g = *grads;
    const kattn_block_params& p = blk->p;
    const bool ffn = blk->rk4 > 0;
    if (!g.ln1_w || !g.ln1_b || !g.w_attn || !g.b_attn || !g.w_proj || !g.b_proj)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "a gradient of the attention sublayer is NULL");
    if (ffn && (!g.ln2_w || !g.ln2_b || !g.gamma_raw || !g.omega || !g.alpha_beta))
        return fail(KATTN_ERR_INVALID_ARGUMENT, "a gradient of the FFN is NULL");
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int M = static_cast<int>(blk->M), C = blk->C, H = blk->H, d = blk->d;
    const float scale = 1.0f / std::sqrt(static_cast<float>(d));
    const int acc = accumulate ? 1 : 0;
    int launches = 0;
    cudaError_t e;
    // FFN: dh1 = dh_out + LN2^T(KerrODE^T(dh_out)) (src/pipeline.rs:670-690).
    const float* dy1 = dh_out;
    if (ffn) {
        BLK_CALL(kattn_kerr_ode_bwd(ctx, dh_out, C, blk->x2, C, p.gamma_raw, p.omega, p.alpha_beta, blk->t, C,
                                    g.gamma_raw, g.omega, g.alpha_beta, M, C / 2, blk->rk4, acc, stream));
        BLK_CALL(kattn_layernorm_bwd(ctx, blk->t, C, blk->h1, C, p.ln2_w, blk->dh1, C, g.ln2_w, g.ln2_b, M, C, acc,
                                     stream));
        e = add(blk, blk->dh1, blk->dh1, dh_out, s, &launches);
        if (e != cudaSuccess) return cuda_fail(e, "residual add");
        dy1 = blk->dh1;
    }
    // c_proj (src/pipeline.rs:695-704), attention (:705-728), c_attn (:730-737).
    BLK_CALL(kattn_linear_bwd_dx(ctx, dy1, C, p.w_proj, blk->d_o, C, M, C, C, stream));
    BLK_CALL(kattn_linear_bwd_dw(ctx, dy1, C, blk->o, C, g.w_proj, g.b_proj, M, C, C, acc, stream));
    BLK_CALL(kattn_bwd(ctx, blk->qkv, blk->qkv + C, blk->qkv + 2 * C, 3L * C, blk->o, blk->d_o, C, blk->lse,
                       blk->dqkv, blk->dqkv + C, blk->dqkv + 2 * C, 3L * C, blk->B, blk->T, H, d, scale, 1, stream));
    BLK_CALL(kattn_linear_bwd_dx(ctx, blk->dqkv, 3L * C, p.w_attn, blk->t, C, M, 3 * C, C, stream));
    BLK_CALL(kattn_linear_bwd_dw(ctx, blk->dqkv, 3L * C, blk->x1, C, g.w_attn, g.b_attn, M, 3 * C, C, acc, stream));
    // LN1 (:743-750) into the free d_o buffer, then dh = dy1 + that (dh may
    // alias dh_out, which dy1 may be).
    BLK_CALL(kattn_layernorm_bwd(ctx, blk->t, C, blk->h, C, p.ln1_w, blk->d_o, C, g.ln1_w, g.ln1_b, M, C, acc, stream));
    e = add(blk, dh, dy1, blk->d_o, s, &launches);
    if (e != cudaSuccess) return cuda_fail(e, "residual add");
    return ok_with_launches(launches);
}

#pragma GCC visibility pop
}  // extern "C"
