// C ABI of the attention path (include/kerr_attn.h): argument checking,
// device contexts, workspace handling and the host-buffer entry points.
#include <cuda_runtime.h>

#include <climits>
#include <cstdarg>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "kattn_internal.h"
#include "kattn_launch.h"
#include "kerr_attn.h"

// Device-resident state of one forward (the reference's AttnCache):
// q/k/v, o and lse, kept for the backward of the same sequences.
struct kattn_saved {
    kattn_ctx* ctx = nullptr;
    char* buf = nullptr;  // one allocation, grown as needed
    size_t bytes = 0;
    float* qkv = nullptr;  // [B*T][3C]
    float* o = nullptr;    // [B*T][C]
    float* lse = nullptr;  // [B][H][T]
    int B = 0, T = 0, H = 0, d = 0;
    float scale = 0.f;
    int causal = 0;
    bool valid = false;  // a forward completed into it
};

// Fixed backward workspace of kattn_bwd_noalloc: [B][H][T] floats, shared by
// every call on a device.  In host code the name is only a stand-in: the
// device address comes from cudaGetSymbolAddress (kattn_create, per device).
static __device__ __align__(256) float g_noalloc_ws[KATTN_NOALLOC_MAX_ROWS];

namespace kattn_abi {

thread_local char g_last_error[512] = "";
thread_local int g_last_launches = 0;

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    const int status = (e == cudaErrorMemoryAllocation) ? KATTN_ERR_OUT_OF_MEMORY : KATTN_ERR_CUDA;
    return fail(status, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int ok_with_launches(int n) {
    g_last_launches = n;
    return KATTN_OK;
}

}  // namespace kattn_abi

using namespace kattn_abi;

namespace {

constexpr int kTile = 64;  // query / key tile rows of the kernels

int check_shape(const kattn_ctx* ctx, int B, int T, int H, int d, float scale, int causal) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (B < 0 || T < 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "negative size: B=%d T=%d", B, T);
    if (H <= 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "n_head must be positive (got %d)", H);
    if (d != 32 && d != 64 && d != 128)
        return fail(KATTN_ERR_UNSUPPORTED, "head_dim %d unsupported (32, 64 or 128)", d);
    if (!std::isfinite(scale)) return fail(KATTN_ERR_INVALID_ARGUMENT, "scale is not finite");
    if (causal != 0 && causal != 1) return fail(KATTN_ERR_INVALID_ARGUMENT, "causal must be 0 or 1");
    const long tiles = (static_cast<long>(T) + kTile - 1) / kTile;
    if (static_cast<long>(B) * H * tiles > INT_MAX)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "problem too large: B*H*ceil(T/64) exceeds 2^31-1");
    if (static_cast<long>(H) * d > INT_MAX / 4) return fail(KATTN_ERR_INVALID_ARGUMENT, "H*d too large");
    return KATTN_OK;
}

int check_tensor(const char* name, const void* p, long ld, int C, bool device) {
    if (!p) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    if (ld < C) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s row stride %ld < H*d = %d", name, ld, C);
    if (device) {
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
            return fail(KATTN_ERR_MISALIGNED, "%s is not 16-byte aligned", name);
        if (ld % 4 != 0) return fail(KATTN_ERR_MISALIGNED, "%s row stride %ld is not a multiple of 4", name, ld);
    }
    return KATTN_OK;
}

int check_vec(const char* name, const void* p, bool device) {
    if (!p) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    if (device && reinterpret_cast<uintptr_t>(p) % 4 != 0)
        return fail(KATTN_ERR_MISALIGNED, "%s is not 4-byte aligned", name);
    return KATTN_OK;
}

#define KATTN_TRY(expr)                  \
    do {                                 \
        const int _s = (expr);           \
        if (_s != KATTN_OK) return _s;   \
    } while (0)

int fwd_checks(const kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv,
               const float* o, long ld_o, const float* lse, int B, int T, int H, int d, float scale,
               int causal, bool device) {
    KATTN_TRY(check_shape(ctx, B, T, H, d, scale, causal));
    if (B == 0 || T == 0) return KATTN_OK;
    const int C = H * d;
    KATTN_TRY(check_tensor("q", q, ld_qkv, C, device));
    KATTN_TRY(check_tensor("k", k, ld_qkv, C, device));
    KATTN_TRY(check_tensor("v", v, ld_qkv, C, device));
    KATTN_TRY(check_tensor("o", o, ld_o, C, device));
    KATTN_TRY(check_vec("lse", lse, device));
    return KATTN_OK;
}

int bwd_checks(const kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv,
               const float* o, const float* dout, long ld_o, const float* lse, const float* dq,
               const float* dk, const float* dv, long ld_d, int B, int T, int H, int d, float scale,
               int causal, bool device) {
    KATTN_TRY(check_shape(ctx, B, T, H, d, scale, causal));
    if (B == 0 || T == 0) return KATTN_OK;
    const int C = H * d;
    KATTN_TRY(check_tensor("q", q, ld_qkv, C, device));
    KATTN_TRY(check_tensor("k", k, ld_qkv, C, device));
    KATTN_TRY(check_tensor("v", v, ld_qkv, C, device));
    KATTN_TRY(check_tensor("o", o, ld_o, C, device));
    KATTN_TRY(check_tensor("dout", dout, ld_o, C, device));
    KATTN_TRY(check_vec("lse", lse, device));
    KATTN_TRY(check_tensor("dq", dq, ld_d, C, device));
    KATTN_TRY(check_tensor("dk", dk, ld_d, C, device));
    KATTN_TRY(check_tensor("dv", dv, ld_d, C, device));
    return KATTN_OK;
}

// AUTO's kernel family: the tensor-core kernels at head_dim 64, and at head_dim
// 32 from 16384 (batch, head, position) rows up.  Below that the FFMA kernels'
// shorter set-up wins: at 4 x 4 heads x 64 positions a forward + backward took
// 60 us on FFMA against 76 us on the tensor cores; at 64 x 4 x 256, 170 us
// against 65 us.
bool auto_tensor(int d, long rows) { return d == 64 || (d == 32 && rows >= 16384); }

// Forward launch on the kernel family the context selects, with the
// context's wait limit (and, once, its diagnostic hook) on the tensor path.
cudaError_t dispatch_fwd(kattn_ctx* ctx, const kattn::FwdArgs& a, cudaStream_t s, int* launches) {
    const int path = ctx->path.load(std::memory_order_relaxed);
    const long rows = static_cast<long>(a.B) * a.H * a.T;
    if (kattn::fwd_tc_supported(a) &&
        (path == KATTN_PATH_TENSOR || (path == KATTN_PATH_AUTO && auto_tensor(a.d, rows)))) {
        kattn::FwdArgs b = a;
        b.wait_ns = ctx->wait_ns.load(std::memory_order_relaxed);
        b.withhold_first_key_load = ctx->withhold_next_load.exchange(0);
        return kattn::launch_fwd_tc(b, ctx->num_sms, ctx->d_status, s, launches);
    }
    return kattn::launch_fwd(a, ctx->num_sms, s, launches);
}

// Backward launch on the kernel family the context selects.
cudaError_t dispatch_bwd(kattn_ctx* ctx, const kattn::BwdArgs& a, cudaStream_t s, int* launches) {
    const int path = ctx->path.load(std::memory_order_relaxed);
    const long rows = static_cast<long>(a.B) * a.H * a.T;
    const bool tensor = kattn::bwd_tc_supported(a) &&
                        (path == KATTN_PATH_TENSOR || (path == KATTN_PATH_AUTO && auto_tensor(a.d, rows)));
    kattn::BwdArgs b = a;
    b.wait_ns = ctx->wait_ns.load(std::memory_order_relaxed);
    // Deterministic dQ: every key tile stores its contribution into its own
    // slice of a pool workspace, and one pass adds the slices in key-tile
    // order (the reference sums dQ over keys sequentially,
    // src/backward.rs:508-512); otherwise the tiles add into dq directly.
    const bool det = ctx->deterministic.load(std::memory_order_relaxed) != 0;
    const int key_rows = tensor ? kattn::kBwdTcKeyRows : kattn::kBwdF32KeyRows;
    if (det) {
        const size_t n_kt = static_cast<size_t>((a.T + key_rows - 1) / key_rows);
        const size_t bytes = sizeof(float) * n_kt * a.B * a.T * a.H * a.d;
        const cudaError_t e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&b.dq_part), bytes, ctx->pool, s);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = tensor ? kattn::launch_bwd_tc(b, ctx->num_sms, ctx->d_status, s, launches)
                           : kattn::launch_bwd(b, ctx->num_sms, s, launches);
    if (det) {
        if (e == cudaSuccess) e = kattn::launch_bwd_dq_reduce(b, key_rows, ctx->num_sms, s, launches);
        const cudaError_t ef = cudaFreeAsync(b.dq_part, s);
        if (e == cudaSuccess) e = ef;
    }
    return e;
}

int path_check(const kattn_ctx* ctx, int d) {
    if (ctx->path.load(std::memory_order_relaxed) == KATTN_PATH_TENSOR && d != 64 && d != 32)
        return fail(KATTN_ERR_UNSUPPORTED, "the tensor-core path supports head_dim 64 and 32 (got %d)", d);
    return KATTN_OK;
}

// Checks of a row-major f32 operand of the projection calls: rows x cols at
// row stride ld, 16-byte aligned, ld and cols multiples of 4 floats.
int check_matrix(const char* name, const void* p, long ld, long rows, long cols) {
    if (rows > 0 && cols > 0 && !p) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    if (ld < cols) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s row stride %ld < %ld columns", name, ld, cols);
    if (p && reinterpret_cast<uintptr_t>(p) % 16 != 0)
        return fail(KATTN_ERR_MISALIGNED, "%s is not 16-byte aligned", name);
    if (ld % 4 != 0 || cols % 4 != 0)
        return fail(KATTN_ERR_MISALIGNED, "%s row stride %ld / width %ld not a multiple of 4", name, ld, cols);
    return KATTN_OK;
}

int check_dims(int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "negative size (M=%d N=%d K=%d)", M, N, K);
    if (static_cast<long>(M) * N > INT_MAX || static_cast<long>(M) * K > INT_MAX || static_cast<long>(N) * K > INT_MAX)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "problem too large (M=%d N=%d K=%d)", M, N, K);
    return KATTN_OK;
}

int proj_result(const kattn::ProjStatus& st, int launches) {
    if (st.cuda != cudaSuccess) return cuda_fail(st.cuda, st.what);
    return ok_with_launches(launches);
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int ensure_arena(kattn_ctx* ctx, size_t bytes) {
    if (ctx->arena_bytes >= bytes) return KATTN_OK;
    if (ctx->arena) {
        cudaError_t e = cudaFree(ctx->arena);
        ctx->arena = nullptr;
        ctx->arena_bytes = 0;
        if (e != cudaSuccess) return cuda_fail(e, "cudaFree(staging)");
    }
    cudaError_t e = cudaMalloc(&ctx->arena, bytes);
    if (e != cudaSuccess) {
        ctx->arena = nullptr;
        return cuda_fail(e, "cudaMalloc(staging)");
    }
    ctx->arena_bytes = bytes;
    return KATTN_OK;
}

// Copies a [rows][C] block with row stride ld (elements) between host and a
// packed device block with row stride ldd.
cudaError_t copy_rows(float* dst, long ld_dst, const float* src, long ld_src, int C, long rows,
                      cudaMemcpyKind kind, cudaStream_t s) {
    if (ld_dst == C && ld_src == C)
        return cudaMemcpyAsync(dst, src, sizeof(float) * C * rows, kind, s);
    return cudaMemcpy2DAsync(dst, sizeof(float) * ld_dst, src, sizeof(float) * ld_src, sizeof(float) * C,
                             static_cast<size_t>(rows), kind, s);
}

// Host-buffer calls are pipelined over chunks of whole sequences: chunk c's
// inputs go up on ctx->h2d, its kernels run on ctx->stream once they have
// landed, and its outputs come down on ctx->d2h once the kernels are done.
// So one chunk's download overlaps the next chunk's kernels and the upload
// of the one after (the link carries both directions at once).  Chunks move
// at least ~8 MB (inputs plus outputs) and are at most 8; a small problem is
// one chunk.
struct Chunks {
    int n = 1, per = 0;  // chunk count, sequences per chunk
    Chunks(int B, size_t bytes) {
        const size_t target = 8u << 20;
        long want = static_cast<long>(bytes / target);
        if (want < 1) want = 1;
        if (want > 8) want = 8;
        if (want > B) want = B;
        per = static_cast<int>((B + want - 1) / want);
        n = (B + per - 1) / per;
    }
    int b0(int c) const { return c * per; }
    int count(int c, int B) const { return std::min(per, B - c * per); }
};

int ensure_events(kattn_ctx* ctx, size_t n) {
    while (ctx->events.size() < n) {
        cudaEvent_t ev;
        const cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
        ctx->events.push_back(ev);
    }
    return KATTN_OK;
}

// Makes `waiter` wait for the work enqueued so far on `from` (event `ev`).
cudaError_t hand_off(cudaStream_t from, cudaStream_t waiter, cudaEvent_t ev) {
    cudaError_t e = cudaEventRecord(ev, from);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(waiter, ev, 0);
    return e;
}

// Waits for everything the three host-call streams hold (also after an
// error, so that no copy into the staging buffers outlives the call).
cudaError_t drain_host_streams(kattn_ctx* ctx) {
    cudaError_t e1 = cudaStreamSynchronize(ctx->h2d);
    cudaError_t e2 = cudaStreamSynchronize(ctx->stream);
    cudaError_t e3 = cudaStreamSynchronize(ctx->d2h);
    return e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3);
}

// Host q/k/v rows [r0, r0+rows) -> the packed device [rows][3C] block at dqkv.
cudaError_t upload_qkv(float* dqkv, const float* q, const float* k, const float* v, long ld_qkv, int C, long r0,
                       long rows, cudaStream_t s) {
    if (k == q + C && v == q + 2 * C && ld_qkv == 3L * C)
        return cudaMemcpyAsync(dqkv, q + r0 * ld_qkv, sizeof(float) * rows * 3 * C, cudaMemcpyHostToDevice, s);
    cudaError_t e = copy_rows(dqkv, 3L * C, q + r0 * ld_qkv, ld_qkv, C, rows, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = copy_rows(dqkv + C, 3L * C, k + r0 * ld_qkv, ld_qkv, C, rows, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = copy_rows(dqkv + 2 * C, 3L * C, v + r0 * ld_qkv, ld_qkv, C, rows, cudaMemcpyHostToDevice, s);
    return e;
}

// The packed device [rows][3C] gradient block -> host dq/dk/dv rows [r0, r0+rows).
cudaError_t download_grads(float* dq, float* dk, float* dv, long ld_d, const float* dgrad, int C, long r0, long rows,
                           cudaStream_t s) {
    if (dk == dq + C && dv == dq + 2 * C && ld_d == 3L * C)
        return cudaMemcpyAsync(dq + r0 * ld_d, dgrad, sizeof(float) * rows * 3 * C, cudaMemcpyDeviceToHost, s);
    cudaError_t e = copy_rows(dq + r0 * ld_d, ld_d, dgrad, 3L * C, C, rows, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = copy_rows(dk + r0 * ld_d, ld_d, dgrad + C, 3L * C, C, rows, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess)
        e = copy_rows(dv + r0 * ld_d, ld_d, dgrad + 2 * C, 3L * C, C, rows, cudaMemcpyDeviceToHost, s);
    return e;
}

// Forward from host buffers through the pipelined chunks, into the device
// buffers dqkv [B*T][3C], d_o [B*T][C], d_lse [B][H][T] (o and lse also come
// back to the host).  The caller holds host_mu and has the device current.
int fwd_host_run(kattn_ctx* ctx, float* dqkv, float* d_o, float* d_lse, const float* q, const float* k,
                 const float* v, long ld_qkv, float* o, long ld_o, float* lse, int B, int T, int H, int d,
                 float scale, int causal) {
    const int C = H * d;
    const Chunks ch(B, sizeof(float) * static_cast<size_t>(B) * T * (4 * C + H));  // q/k/v up; o, lse down
    KATTN_TRY(ensure_events(ctx, 2 * static_cast<size_t>(ch.n)));
    int launches = 0;
    cudaError_t e = cudaSuccess;
    const char* what = "";
    for (int c = 0; c < ch.n && e == cudaSuccess; ++c) {
        const int b0 = ch.b0(c), bc = ch.count(c, B);
        const long r0 = static_cast<long>(b0) * T, rows = static_cast<long>(bc) * T;
        const long l0 = static_cast<long>(b0) * H * T;
        float* cq = dqkv + r0 * 3 * C;
        what = "host-to-device copy";
        e = upload_qkv(cq, q, k, v, ld_qkv, C, r0, rows, ctx->h2d);
        if (e == cudaSuccess) e = hand_off(ctx->h2d, ctx->stream, ctx->events[2 * c]);
        if (e != cudaSuccess) break;
        what = "forward launch";
        const kattn::FwdArgs a{cq, cq + C, cq + 2 * C, 3L * C, d_o + r0 * C, C, d_lse + l0, bc, T, H, d, scale, causal};
        e = dispatch_fwd(ctx, a, ctx->stream, &launches);
        if (e == cudaSuccess) e = hand_off(ctx->stream, ctx->d2h, ctx->events[2 * c + 1]);
        if (e != cudaSuccess) break;
        what = "device-to-host copy";
        e = copy_rows(o + r0 * ld_o, ld_o, d_o + r0 * C, C, C, rows, cudaMemcpyDeviceToHost, ctx->d2h);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(lse + l0, d_lse + l0, sizeof(float) * static_cast<size_t>(bc) * H * T,
                                cudaMemcpyDeviceToHost, ctx->d2h);
    }
    const cudaError_t es = drain_host_streams(ctx);
    if (e != cudaSuccess) return cuda_fail(e, what);
    if (es != cudaSuccess) return cuda_fail(es, "cudaStreamSynchronize");
    return ok_with_launches(launches);
}

// Backward from host buffers through the pipelined chunks.  q/k/v, o and lse
// are uploaded into d_qkv / d_o / d_lse when `upload_saved` is set and are
// already resident there otherwise; dout goes up to d_do; the gradients come
// down from d_grad.  d_dsum is the [B][H][T] workspace.
int bwd_host_run(kattn_ctx* ctx, float* d_qkv, float* d_o, float* d_lse, bool upload_saved, const float* q,
                 const float* k, const float* v, long ld_qkv, const float* o, const float* lse, const float* dout,
                 long ld_o, float* dq, float* dk, float* dv, long ld_d, float* d_do, float* d_grad, float* d_dsum,
                 int B, int T, int H, int d, float scale, int causal) {
    const int C = H * d;
    const size_t per_row = (upload_saved ? 5u * C + H : 1u * C) + 3u * C;  // inputs up, gradients down
    const Chunks ch(B, sizeof(float) * static_cast<size_t>(B) * T * per_row);
    KATTN_TRY(ensure_events(ctx, 2 * static_cast<size_t>(ch.n)));
    int launches = 0;
    cudaError_t e = cudaSuccess;
    const char* what = "";
    for (int c = 0; c < ch.n && e == cudaSuccess; ++c) {
        const int b0 = ch.b0(c), bc = ch.count(c, B);
        const long r0 = static_cast<long>(b0) * T, rows = static_cast<long>(bc) * T;
        const long l0 = static_cast<long>(b0) * H * T;
        float* cq = d_qkv + r0 * 3 * C;
        float* cg = d_grad + r0 * 3 * C;
        what = "host-to-device copy";
        if (upload_saved) {
            e = upload_qkv(cq, q, k, v, ld_qkv, C, r0, rows, ctx->h2d);
            if (e == cudaSuccess) e = copy_rows(d_o + r0 * C, C, o + r0 * ld_o, ld_o, C, rows, cudaMemcpyHostToDevice, ctx->h2d);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(d_lse + l0, lse + l0, sizeof(float) * static_cast<size_t>(bc) * H * T,
                                    cudaMemcpyHostToDevice, ctx->h2d);
        }
        if (e == cudaSuccess)
            e = copy_rows(d_do + r0 * C, C, dout + r0 * ld_o, ld_o, C, rows, cudaMemcpyHostToDevice, ctx->h2d);
        if (e == cudaSuccess) e = hand_off(ctx->h2d, ctx->stream, ctx->events[2 * c]);
        if (e != cudaSuccess) break;
        what = "backward launch";
        const kattn::BwdArgs a{cq, cq + C, cq + 2 * C, 3L * C, d_o + r0 * C, d_do + r0 * C, C, d_lse + l0,
                               cg, cg + C, cg + 2 * C, 3L * C, d_dsum + l0, bc, T, H, d, scale, causal};
        e = dispatch_bwd(ctx, a, ctx->stream, &launches);
        if (e == cudaSuccess) e = hand_off(ctx->stream, ctx->d2h, ctx->events[2 * c + 1]);
        if (e != cudaSuccess) break;
        what = "device-to-host copy";
        e = download_grads(dq, dk, dv, ld_d, cg, C, r0, rows, ctx->d2h);
    }
    const cudaError_t es = drain_host_streams(ctx);
    if (e != cudaSuccess) return cuda_fail(e, what);
    if (es != cudaSuccess) return cuda_fail(es, "cudaStreamSynchronize");
    return ok_with_launches(launches);
}

}  // namespace

extern "C" {
#pragma GCC visibility push(default)

int kattn_version(void) { return 100; }

const char* kattn_strerror(int status) {
    switch (status) {
        case KATTN_OK: return "ok";
        case KATTN_ERR_INVALID_ARGUMENT: return "invalid argument";
        case KATTN_ERR_UNSUPPORTED: return "unsupported shape";
        case KATTN_ERR_MISALIGNED: return "misaligned pointer or stride";
        case KATTN_ERR_DEVICE: return "no usable sm_100 CUDA device";
        case KATTN_ERR_CUDA: return "CUDA runtime error";
        case KATTN_ERR_OUT_OF_MEMORY: return "out of memory";
        case KATTN_ERR_DEVICE_TIMEOUT: return "a kernel gave up a bounded wait on the device";
        default: return "unknown status";
    }
}

const char* kattn_last_error(void) { return g_last_error; }

int kattn_last_launch_count(void) { return g_last_launches; }

int kattn_create(int device, kattn_ctx** out) {
    if (!out) return fail(KATTN_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(KATTN_ERR_DEVICE, "no CUDA device (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
    }
    if (device < 0 || device >= n) return fail(KATTN_ERR_DEVICE, "device %d out of range [0, %d)", device, n);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        return fail(KATTN_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a only", device,
                    prop.major, prop.minor);
    DeviceScope scope(device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    kattn_ctx* ctx = new (std::nothrow) kattn_ctx();
    if (!ctx) return fail(KATTN_ERR_OUT_OF_MEMORY, "host allocation of the context failed");
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->d2h, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
        delete ctx;
        return cuda_fail(e, "cudaStreamCreate");
    }
    e = cudaMalloc(&ctx->d_status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(int));
    if (e != cudaSuccess) {
        cudaStreamDestroy(ctx->stream);
        cudaStreamDestroy(ctx->h2d);
        cudaStreamDestroy(ctx->d2h);
        if (ctx->d_status) cudaFree(ctx->d_status);
        delete ctx;
        return cuda_fail(e, "status word");
    }
    // Device address of the fixed workspace of kattn_bwd_noalloc (this
    // device is current here).
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ctx->noalloc_ws), g_noalloc_ws);
    const char* what = "cudaGetSymbolAddress(workspace)";
    if (e == cudaSuccess) {
        // Per-call workspace (the backward's [B][H][T] rows, column-sum
        // partials) comes from a pool this context owns.  It keeps freed
        // blocks cached until kattn_destroy, so a steady stream of calls does
        // not return memory to the driver at every synchronisation; the
        // device's default pool and its settings are left as they are.
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        what = "cudaMemPoolCreate";
        e = cudaMemPoolCreate(&ctx->pool, &props);
        if (e == cudaSuccess) {
            uint64_t keep = UINT64_MAX;
            what = "cudaMemPoolSetAttribute";
            e = cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
    }
    if (e != cudaSuccess) {
        if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
        cudaStreamDestroy(ctx->stream);
        cudaStreamDestroy(ctx->h2d);
        cudaStreamDestroy(ctx->d2h);
        cudaFree(ctx->d_status);
        delete ctx;
        return cuda_fail(e, what);
    }
    *out = ctx;
    return KATTN_OK;
}

int kattn_destroy(kattn_ctx* ctx) {
    if (!ctx) return KATTN_OK;
    int status = KATTN_OK;
    {
        DeviceScope scope(ctx->device);
        for (cudaStream_t* s : {&ctx->h2d, &ctx->stream, &ctx->d2h}) {
            if (!*s) continue;
            cudaError_t e = cudaStreamSynchronize(*s);
            if (e != cudaSuccess && status == KATTN_OK) status = cuda_fail(e, "cudaStreamSynchronize");
            cudaStreamDestroy(*s);
        }
        for (cudaEvent_t ev : ctx->events) cudaEventDestroy(ev);
        if (ctx->arena) cudaFree(ctx->arena);
        if (ctx->d_status) cudaFree(ctx->d_status);
        // Blocks still owed to the pool by work in flight on callers' streams
        // are released by the driver once that work frees them.
        if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
    }
    delete ctx;
    return status;
}

int kattn_set_path(kattn_ctx* ctx, int path) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (path != KATTN_PATH_AUTO && path != KATTN_PATH_FFMA && path != KATTN_PATH_TENSOR)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "unknown path %d", path);
    ctx->path.store(path);
    return KATTN_OK;
}

int kattn_set_wait_limit(kattn_ctx* ctx, unsigned long long ns) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    ctx->wait_ns.store(ns == 0 ? kDefaultWaitNs : ns);
    return KATTN_OK;
}

int kattn_set_deterministic(kattn_ctx* ctx, int on) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    ctx->deterministic.store(on ? 1 : 0);
    return KATTN_OK;
}

int kattn_test_withhold_next_load(kattn_ctx* ctx) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    ctx->withhold_next_load.store(1);
    return KATTN_OK;
}

int kattn_check_device(kattn_ctx* ctx) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
    int flag = 0;
    e = cudaMemcpy(&flag, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && flag != 0) e = cudaMemset(ctx->d_status, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "status word");
    if (flag != 0) return fail(KATTN_ERR_DEVICE_TIMEOUT, "a kernel reported a wait timeout (flags 0x%x)", flag);
    return KATTN_OK;
}

int kattn_fwd(kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv, float* o, long ld_o,
              float* lse, int B, int T, int H, int d, float scale, int causal, void* stream) {
    g_last_launches = 0;
    KATTN_TRY(fwd_checks(ctx, q, k, v, ld_qkv, o, ld_o, lse, B, T, H, d, scale, causal, true));
    if (B == 0 || T == 0) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    KATTN_TRY(path_check(ctx, d));
    kattn::FwdArgs a{q, k, v, ld_qkv, o, ld_o, lse, B, T, H, d, scale, causal};
    int launches = 0;
    cudaError_t e = dispatch_fwd(ctx, a, static_cast<cudaStream_t>(stream), &launches);
    if (e != cudaSuccess) return cuda_fail(e, "forward launch");
    return ok_with_launches(launches);
}

int kattn_bwd(kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv, const float* o,
              const float* dout, long ld_o, const float* lse, float* dq, float* dk, float* dv, long ld_dqkv, int B,
              int T, int H, int d, float scale, int causal, void* stream) {
    g_last_launches = 0;
    KATTN_TRY(bwd_checks(ctx, q, k, v, ld_qkv, o, dout, ld_o, lse, dq, dk, dv, ld_dqkv, B, T, H, d, scale, causal,
                         true));
    if (B == 0 || T == 0) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    kattn::BwdArgs a{q, k, v, ld_qkv, o, dout, ld_o, lse, dq, dk, dv, ld_dqkv, nullptr, B, T, H, d, scale, causal};
    // D = rowsum(dout * o) is staged in a [B][H][T] workspace.
    const size_t ws = sizeof(float) * static_cast<size_t>(B) * H * T;
    cudaError_t e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&a.dsum), ws, ctx->pool, s);
    if (e != cudaSuccess) return cuda_fail(e, "workspace allocation");
    int launches = 0;
    e = dispatch_bwd(ctx, a, s, &launches);
    const cudaError_t ef = a.dsum ? cudaFreeAsync(a.dsum, s) : cudaSuccess;
    if (e != cudaSuccess) return cuda_fail(e, "backward launch");
    if (ef != cudaSuccess) return cuda_fail(ef, "cudaFreeAsync(workspace)");
    return ok_with_launches(launches);
}

int kattn_bwd_noalloc(kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv,
                      const float* o, const float* dout, long ld_o, const float* lse, float* dq, float* dk,
                      float* dv, long ld_dqkv, int B, int T, int H, int d, float scale, int causal,
                      void* stream) {
    g_last_launches = 0;
    KATTN_TRY(bwd_checks(ctx, q, k, v, ld_qkv, o, dout, ld_o, lse, dq, dk, dv, ld_dqkv, B, T, H, d, scale, causal,
                         true));
    if (B == 0 || T == 0) return ok_with_launches(0);
    const long rows = static_cast<long>(B) * H * T;
    if (rows > KATTN_NOALLOC_MAX_ROWS)
        return fail(KATTN_ERR_INVALID_ARGUMENT,
                    "B*H*T = %ld exceeds the fixed workspace of the allocation-free backward (%ld)", rows,
                    static_cast<long>(KATTN_NOALLOC_MAX_ROWS));
    KATTN_TRY(path_check(ctx, d));
    if (ctx->deterministic.load(std::memory_order_relaxed))
        return fail(KATTN_ERR_UNSUPPORTED,
                    "the deterministic dQ mode needs a per-call workspace: use kattn_bwd on this context");
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    kattn::BwdArgs a{q, k, v, ld_qkv, o, dout, ld_o, lse, dq, dk, dv, ld_dqkv, ctx->noalloc_ws,
                     B, T, H, d, scale, causal};
    int launches = 0;
    cudaError_t e = dispatch_bwd(ctx, a, static_cast<cudaStream_t>(stream), &launches);
    if (e != cudaSuccess) return cuda_fail(e, "backward launch");
    return ok_with_launches(launches);
}

int kattn_fwd_host(kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv, float* o,
                   long ld_o, float* lse, int B, int T, int H, int d, float scale, int causal) {
    g_last_launches = 0;
    KATTN_TRY(fwd_checks(ctx, q, k, v, ld_qkv, o, ld_o, lse, B, T, H, d, scale, causal, false));
    if (B == 0 || T == 0) return ok_with_launches(0);
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    KATTN_TRY(path_check(ctx, d));
    const int C = H * d;
    const long rows = static_cast<long>(B) * T;
    const size_t qkv_b = align256(sizeof(float) * rows * 3 * C);
    const size_t o_b = align256(sizeof(float) * rows * C);
    const size_t lse_b = align256(sizeof(float) * static_cast<size_t>(B) * H * T);
    KATTN_TRY(ensure_arena(ctx, qkv_b + o_b + lse_b));
    return fwd_host_run(ctx, reinterpret_cast<float*>(ctx->arena), reinterpret_cast<float*>(ctx->arena + qkv_b),
                        reinterpret_cast<float*>(ctx->arena + qkv_b + o_b), q, k, v, ld_qkv, o, ld_o, lse, B, T, H, d,
                        scale, causal);
}

int kattn_bwd_host(kattn_ctx* ctx, const float* q, const float* k, const float* v, long ld_qkv, const float* o,
                   const float* dout, long ld_o, const float* lse, float* dq, float* dk, float* dv, long ld_dqkv,
                   int B, int T, int H, int d, float scale, int causal) {
    g_last_launches = 0;
    KATTN_TRY(bwd_checks(ctx, q, k, v, ld_qkv, o, dout, ld_o, lse, dq, dk, dv, ld_dqkv, B, T, H, d, scale, causal,
                         false));
    if (B == 0 || T == 0) return ok_with_launches(0);
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    KATTN_TRY(path_check(ctx, d));
    const int C = H * d;
    const long rows = static_cast<long>(B) * T;
    const size_t qkv_b = align256(sizeof(float) * rows * 3 * C);
    const size_t row_b = align256(sizeof(float) * rows * C);
    const size_t lse_b = align256(sizeof(float) * static_cast<size_t>(B) * H * T);
    KATTN_TRY(ensure_arena(ctx, 2 * qkv_b + 2 * row_b + 2 * lse_b));
    char* base = ctx->arena;
    float* d_qkv = reinterpret_cast<float*>(base);
    float* d_grad = reinterpret_cast<float*>(base + qkv_b);
    float* d_o = reinterpret_cast<float*>(base + 2 * qkv_b);
    float* d_do = reinterpret_cast<float*>(base + 2 * qkv_b + row_b);
    float* d_lse = reinterpret_cast<float*>(base + 2 * qkv_b + 2 * row_b);
    float* d_dsum = reinterpret_cast<float*>(base + 2 * qkv_b + 2 * row_b + lse_b);
    return bwd_host_run(ctx, d_qkv, d_o, d_lse, true, q, k, v, ld_qkv, o, lse, dout, ld_o, dq, dk, dv, ld_dqkv, d_do,
                        d_grad, d_dsum, B, T, H, d, scale, causal);
}

int kattn_saved_create(kattn_ctx* ctx, kattn_saved** out) {
    if (!out) return fail(KATTN_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    kattn_saved* s = new (std::nothrow) kattn_saved();
    if (!s) return fail(KATTN_ERR_OUT_OF_MEMORY, "host allocation of the saved state failed");
    s->ctx = ctx;
    *out = s;
    return KATTN_OK;
}

int kattn_saved_destroy(kattn_saved* saved) {
    if (!saved) return KATTN_OK;
    int status = KATTN_OK;
    if (saved->buf) {
        kattn_ctx* ctx = saved->ctx;
        std::lock_guard<std::mutex> lock(ctx->host_mu);
        DeviceScope scope(ctx->device);
        const cudaError_t e = cudaFree(saved->buf);
        if (e != cudaSuccess) status = cuda_fail(e, "cudaFree(saved state)");
    }
    delete saved;
    return status;
}

int kattn_fwd_host_save(kattn_ctx* ctx, kattn_saved* saved, const float* q, const float* k, const float* v,
                        long ld_qkv, float* o, long ld_o, float* lse, int B, int T, int H, int d, float scale,
                        int causal) {
    g_last_launches = 0;
    if (!saved) return fail(KATTN_ERR_INVALID_ARGUMENT, "saved is NULL");
    if (saved->ctx != ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "saved state belongs to another context");
    KATTN_TRY(fwd_checks(ctx, q, k, v, ld_qkv, o, ld_o, lse, B, T, H, d, scale, causal, false));
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    saved->valid = false;
    saved->B = B;
    saved->T = T;
    saved->H = H;
    saved->d = d;
    saved->scale = scale;
    saved->causal = causal;
    if (B == 0 || T == 0) {
        saved->valid = true;
        return ok_with_launches(0);
    }
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    KATTN_TRY(path_check(ctx, d));
    const int C = H * d;
    const long rows = static_cast<long>(B) * T;
    const size_t qkv_b = align256(sizeof(float) * rows * 3 * C);
    const size_t o_b = align256(sizeof(float) * rows * C);
    const size_t lse_b = align256(sizeof(float) * static_cast<size_t>(B) * H * T);
    if (saved->bytes < qkv_b + o_b + lse_b) {
        if (saved->buf) {
            const cudaError_t e = cudaFree(saved->buf);
            saved->buf = nullptr;
            saved->bytes = 0;
            if (e != cudaSuccess) return cuda_fail(e, "cudaFree(saved state)");
        }
        const cudaError_t e = cudaMalloc(&saved->buf, qkv_b + o_b + lse_b);
        if (e != cudaSuccess) {
            saved->buf = nullptr;
            return cuda_fail(e, "cudaMalloc(saved state)");
        }
        saved->bytes = qkv_b + o_b + lse_b;
    }
    saved->qkv = reinterpret_cast<float*>(saved->buf);
    saved->o = reinterpret_cast<float*>(saved->buf + qkv_b);
    saved->lse = reinterpret_cast<float*>(saved->buf + qkv_b + o_b);
    const int st = fwd_host_run(ctx, saved->qkv, saved->o, saved->lse, q, k, v, ld_qkv, o, ld_o, lse, B, T, H, d,
                                scale, causal);
    saved->valid = st == KATTN_OK;
    return st;
}

int kattn_bwd_host_saved(kattn_ctx* ctx, const kattn_saved* saved, const float* dout, long ld_o, float* dq,
                         float* dk, float* dv, long ld_dqkv) {
    g_last_launches = 0;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (!saved) return fail(KATTN_ERR_INVALID_ARGUMENT, "saved is NULL");
    if (saved->ctx != ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "saved state belongs to another context");
    if (!saved->valid) return fail(KATTN_ERR_INVALID_ARGUMENT, "saved state holds no completed forward");
    const int B = saved->B, T = saved->T, H = saved->H, d = saved->d;
    if (B == 0 || T == 0) return ok_with_launches(0);
    const int C = H * d;
    KATTN_TRY(check_tensor("dout", dout, ld_o, C, false));
    KATTN_TRY(check_tensor("dq", dq, ld_dqkv, C, false));
    KATTN_TRY(check_tensor("dk", dk, ld_dqkv, C, false));
    KATTN_TRY(check_tensor("dv", dv, ld_dqkv, C, false));
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    KATTN_TRY(path_check(ctx, d));
    const long rows = static_cast<long>(B) * T;
    const size_t qkv_b = align256(sizeof(float) * rows * 3 * C);
    const size_t row_b = align256(sizeof(float) * rows * C);
    const size_t lse_b = align256(sizeof(float) * static_cast<size_t>(B) * H * T);
    KATTN_TRY(ensure_arena(ctx, qkv_b + row_b + lse_b));
    float* d_grad = reinterpret_cast<float*>(ctx->arena);
    float* d_do = reinterpret_cast<float*>(ctx->arena + qkv_b);
    float* d_dsum = reinterpret_cast<float*>(ctx->arena + qkv_b + row_b);
    return bwd_host_run(ctx, saved->qkv, saved->o, saved->lse, false, nullptr, nullptr, nullptr, 0, nullptr, nullptr,
                        dout, ld_o, dq, dk, dv, ld_dqkv, d_do, d_grad, d_dsum, B, T, H, d, saved->scale,
                        saved->causal);
}

int kattn_linear_fwd(kattn_ctx* ctx, const float* x, long ld_x, const float* w, const float* b, float* y, long ld_y,
                     int M, int N, int K, void* stream) {
    g_last_launches = 0;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    KATTN_TRY(check_dims(M, N, K));
    KATTN_TRY(check_matrix("x", x, ld_x, M, K));
    KATTN_TRY(check_matrix("w", w, K, N, K));
    KATTN_TRY(check_matrix("y", y, ld_y, M, N));
    if (b && reinterpret_cast<uintptr_t>(b) % 4 != 0) return fail(KATTN_ERR_MISALIGNED, "b is not 4-byte aligned");
    if (M == 0 || N == 0) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int launches = 0;
    const kattn::ProjStatus st = kattn::proj_forward(ctx->num_sms, s, ctx->pool, ctx->d_status, ctx->wait_ns.load(),
                                                     x, ld_x, w, b, y, ld_y, M, N, K, &launches);
    return proj_result(st, launches);
}

int kattn_linear_bwd_dx(kattn_ctx* ctx, const float* dy, long ld_dy, const float* w, float* dx, long ld_dx, int M,
                        int N, int K, void* stream) {
    g_last_launches = 0;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    KATTN_TRY(check_dims(M, N, K));
    KATTN_TRY(check_matrix("dy", dy, ld_dy, M, N));
    KATTN_TRY(check_matrix("w", w, K, N, K));
    KATTN_TRY(check_matrix("dx", dx, ld_dx, M, K));
    if (M == 0 || K == 0) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int launches = 0;
    const kattn::ProjStatus st = kattn::proj_backward_dx(ctx->num_sms, s, ctx->pool, ctx->d_status,
                                                         ctx->wait_ns.load(), dy, ld_dy, w, dx, ld_dx, M, N, K,
                                                         &launches);
    return proj_result(st, launches);
}

int kattn_linear_bwd_dw(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x, float* dw, float* db,
                        int M, int N, int K, int accumulate, void* stream) {
    g_last_launches = 0;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    KATTN_TRY(check_dims(M, N, K));
    KATTN_TRY(check_matrix("dy", dy, ld_dy, M, N));
    KATTN_TRY(check_matrix("x", x, ld_x, M, K));
    KATTN_TRY(check_matrix("dw", dw, K, N, K));
    if (db && reinterpret_cast<uintptr_t>(db) % 4 != 0) return fail(KATTN_ERR_MISALIGNED, "db is not 4-byte aligned");
    if (N == 0 || (K == 0 && !db)) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int launches = 0;
    const kattn::ProjStatus st = kattn::proj_backward_dw(ctx->num_sms, s, ctx->pool, ctx->d_status,
                                                         ctx->wait_ns.load(), dy, ld_dy, x, ld_x, dw, db, M, N, K,
                                                         accumulate, &launches);
    return proj_result(st, launches);
}

int kattn_layernorm_fwd(kattn_ctx* ctx, const float* x, long ld_x, const float* w, const float* b, float* y,
                        long ld_y, int M, int N, void* stream) {
    g_last_launches = 0;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (M < 0 || N < 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "negative size (M=%d N=%d)", M, N);
    if (N > KATTN_LN_MAX_N) return fail(KATTN_ERR_UNSUPPORTED, "N=%d exceeds KATTN_LN_MAX_N=%d", N, KATTN_LN_MAX_N);
    KATTN_TRY(check_matrix("x", x, ld_x, M, N));
    KATTN_TRY(check_matrix("y", y, ld_y, M, N));
    KATTN_TRY(check_matrix("w", w, N, 1, N));
    KATTN_TRY(check_matrix("b", b, N, 1, N));
    if (M == 0 || N == 0) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    int launches = 0;
    const kattn::ProjStatus st =
        kattn::ln_forward(static_cast<cudaStream_t>(stream), ctx->num_sms, x, ld_x, w, b, y, ld_y, M, N, &launches);
    return proj_result(st, launches);
}

int kattn_layernorm_bwd(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x, const float* w,
                        float* dx, long ld_dx, float* dw, float* db, int M, int N, int accumulate, void* stream) {
    g_last_launches = 0;
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (M < 0 || N < 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "negative size (M=%d N=%d)", M, N);
    if (N > KATTN_LN_MAX_N) return fail(KATTN_ERR_UNSUPPORTED, "N=%d exceeds KATTN_LN_MAX_N=%d", N, KATTN_LN_MAX_N);
    KATTN_TRY(check_matrix("dy", dy, ld_dy, M, N));
    KATTN_TRY(check_matrix("x", x, ld_x, M, N));
    KATTN_TRY(check_matrix("dx", dx, ld_dx, M, N));
    KATTN_TRY(check_matrix("w", w, N, 1, N));
    if (dw) KATTN_TRY(check_matrix("dw", dw, N, 1, N));
    if (db) KATTN_TRY(check_matrix("db", db, N, 1, N));
    if (N == 0 || (M == 0 && accumulate)) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    int launches = 0;
    const kattn::ProjStatus st = kattn::ln_backward(static_cast<cudaStream_t>(stream), ctx->pool, dy, ld_dy, x, ld_x, w, dx,
                                                    ld_dx, dw, db, M, N, accumulate, &launches);
    return proj_result(st, launches);
}

namespace {

// Checks shared by the Kerr-ODE entry points.
int kode_checks(const kattn_ctx* ctx, int M, int n_bands, int n_steps, const float* gamma_raw, const float* omega,
                const float* alpha_beta) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (M < 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "negative number of positions (M=%d)", M);
    if (n_bands <= 0) return fail(KATTN_ERR_INVALID_ARGUMENT, "n_bands must be positive (got %d)", n_bands);
    if (n_steps < 1) return fail(KATTN_ERR_INVALID_ARGUMENT, "n_steps must be positive (got %d)", n_steps);
    if (n_bands % 4 != 0)
        return fail(KATTN_ERR_UNSUPPORTED, "n_bands %d is not a multiple of 4 (n_embd a multiple of 8)", n_bands);
    if (n_bands > KATTN_KODE_MAX_BANDS)
        return fail(KATTN_ERR_UNSUPPORTED, "n_bands %d exceeds KATTN_KODE_MAX_BANDS=%d", n_bands,
                    KATTN_KODE_MAX_BANDS);
    if (!kattn::kode_supported(n_bands, n_steps))
        return fail(KATTN_ERR_UNSUPPORTED, "n_steps %d x n_bands %d: the backward's saved states exceed shared memory",
                    n_steps, n_bands);
    KATTN_TRY(check_vec("gamma_raw", gamma_raw, true));
    KATTN_TRY(check_vec("omega", omega, true));
    KATTN_TRY(check_vec("alpha_beta", alpha_beta, true));
    return KATTN_OK;
}

}  // namespace

int kattn_kerr_ode_fwd(kattn_ctx* ctx, const float* x, long ld_x, float* y, long ld_y, const float* gamma_raw,
                       const float* omega, const float* alpha_beta, int M, int n_bands, int n_steps, void* stream) {
    g_last_launches = 0;
    KATTN_TRY(kode_checks(ctx, M, n_bands, n_steps, gamma_raw, omega, alpha_beta));
    KATTN_TRY(check_matrix("x", x, ld_x, M, 2L * n_bands));
    KATTN_TRY(check_matrix("y", y, ld_y, M, 2L * n_bands));
    if (M == 0) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    int launches = 0;
    const kattn::ProjStatus st = kattn::kode_forward(static_cast<cudaStream_t>(stream), ctx->num_sms, x, ld_x, y, ld_y,
                                                     gamma_raw, omega, alpha_beta, M, n_bands, n_steps, &launches);
    return proj_result(st, launches);
}

int kattn_kerr_ode_bwd(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x,
                       const float* gamma_raw, const float* omega, const float* alpha_beta, float* dx, long ld_dx,
                       float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int M, int n_bands, int n_steps,
                       int accumulate, void* stream) {
    g_last_launches = 0;
    KATTN_TRY(kode_checks(ctx, M, n_bands, n_steps, gamma_raw, omega, alpha_beta));
    KATTN_TRY(check_matrix("dy", dy, ld_dy, M, 2L * n_bands));
    KATTN_TRY(check_matrix("x", x, ld_x, M, 2L * n_bands));
    KATTN_TRY(check_matrix("dx", dx, ld_dx, M, 2L * n_bands));
    KATTN_TRY(check_vec("d_gamma_raw", d_gamma_raw, true));
    KATTN_TRY(check_vec("d_omega", d_omega, true));
    KATTN_TRY(check_vec("d_alpha_beta", d_alpha_beta, true));
    if (M == 0 && accumulate) return ok_with_launches(0);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rows = 0;
    cudaError_t e = kattn::kode_backward_grid(ctx->num_sms, M, n_bands, n_steps, &rows);
    if (e != cudaSuccess) return cuda_fail(e, "Kerr-ODE backward occupancy");
    float* part = nullptr;
    if (rows > 0) {
        e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&part),
                                    sizeof(float) * static_cast<size_t>(rows) * kattn::kode_part_width(n_bands),
                                    ctx->pool, s);
        if (e != cudaSuccess) return cuda_fail(e, "workspace allocation (Kerr-ODE partial sums)");
    }
    int launches = 0;
    const kattn::ProjStatus st =
        kattn::kode_backward(s, ctx->num_sms, dy, ld_dy, x, ld_x, gamma_raw, omega, alpha_beta, dx, ld_dx, d_gamma_raw,
                             d_omega, d_alpha_beta, M, n_bands, n_steps, accumulate, part, rows, &launches);
    if (part) {
        const cudaError_t ef = cudaFreeAsync(part, s);
        if (st.ok() && ef != cudaSuccess) return cuda_fail(ef, "cudaFreeAsync(Kerr-ODE partial sums)");
    }
    return proj_result(st, launches);
}

namespace {

// Host arrays of the Kerr-ODE parameters -> the device block
// [gamma_raw | omega | alpha, beta] (the layout the kernels read).
cudaError_t upload_kode_params(float* d, const float* gamma_raw, const float* omega, float alpha, float beta, int nb,
                               cudaStream_t s) {
    const float ab[2] = {alpha, beta};  // pageable: staged before cudaMemcpyAsync returns
    cudaError_t e = cudaMemcpyAsync(d, gamma_raw, sizeof(float) * nb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d + nb, omega, sizeof(float) * nb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d + 2 * nb, ab, sizeof(ab), cudaMemcpyHostToDevice, s);
    return e;
}

int kode_host_checks(const kattn_ctx* ctx, int M, int n_bands, int n_steps, const float* gamma_raw,
                     const float* omega) {
    if (!ctx) return fail(KATTN_ERR_INVALID_ARGUMENT, "ctx is NULL");
    // Device-side alignment does not apply to host arrays: check shapes with
    // an aligned stand-in for the parameter pointers.
    KATTN_TRY(kode_checks(ctx, M, n_bands, n_steps, gamma_raw, omega, gamma_raw));
    return KATTN_OK;
}

int check_host_rows(const char* name, const void* p, long ld, long rows, long cols) {
    if (rows > 0 && !p) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    if (ld < cols) return fail(KATTN_ERR_INVALID_ARGUMENT, "%s row stride %ld < %ld columns", name, ld, cols);
    return KATTN_OK;
}

}  // namespace

int kattn_kerr_ode_fwd_host(kattn_ctx* ctx, const float* x, long ld_x, float* y, long ld_y, const float* gamma_raw,
                            const float* omega, float alpha, float beta, int M, int n_bands, int n_steps) {
    g_last_launches = 0;
    if (!gamma_raw || !omega) return fail(KATTN_ERR_INVALID_ARGUMENT, "gamma_raw / omega is NULL");
    KATTN_TRY(kode_host_checks(ctx, M, n_bands, n_steps, gamma_raw, omega));
    const int n = 2 * n_bands;
    KATTN_TRY(check_host_rows("x", x, ld_x, M, n));
    KATTN_TRY(check_host_rows("y", y, ld_y, M, n));
    if (M == 0) return ok_with_launches(0);
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    const size_t par_b = align256(sizeof(float) * (2 * static_cast<size_t>(n_bands) + 2));
    const size_t rows_b = align256(sizeof(float) * static_cast<size_t>(M) * n);
    KATTN_TRY(ensure_arena(ctx, par_b + 2 * rows_b));
    float* d_par = reinterpret_cast<float*>(ctx->arena);
    float* d_x = reinterpret_cast<float*>(ctx->arena + par_b);
    float* d_y = reinterpret_cast<float*>(ctx->arena + par_b + rows_b);
    const Chunks ch(M, 2 * sizeof(float) * static_cast<size_t>(M) * n);  // x up, y down
    KATTN_TRY(ensure_events(ctx, 2 * static_cast<size_t>(ch.n)));
    int launches = 0;
    const char* what = "host-to-device copy";
    cudaError_t e = upload_kode_params(d_par, gamma_raw, omega, alpha, beta, n_bands, ctx->h2d);
    for (int c = 0; c < ch.n && e == cudaSuccess; ++c) {
        const long r0 = ch.b0(c), rows = ch.count(c, M);
        what = "host-to-device copy";
        e = copy_rows(d_x + r0 * n, n, x + r0 * ld_x, ld_x, n, rows, cudaMemcpyHostToDevice, ctx->h2d);
        if (e == cudaSuccess) e = hand_off(ctx->h2d, ctx->stream, ctx->events[2 * c]);
        if (e != cudaSuccess) break;
        what = "Kerr-ODE forward launch";
        const kattn::ProjStatus st =
            kattn::kode_forward(ctx->stream, ctx->num_sms, d_x + r0 * n, n, d_y + r0 * n, n, d_par, d_par + n_bands,
                                d_par + 2 * n_bands, static_cast<int>(rows), n_bands, n_steps, &launches);
        e = st.cuda;
        if (e == cudaSuccess) e = hand_off(ctx->stream, ctx->d2h, ctx->events[2 * c + 1]);
        if (e != cudaSuccess) break;
        what = "device-to-host copy";
        e = copy_rows(y + r0 * ld_y, ld_y, d_y + r0 * n, n, n, rows, cudaMemcpyDeviceToHost, ctx->d2h);
    }
    const cudaError_t es = drain_host_streams(ctx);
    if (e != cudaSuccess) return cuda_fail(e, what);
    if (es != cudaSuccess) return cuda_fail(es, "cudaStreamSynchronize");
    return ok_with_launches(launches);
}

int kattn_kerr_ode_bwd_host(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x,
                            const float* gamma_raw, const float* omega, float alpha, float beta, float* dx, long ld_dx,
                            float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int M, int n_bands, int n_steps,
                            int accumulate) {
    g_last_launches = 0;
    if (!gamma_raw || !omega) return fail(KATTN_ERR_INVALID_ARGUMENT, "gamma_raw / omega is NULL");
    KATTN_TRY(kode_host_checks(ctx, M, n_bands, n_steps, gamma_raw, omega));
    const int n = 2 * n_bands;
    KATTN_TRY(check_host_rows("dy", dy, ld_dy, M, n));
    KATTN_TRY(check_host_rows("x", x, ld_x, M, n));
    KATTN_TRY(check_host_rows("dx", dx, ld_dx, M, n));
    if (!d_gamma_raw || !d_omega || !d_alpha_beta)
        return fail(KATTN_ERR_INVALID_ARGUMENT, "d_gamma_raw / d_omega / d_alpha_beta is NULL");
    if (M == 0) {
        // No positions: the sums are zero (nothing to add when accumulating).
        if (!accumulate) {
            std::memset(d_gamma_raw, 0, sizeof(float) * n_bands);
            std::memset(d_omega, 0, sizeof(float) * n_bands);
            d_alpha_beta[0] = d_alpha_beta[1] = 0.f;
        }
        return ok_with_launches(0);
    }
    std::lock_guard<std::mutex> lock(ctx->host_mu);
    DeviceScope scope(ctx->device);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "cudaSetDevice");
    const Chunks ch(M, 3 * sizeof(float) * static_cast<size_t>(M) * n);  // x, dy up; dx down
    // Partial-row slices of the chunks' backward launches, one after another.
    std::vector<int> part0(ch.n + 1, 0);
    for (int c = 0; c < ch.n; ++c) {
        int g = 0;
        const cudaError_t eg = kattn::kode_backward_grid(ctx->num_sms, ch.count(c, M), n_bands, n_steps, &g);
        if (eg != cudaSuccess) return cuda_fail(eg, "Kerr-ODE backward occupancy");
        part0[c + 1] = part0[c] + g;
    }
    const size_t width = static_cast<size_t>(kattn::kode_part_width(n_bands));
    const size_t par_b = align256(sizeof(float) * (2 * static_cast<size_t>(n_bands) + 2));
    const size_t rows_b = align256(sizeof(float) * static_cast<size_t>(M) * n);
    const size_t part_b = align256(sizeof(float) * width * part0[ch.n]);
    KATTN_TRY(ensure_arena(ctx, 2 * par_b + 2 * rows_b + part_b));
    float* d_par = reinterpret_cast<float*>(ctx->arena);
    float* d_grads = reinterpret_cast<float*>(ctx->arena + par_b);  // [d_gamma_raw | d_omega | d_alpha, d_beta]
    float* d_x = reinterpret_cast<float*>(ctx->arena + 2 * par_b);
    float* d_dy = reinterpret_cast<float*>(ctx->arena + 2 * par_b + rows_b);  // dx overwrites dy in place
    float* d_part = reinterpret_cast<float*>(ctx->arena + 2 * par_b + 2 * rows_b);
    KATTN_TRY(ensure_events(ctx, 2 * static_cast<size_t>(ch.n) + 2));
    int launches = 0;
    const char* what = "host-to-device copy";
    cudaError_t e = upload_kode_params(d_par, gamma_raw, omega, alpha, beta, n_bands, ctx->h2d);
    if (e == cudaSuccess && accumulate)
        e = upload_kode_params(d_grads, d_gamma_raw, d_omega, d_alpha_beta[0], d_alpha_beta[1], n_bands, ctx->h2d);
    for (int c = 0; c < ch.n && e == cudaSuccess; ++c) {
        const long r0 = ch.b0(c), rows = ch.count(c, M);
        what = "host-to-device copy";
        e = copy_rows(d_x + r0 * n, n, x + r0 * ld_x, ld_x, n, rows, cudaMemcpyHostToDevice, ctx->h2d);
        if (e == cudaSuccess)
            e = copy_rows(d_dy + r0 * n, n, dy + r0 * ld_dy, ld_dy, n, rows, cudaMemcpyHostToDevice, ctx->h2d);
        if (e == cudaSuccess) e = hand_off(ctx->h2d, ctx->stream, ctx->events[2 * c]);
        if (e != cudaSuccess) break;
        what = "Kerr-ODE backward launch";
        const kattn::ProjStatus st = kattn::kode_backward_rows(
            ctx->stream, d_dy + r0 * n, n, d_x + r0 * n, n, d_par, d_par + n_bands, d_par + 2 * n_bands,
            d_dy + r0 * n, n, static_cast<int>(rows), n_bands, n_steps, d_part + width * part0[c],
            part0[c + 1] - part0[c], &launches);
        e = st.cuda;
        if (e == cudaSuccess) e = hand_off(ctx->stream, ctx->d2h, ctx->events[2 * c + 1]);
        if (e != cudaSuccess) break;
        what = "device-to-host copy";
        e = copy_rows(dx + r0 * ld_dx, ld_dx, d_dy + r0 * n, n, n, rows, cudaMemcpyDeviceToHost, ctx->d2h);
    }
    if (e == cudaSuccess) {
        what = "Kerr-ODE parameter-gradient launch";
        const kattn::ProjStatus st =
            kattn::kode_backward_final(ctx->stream, d_part, part0[ch.n], n_bands, d_par, d_grads, d_grads + n_bands,
                                       d_grads + 2 * n_bands, accumulate, &launches);
        e = st.cuda;
        if (e == cudaSuccess) e = hand_off(ctx->stream, ctx->d2h, ctx->events[2 * ch.n]);
        what = "device-to-host copy";
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_gamma_raw, d_grads, sizeof(float) * n_bands, cudaMemcpyDeviceToHost, ctx->d2h);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_omega, d_grads + n_bands, sizeof(float) * n_bands, cudaMemcpyDeviceToHost,
                                ctx->d2h);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_alpha_beta, d_grads + 2 * n_bands, 2 * sizeof(float), cudaMemcpyDeviceToHost,
                                ctx->d2h);
    }
    const cudaError_t es = drain_host_streams(ctx);
    if (e != cudaSuccess) return cuda_fail(e, what);
    if (es != cudaSuccess) return cuda_fail(es, "cudaStreamSynchronize");
    return ok_with_launches(launches);
}

#pragma GCC visibility pop
}  // extern "C"
