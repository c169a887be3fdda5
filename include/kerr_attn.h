/*
 * kerr_attn.h — C ABI of the B200 (sm_100a) causal self-attention path of
 * kerr-engine: forward (Q·Kᵀ scores, causal mask, softmax, P·V) and backward
 * (dQ, dK, dV recomputed from the saved log-sum-exp).
 *
 * What each entry point replaces in the reference (paths inside kerr-engine):
 *   kattn_fwd       the inline scalar head loop of attention_with_cache,
 *                   src/pipeline.rs:305-347 (same math as
 *                   src/model.rs:364-431).  It saves the row log-sum-exp
 *                   [B][H][T] instead of AttnCache.att_weights [H][T][T]
 *                   (src/pipeline.rs:157-164, :305, :337).
 *   kattn_bwd       ComputeBackend::attention_backward, src/backend.rs:223-231,
 *                   implemented today by CpuBackend (src/backend.rs:344-373 ->
 *                   src/backward.rs:464-514) and by GpuBackend
 *                   (src/gpu_dispatch.rs:921-1033 + shaders
 *                   attn_backward_scores.wgsl / attn_backward_dkv.wgsl).
 *   kattn_fwd_host, kattn_bwd_host
 *                   the same two operations at the reference's call boundary:
 *                   host buffers in, host buffers out, synchronous — the shape
 *                   of the trait call made from src/pipeline.rs:707-714.
 *
 * Conventions
 *   - All tensors are float32.  q, k, v (and dq, dk, dv) are [B][T][H][d]
 *     row-major with a row stride (elements) ld >= H*d, so they may be the
 *     q|k|v column blocks of one [B*T][3C] buffer (ld = 3C) exactly as
 *     c_attn produces it (src/pipeline.rs:289-303).  o and dout use ld_o.
 *     lse is [B][H][T], natural log: lse = log(sum_j exp(scale * q·k_j)).
 *   - Device pointers (kattn_fwd / kattn_bwd) are caller-owned, 16-byte
 *     aligned, with ld a multiple of 4 and d in {32, 64, 128}.  Outputs must
 *     not alias inputs.  The backward is faster when q, k, v, o, dout and dq
 *     are 32-byte aligned with row strides a multiple of 8: it then moves
 *     rows with 256-bit loads (same results either way).
 *   - No exception or exit crosses the ABI; every call returns a status.
 *     kattn_last_error() gives the detail of the last failure on the calling
 *     thread.
 *   - kattn_fwd / kattn_bwd only enqueue work on `stream` (a cudaStream_t,
 *     NULL = legacy default stream) and never synchronise the host.
 *     kattn_bwd takes a [B][H][T] float workspace on that stream from a
 *     stream-ordered memory pool the context owns and returns it there.
 *   - Workspace pool: each context creates its own pool (cudaMemPoolCreate)
 *     on its device.  Freed blocks stay cached in it until kattn_destroy
 *     (at most the largest workspace that calls in flight held at once);
 *     the device's default pool and its settings are not touched.
 *   - A context may be shared by threads: the device-pointer calls keep no
 *     per-call state in it; the host-buffer calls serialise on a lock inside
 *     it (as the reference's GPU backend serialises on its buffer pool,
 *     src/gpu_dispatch.rs:550).
 */
#ifndef KERR_ATTN_H
#define KERR_ATTN_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kattn_ctx kattn_ctx;

enum {
    KATTN_OK = 0,
    KATTN_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad stride */
    KATTN_ERR_UNSUPPORTED = 2,      /* head_dim outside {32, 64, 128} */
    KATTN_ERR_MISALIGNED = 3,       /* pointer not 16-byte aligned or ld % 4 != 0 */
    KATTN_ERR_DEVICE = 4,           /* no CUDA device, or not an sm_100 part */
    KATTN_ERR_CUDA = 5,             /* a CUDA runtime call failed */
    KATTN_ERR_OUT_OF_MEMORY = 6,    /* device or pinned allocation failed */
    KATTN_ERR_DEVICE_TIMEOUT = 7    /* a kernel gave up a bounded wait on the tensor core */
};

/* Kernel families (kattn_set_path).  AUTO uses the tensor-core kernels at
 * head_dim 64, and at head_dim 32 for problems of at least 16384 (batch,
 * head, position) rows, where they are faster; the FFMA kernels elsewhere. */
enum {
    KATTN_PATH_AUTO = 0,
    KATTN_PATH_FFMA = 1,   /* f32 CUDA-core kernels, every supported head_dim */
    KATTN_PATH_TENSOR = 2  /* tcgen05 bf16x3 kernels: head_dim 64 and 32; others refused */
};

/* Library version, major*10000 + minor*100 + patch. */
int kattn_version(void);

/* Human-readable name of a status code (static storage). */
const char* kattn_strerror(int status);

/* Detail of the last non-OK status returned on this thread (static per thread). */
const char* kattn_last_error(void);

/* Open a context on CUDA device `device` (the Rust GpuBackend's adapter index,
 * src/backend.rs:51-79).  Fails with KATTN_ERR_DEVICE when the device is absent
 * or is not compute capability 10.0. */
int kattn_create(int device, kattn_ctx** out);
int kattn_destroy(kattn_ctx* ctx);

/* Select the kernel family for later calls on this context (no counterpart
 * in the reference, whose backend choice is src/backend.rs:22-47).
 * KATTN_ERR_INVALID_ARGUMENT for an unknown value. */
int kattn_set_path(kattn_ctx* ctx, int path);

/* Wall-time limit, in nanoseconds, of every bounded wait inside the
 * tensor-core kernels launched on this context from now on (0 restores the
 * default of one second).  A kernel whose wait runs out sets the context's
 * device status word, frees its tensor memory and returns; kattn_check_device
 * then reports KATTN_ERR_DEVICE_TIMEOUT.  No counterpart in the reference,
 * whose GPU backend panics on device errors (src/gpu_ops_forward.rs:63). */
int kattn_set_wait_limit(kattn_ctx* ctx, unsigned long long ns);

/* Deterministic dQ (on != 0; off by default).  By default the backward adds
 * every key tile's dQ contribution into dq with floating-point reductions
 * whose order depends on scheduling, so dq can differ in the last bits from
 * run to run (dk, dv and the forward are always deterministic).  With the
 * mode on, each key tile stores its contribution into its own slice of a
 * [key tiles][B*T][H*d] float workspace from the context's pool (128 key
 * rows per tile on the tensor-core kernels, 64 on the FFMA kernels), and one
 * more kernel adds the slices in key-tile order: the same inputs then give
 * the same bits, at the cost of that workspace and a pass over it.  Replaces
 * the order the reference fixes by summing sequentially over keys
 * (src/backward.rs:508-512).  kattn_bwd_noalloc refuses to run in this mode
 * (KATTN_ERR_UNSUPPORTED): it allocates nothing. */
int kattn_set_deterministic(kattn_ctx* ctx, int on);

/* Diagnostic for the bounded waits: the next tensor-core forward launched on
 * this context issues no copy of its first key tile, so the waits on that
 * tile run out after the wait limit and the kernel unwinds as above (its
 * outputs are undefined).  Later calls run normally.  For tests of the
 * timeout path; no counterpart in the reference. */
int kattn_test_withhold_next_load(kattn_ctx* ctx);

/* Waits for the context's device to finish its work and reports whether any
 * kernel gave up a bounded wait since the last check (KATTN_ERR_DEVICE_TIMEOUT,
 * after which results of the affected calls are undefined); clears the flag. */
int kattn_check_device(kattn_ctx* ctx);

/* Forward.  o[b,t,h,:] = sum_{j<=t} softmax_j(scale * q[b,t,h,:]·k[b,j,h,:]) v[b,j,h,:]
 * (j < T instead of j <= t when causal == 0); lse[b,h,t] as above. */
int kattn_fwd(kattn_ctx* ctx,
              const float* q, const float* k, const float* v, long ld_qkv,
              float* o, long ld_o, float* lse,
              int B, int T, int H, int d, float scale, int causal, void* stream);

/* Backward from the forward's o and lse.  dout is the gradient of o (the
 * reference's d_pre_proj, same ld_o as o).  dq, dk, dv are fully overwritten. */
int kattn_bwd(kattn_ctx* ctx,
              const float* q, const float* k, const float* v, long ld_qkv,
              const float* o, const float* dout, long ld_o, const float* lse,
              float* dq, float* dk, float* dv, long ld_dqkv,
              int B, int T, int H, int d, float scale, int causal, void* stream);

/* Largest B*H*T that kattn_bwd_noalloc accepts (its fixed workspace: 4 MiB
 * of device memory per GPU that loads the library, held until exit). */
#define KATTN_NOALLOC_MAX_ROWS (1L << 20)

/* kattn_bwd for callers that cannot allocate device memory: a framework that
 * accounts for every byte through its own caching allocator, or a runtime
 * that reserves all device memory up front, cannot let a library take
 * memory from a stream-ordered pool as kattn_bwd does for its
 * [B][H][T] workspace.  This variant allocates nothing: the workspace is a
 * fixed array in the library's device image, whose address kattn_create
 * looks up once per context (so create the context before relying on this
 * call).  Same arguments, results and launches as kattn_bwd.
 *   - B*H*T above KATTN_NOALLOC_MAX_ROWS fails with KATTN_ERR_INVALID_ARGUMENT.
 *   - Every call on a device shares the one array and it keeps the last
 *     call's contents; each call writes every workspace element it reads
 *     before reading it, so nothing needs clearing between calls.
 *   - Calls whose kernels overlap on the GPU (other streams, other threads,
 *     other contexts on the same device) race on the array: serialise them.
 * No counterpart in the reference (its CPU and wgpu backends allocate per call). */
int kattn_bwd_noalloc(kattn_ctx* ctx,
                      const float* q, const float* k, const float* v, long ld_qkv,
                      const float* o, const float* dout, long ld_o, const float* lse,
                      float* dq, float* dk, float* dv, long ld_dqkv,
                      int B, int T, int H, int d, float scale, int causal, void* stream);

/* Host-buffer forms: same arguments as above, but every pointer is host
 * memory (pinned or pageable).  The call copies inputs to device buffers owned
 * by the context, runs the kernels, copies the outputs back and returns when
 * they are in host memory.  No alignment rule applies to host pointers. */
int kattn_fwd_host(kattn_ctx* ctx,
                   const float* q, const float* k, const float* v, long ld_qkv,
                   float* o, long ld_o, float* lse,
                   int B, int T, int H, int d, float scale, int causal);

int kattn_bwd_host(kattn_ctx* ctx,
                   const float* q, const float* k, const float* v, long ld_qkv,
                   const float* o, const float* dout, long ld_o, const float* lse,
                   float* dq, float* dk, float* dv, long ld_dqkv,
                   int B, int T, int H, int d, float scale, int causal);

/* Host-buffer calls, as above, keep their copies off the critical path: the
 * sequences are split into up to 8 chunks that move at least ~8 MB each, and one
 * chunk's results are copied back while the next chunk's kernels run and
 * the chunk after that is copied in (three streams of the context).  Pinned
 * host memory lets the copies run at link speed; pageable memory works too. */

/* ---- Saved forward state (the reference's AttnCache) ----------------------
 * The reference keeps q, k, v and the attention weights of each layer's
 * forward in an AttnCache (src/pipeline.rs:157-164) and hands them back to
 * attention_backward (src/pipeline.rs:707-714).  A kattn_saved is that cache
 * on the device: kattn_fwd_host_save runs kattn_fwd_host and keeps q/k/v, o
 * and lse resident; kattn_bwd_host_saved then needs only dout from the host,
 * so a training step moves q/k/v, o and lse across the link once instead of
 * twice.  A saved state belongs to the context it was created on; it is
 * reused (and its device memory regrown when a larger forward needs it) by
 * every later kattn_fwd_host_save into it. */
typedef struct kattn_saved kattn_saved;

int kattn_saved_create(kattn_ctx* ctx, kattn_saved** out);
int kattn_saved_destroy(kattn_saved* saved);

/* kattn_fwd_host, keeping the forward's device state in `saved`. */
int kattn_fwd_host_save(kattn_ctx* ctx, kattn_saved* saved,
                        const float* q, const float* k, const float* v, long ld_qkv,
                        float* o, long ld_o, float* lse,
                        int B, int T, int H, int d, float scale, int causal);

/* kattn_bwd_host for the forward held in `saved` (its shape, scale and
 * causal flag): dout in, dq / dk / dv out, all host buffers.
 * KATTN_ERR_INVALID_ARGUMENT when `saved` holds no completed forward. */
int kattn_bwd_host_saved(kattn_ctx* ctx, const kattn_saved* saved,
                         const float* dout, long ld_o,
                         float* dq, float* dk, float* dv, long ld_dqkv);

/* Number of kernel launches the last kattn_fwd / kattn_bwd call on this
 * thread enqueued (0 for an empty problem or an error); the same for every
 * other entry point below. */
int kattn_last_launch_count(void);

/* ---- Attention projections c_attn / c_proj (dense layers) -----------------
 * Replace CpuBackend::linear_batch (src/backend.rs:296-298, :508-520),
 * linear_backward_dx_batch (src/backend.rs:316-318 -> src/backward.rs:48-60)
 * and outer_product_accum (src/backend.rs:320-342) at src/pipeline.rs:289,
 * :353 and :695-737.  Rows are positions (M = B*T); weights keep the
 * reference's [out][in] layout (src/model.rs:184-185): w is [N][K]
 * contiguous.  Device pointers, 16-byte aligned; every row stride and K, N
 * a multiple of 4 floats; b and db need only 4-byte alignment.  Each product
 * is formed in bf16 hi/lo pairs (hi*hi + hi*lo + lo*hi, f32 accumulation;
 * ~1e-5 relative) by this library's tcgen05 GEMM, which splits the f32
 * operands on chip.  Split-K and column-sum workspace comes from the
 * context's stream-ordered pool; nothing synchronises the host. */

/* y[m][n] = b[n] + sum_k w[n][k] x[m][k];  b may be NULL (no bias). */
int kattn_linear_fwd(kattn_ctx* ctx, const float* x, long ld_x, const float* w, const float* b,
                     float* y, long ld_y, int M, int N, int K, void* stream);

/* dx[m][k] = sum_n dy[m][n] w[n][k]  (dx fully overwritten). */
int kattn_linear_bwd_dx(kattn_ctx* ctx, const float* dy, long ld_dy, const float* w,
                        float* dx, long ld_dx, int M, int N, int K, void* stream);

/* dw[n][k] (+)= sum_m dy[m][n] x[m][k] and db[n] (+)= sum_m dy[m][n]: added
 * to dw / db when accumulate != 0 (the += of src/pipeline.rs:701-704,
 * :733-736), written otherwise.  dw is [N][K] contiguous; db may be NULL. */
int kattn_linear_bwd_dw(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x,
                        float* dw, float* db, int M, int N, int K, int accumulate, void* stream);

/* ---- LayerNorm LN1 / LN2 (rows of n_embd) ----------------------------------
 * Replace layer_norm / layer_norm_batch (src/backend.rs:103, :140-142, CPU
 * :258-267) and layer_norm_backward / layer_norm_backward_batch
 * (src/backend.rs:184, :195-206, CPU src/backward.rs:93-128), called at
 * src/pipeline.rs:236, :250, :678, :743.  eps = 1e-5; the variance is the
 * mean of squared deviations, as in the reference.  Device pointers, rows
 * 16-byte aligned, N and every row stride a multiple of 4 floats,
 * N <= KATTN_LN_MAX_N.  Nothing synchronises the host. */
#define KATTN_LN_MAX_N 1536

/* y[m][:] = (x[m][:] - mean) / sqrt(var + eps) * w + b for m < M rows of N. */
int kattn_layernorm_fwd(kattn_ctx* ctx, const float* x, long ld_x, const float* w, const float* b,
                        float* y, long ld_y, int M, int N, void* stream);

/* dx from dy and x (statistics recomputed from x, as the reference does);
 * dw[n] (+)= sum_m dy[m][n] * xhat[m][n] and db[n] (+)= sum_m dy[m][n] when
 * accumulate != 0 (the += of src/pipeline.rs:747-750), written otherwise.
 * dw or db may be NULL.  The column sums are formed in a fixed order (no
 * atomics): the same inputs give the same bits. */
int kattn_layernorm_bwd(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x,
                        const float* w, float* dx, long ld_dx, float* dw, float* db,
                        int M, int N, int accumulate, void* stream);

/* ---- Kerr-ODE, the ODE core of the FFN (KerrMaestroAdd / KerrDualMaestro) --
 * Replace ComputeBackend::kerr_ode_batch (src/backend.rs:109-111; CPU
 * kerr_ode_cpu :387-417) and kerr_ode_backward_batch (src/backend.rs:147-176;
 * CPU kerr_ode_backward, src/backward.rs:382-458), called at
 * src/pipeline.rs:504, :626, :1003, :1022, :1067, :1107.  A row is one
 * position: n_embd = 2 n_bands floats, bands interleaved (r_0, s_0, r_1, s_1,
 * ...) as the reference stores them.  KerrWeights (src/model.rs:199-205) is
 * passed as device arrays: gamma_raw and omega of n_bands floats, alpha_beta =
 * {alpha, beta}; rk4_n_steps is n_steps (dt = 1/n_steps).  Rows 16-byte
 * aligned, row strides multiples of 4 floats; n_bands a multiple of 4, at most
 * KATTN_KODE_MAX_BANDS.  Outputs may alias their inputs (y = x, dx = dy).
 * f32 arithmetic (fused multiply-adds; ~1e-7 relative to the reference's
 * loops).  Nothing synchronises the host. */
#define KATTN_KODE_MAX_BANDS 1024

/* y[m] = Kerr-ODE(x[m]) for m < M rows. */
int kattn_kerr_ode_fwd(kattn_ctx* ctx, const float* x, long ld_x, float* y, long ld_y,
                       const float* gamma_raw, const float* omega, const float* alpha_beta,
                       int M, int n_bands, int n_steps, void* stream);

/* dx[m] = dL/dx[m] for upstream dy[m]; d_gamma_raw / d_omega (n_bands floats)
 * and d_alpha_beta (2 floats) receive the parameter gradients summed over the
 * M rows: added to when accumulate != 0 (the += of src/pipeline.rs:627-632),
 * written otherwise.  The sums run in a fixed order (no atomics): the same
 * inputs give the same bits.  Workspace (one row of 2 n_bands + 4 floats per
 * CTA) comes from the context's stream-ordered pool. */
int kattn_kerr_ode_bwd(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x,
                       const float* gamma_raw, const float* omega, const float* alpha_beta,
                       float* dx, long ld_dx, float* d_gamma_raw, float* d_omega, float* d_alpha_beta,
                       int M, int n_bands, int n_steps, int accumulate, void* stream);

/* The same two operations on HOST buffers, the trait's own boundary
 * (kerr_ode_batch / kerr_ode_backward_batch take host slices and
 * &KerrWeights): x, y, dy, dx, gamma_raw, omega and the gradient outputs are
 * host memory and alpha, beta are values.  Synchronous: the results are in
 * the host arrays on return.  The positions move in up to 8 chunks on three
 * streams (copies up, kernels, copies down), so with pinned host memory one
 * chunk's copies overlap another's kernels.  Staging is a per-context device
 * buffer that grows to the largest call; calls on one context are
 * serialised.  The backward's accumulate has the meaning above (the host
 * d_gamma_raw / d_omega / d_alpha_beta are added to). */
int kattn_kerr_ode_fwd_host(kattn_ctx* ctx, const float* x, long ld_x, float* y, long ld_y,
                            const float* gamma_raw, const float* omega, float alpha, float beta,
                            int M, int n_bands, int n_steps);
int kattn_kerr_ode_bwd_host(kattn_ctx* ctx, const float* dy, long ld_dy, const float* x, long ld_x,
                            const float* gamma_raw, const float* omega, float alpha, float beta,
                            float* dx, long ld_dx, float* d_gamma_raw, float* d_omega, float* d_alpha_beta,
                            int M, int n_bands, int n_steps, int accumulate);

/* ---- Device-resident block pipeline ----------------------------------------
 * One transformer block of the reference's batched pipeline, as far as this
 * library covers it, run on the device with every intermediate kept there
 * between the forward and the backward (forward_backward_batch,
 * src/pipeline.rs:764-1222; per block :236-360 forward, :670-750 backward):
 *
 *   x1 = LN1(h);  qkv = c_attn(x1);  o = causal_attention(qkv);
 *   h1 = h + c_proj(o);
 *   h_out = h1 + KerrODE(LN2(h1))     (with the FFN; h_out = h1 without)
 *
 * The FFN's maestro squeeze / process and out_proj layers are dense layers
 * outside this library: the FFN runs as its ODE core (KerrWeights), and a
 * block created with rk4_n_steps = 0 is the attention sublayer alone.  Rows
 * are positions (M = B*T), contiguous [M][C] arrays; head_dim = C / H;
 * scale 1/sqrt(head_dim); causal.  Parameters are device pointers in the
 * reference's layouts (src/model.rs:184-205): w_attn [3C][C], w_proj [C][C],
 * gamma_raw / omega of C/2 bands, alpha_beta = {alpha, beta}.  Each call
 * enqueues its kernels on `stream` and returns; nothing synchronises the
 * host. */
typedef struct kattn_block kattn_block;

typedef struct {
    const float* ln1_w;
    const float* ln1_b;
    const float* w_attn;
    const float* b_attn;
    const float* w_proj;
    const float* b_proj;
    const float* ln2_w;      /* FFN only (ignored when rk4_n_steps = 0) */
    const float* ln2_b;
    const float* gamma_raw;
    const float* omega;
    const float* alpha_beta;
} kattn_block_params;

/* Gradient outputs, one per parameter above (FFN entries ignored without
 * the FFN); written, or added to when accumulate != 0. */
typedef struct {
    float* ln1_w;
    float* ln1_b;
    float* w_attn;
    float* b_attn;
    float* w_proj;
    float* b_proj;
    float* ln2_w;
    float* ln2_b;
    float* gamma_raw;
    float* omega;
    float* alpha_beta;
} kattn_block_grads;

/* Allocates the block's device activations for B x T positions of width C
 * (x1, qkv, o, lse, h1, x2 and the backward's temporaries: 13 M*C floats
 * with the FFN, 10 without).  C a multiple of 8, C / H in {32, 64, 128}, C <=
 * KATTN_LN_MAX_N; rk4_n_steps 0 (no FFN) or the Kerr-ODE's steps. */
int kattn_block_create(kattn_ctx* ctx, int B, int T, int C, int H, int rk4_n_steps, kattn_block** out);
int kattn_block_destroy(kattn_block* blk);

/* Forward of h [M][C] into h_out [M][C] (h_out must not alias h).  h and
 * the parameters must stay unchanged until the matching kattn_block_bwd,
 * which reads them (the reference's block cache holds the same). */
int kattn_block_fwd(kattn_ctx* ctx, kattn_block* blk, const kattn_block_params* params, const float* h,
                    float* h_out, void* stream);

/* Backward of the last forward: dh [M][C] = d(loss)/dh from dh_out =
 * d(loss)/dh_out (dh may alias dh_out), and the parameter gradients. */
int kattn_block_bwd(kattn_ctx* ctx, kattn_block* blk, const float* dh_out, float* dh,
                    const kattn_block_grads* grads, int accumulate, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KERR_ATTN_H */
