/*
 * ORACLE — test infrastructure only.  Nothing in the product library links,
 * loads or calls this code; only tests/, the smoke check and bench.py's CPU
 * baseline leg use it, and only as the checker / the timed CPU reference arm.
 *
 * A plain-C restatement of kerr-engine's CPU causal self-attention:
 *   forward : src/pipeline.rs:305-347 (attention_with_cache head loop), which is
 *             the same arithmetic as src/model.rs:364-431 (causal_self_attention)
 *   backward: src/backend.rs:344-373 (CpuBackend::attention_backward) driving
 *             src/backward.rs:464-514 (attention_backward_single)
 *   batching: src/train.rs:194-198, :241-255 (one host thread per sequence,
 *             parallelism min(cores, batch))
 *
 * PARITY UNPINNED: the reference ships no golden vectors or known-answer tests
 * for attention (its grad_test covers only the Kerr ODE and its gpu-backend-test
 * has no attention case), and the reference is Rust, which cannot be compiled in
 * this environment.  The restatement keeps the reference's loop order, f32
 * accumulation and libm expf so that it is the same arithmetic; it is checked
 * against an independent float64 autograd computation and against algebraic
 * known answers instead.
 *
 * Layout (as in the reference, src/pipeline.rs:296-302, :313): one sequence is
 * [T][ld] rows of floats, head h occupying columns h*hd .. (h+1)*hd.  Batched
 * calls use [B][T][ld] (batch stride T*ld).  att is the reference's
 * AttnCache.att_weights, [H][T][T] per sequence (src/pipeline.rs:305),
 * entries above the diagonal left at -inf exactly as the reference leaves them.
 */
#ifndef KATTN_ORACLE_H
#define KATTN_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* One sequence.  out: [T][ld_o].  att: [H][T][T] or NULL.  lse: [H][T] or NULL
 * (lse is an addition the reference does not compute: max + log(exp_sum) of
 * each softmax row, in float64, used only to feed device backward checks). */
void kattn_oracle_forward_seq(int T, int C, int H,
                              const float* q, const float* k, const float* v, long ld_qkv,
                              float* out, long ld_o, float* att, float* lse);

/* One sequence.  d_out: [T][ld_o] (the reference's d_pre_proj), att: [H][T][T]
 * post-softmax weights.  dq/dk/dv: [T][ld_d], fully overwritten. */
void kattn_oracle_backward_seq(int T, int C, int H,
                               const float* d_out, long ld_o,
                               const float* q, const float* k, const float* v, long ld_qkv,
                               const float* att,
                               float* dq, float* dk, float* dv, long ld_d);

/* Batched drivers over B independent sequences, nthreads host threads
 * (nthreads <= 0: min(online cores, B)).  att: [B][H][T][T], lse: [B][H][T]. */
void kattn_oracle_forward_batch(int B, int T, int C, int H,
                                const float* q, const float* k, const float* v, long ld_qkv,
                                float* out, long ld_o, float* att, float* lse, int nthreads);

void kattn_oracle_backward_batch(int B, int T, int C, int H,
                                 const float* d_out, long ld_o,
                                 const float* q, const float* k, const float* v, long ld_qkv,
                                 const float* att,
                                 float* dq, float* dk, float* dv, long ld_d, int nthreads);

/* Threads the batched drivers use for nthreads <= 0. */
int kattn_oracle_default_threads(int B);

/* LayerNorm LN1 / LN2 (kln_oracle.c): rows of N floats, eps 1e-5.  The
 * backward writes dx and sets (accumulate == 0) or adds to dw / db (either
 * may be NULL) the column sums over the M rows. */
void kln_oracle_forward(int M, int N, const float* x, long ld_x, const float* w, const float* b, float* y,
                        long ld_y);
void kln_oracle_backward(int M, int N, const float* dy, long ld_dy, const float* x, long ld_x, const float* w,
                         float* dx, long ld_dx, float* dw, float* db, int accumulate);

/* Linear layers of the attention projections (kproj_oracle.c): rows are
 * positions, weights [N out][K in] row-major.
 *   forward    : y[m][n] = b[n] + sum_k w[n][k] x[m][k]   (b may be NULL)
 *   backward_dx: dx[m][k] = sum_n dy[m][n] w[n][k]
 *   backward_dw: dw[n][k] += sum_m dy[m][n] x[m][k];  db[n] += sum_m dy[m][n]
 *                (db may be NULL; pass zeroed arrays for fresh gradients) */
void kproj_oracle_forward(int M, int N, int K, const float* x, long ld_x, const float* w, const float* b,
                          float* y, long ld_y, int nthreads);
void kproj_oracle_backward_dx(int M, int N, int K, const float* dy, long ld_dy, const float* w, float* dx,
                              long ld_dx, int nthreads);
void kproj_oracle_backward_dw(int M, int N, int K, const float* dy, long ld_dy, const float* x, long ld_x,
                              float* dw, float* db, int nthreads);

/* Kerr-ODE (kode_oracle.c): M positions of 2*nb interleaved floats
 * (r_0, s_0, r_1, s_1, ...), gamma_raw / omega of nb floats, n_steps RK4
 * steps of dt = 1/n_steps.  The backward writes dx and SETS d_gamma_raw /
 * d_omega (nb floats) and d_alpha_beta[0..1] to the sums over the M
 * positions.  nthreads <= 0: all online cores (at most M). */
void kode_oracle_forward(int M, int nb, int n_steps, const float* x, long ld_x, const float* gamma_raw,
                         const float* omega, float alpha, float beta, float* y, long ld_y, int nthreads);
void kode_oracle_backward(int M, int nb, int n_steps, const float* dy, long ld_dy, const float* x, long ld_x,
                          const float* gamma_raw, const float* omega, float alpha, float beta, float* dx, long ld_dx,
                          float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
