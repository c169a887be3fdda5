/*
 * ORACLE — test infrastructure only (see kattn_oracle.h).  Plain-C
 * restatement of kerr-engine's CPU linear layers, as used by the attention
 * projections c_attn and c_proj (src/pipeline.rs:289, :353, :695-737):
 *
 *   forward : CpuBackend::linear / linear_batch_cpu, src/backend.rs:240-247,
 *             :508-520:  y[i] = b[i] + sum_j w[i][j] * x[j]  (the dot product
 *             summed left to right from -0.0, as Rust's f32 Sum does; then
 *             the bias is added)
 *   dx      : linear_backward_dx_only, src/backward.rs:48-60:
 *             dx[j] = sum_i dy[i] * w[i][j]  (sum from 0.0, i ascending)
 *   dw, db  : CpuBackend::outer_product_accum, src/backend.rs:320-342:
 *             for pos, for i: dw[i][j] += dy[pos][i] * x[pos][j]; db[i] += dy[pos][i]
 *
 * Rows are positions.  Weights are [out][in] row-major (w[i] is out-row i,
 * src/model.rs:184-185).  No fused multiply-add (built -ffp-contract=off).
 * The reference runs these per sequence on one host thread each; the
 * batched drivers below split the independent outputs over host threads
 * instead, which leaves every output's own summation order unchanged.
 */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "kattn_oracle.h"

typedef struct {
    int kind;  /* 0 fwd, 1 dx, 2 dw */
    int lo, hi;  /* range of the split dimension */
    const float *x, *w, *b, *dy;
    float *y, *dx, *dw, *db;
    long ld_x, ld_y, ld_dy, ld_dx;
    int M, N, K;
} lin_job_t;

/* y[m][n] for m in [lo, hi): one position per row, out features in order. */
static void fwd_rows(const lin_job_t* j) {
    for (int m = j->lo; m < j->hi; ++m) {
        const float* x = j->x + (long)m * j->ld_x;
        float* y = j->y + (long)m * j->ld_y;
        for (int n = 0; n < j->N; ++n) {
            const float* w = j->w + (long)n * j->K;
            float s = -0.0f;
            for (int k = 0; k < j->K; ++k) s += w[k] * x[k];
            y[n] = (j->b ? j->b[n] : 0.0f) + s;
        }
    }
}

/* dx[m][k] for m in [lo, hi). */
static void dx_rows(const lin_job_t* j) {
    for (int m = j->lo; m < j->hi; ++m) {
        const float* dy = j->dy + (long)m * j->ld_dy;
        float* dx = j->dx + (long)m * j->ld_dx;
        for (int k = 0; k < j->K; ++k) {
            float s = 0.0f;
            for (int n = 0; n < j->N; ++n) s += dy[n] * j->w[(long)n * j->K + k];
            dx[k] = s;
        }
    }
}

/* dw[n][.] and db[n] for n in [lo, hi): positions in order, as the
 * reference's outer loop over pos. */
static void dw_rows(const lin_job_t* j) {
    for (int n = j->lo; n < j->hi; ++n) {
        float* dw = j->dw + (long)n * j->K;
        float db = 0.0f;
        for (int m = 0; m < j->M; ++m) {
            const float d = j->dy[(long)m * j->ld_dy + n];
            const float* x = j->x + (long)m * j->ld_x;
            for (int k = 0; k < j->K; ++k) dw[k] += d * x[k];
            db += d;
        }
        if (j->db) j->db[n] += db;
    }
}

static void* lin_run(void* p) {
    const lin_job_t* j = (const lin_job_t*)p;
    if (j->kind == 0) fwd_rows(j);
    else if (j->kind == 1) dx_rows(j);
    else dw_rows(j);
    return NULL;
}

static void lin_batch(lin_job_t proto, int total, int nthreads) {
    if (nthreads <= 0) nthreads = kattn_oracle_default_threads(total);
    if (nthreads > total) nthreads = total;
    if (nthreads < 1) nthreads = 1;
    pthread_t th[256];
    lin_job_t jobs[256];
    if (nthreads > 256) nthreads = 256;
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = proto;
        jobs[t].lo = (int)((long)total * t / nthreads);
        jobs[t].hi = (int)((long)total * (t + 1) / nthreads);
        pthread_create(&th[t], NULL, lin_run, &jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
}

void kproj_oracle_forward(int M, int N, int K, const float* x, long ld_x, const float* w, const float* b,
                          float* y, long ld_y, int nthreads) {
    lin_job_t j;
    memset(&j, 0, sizeof j);
    j.kind = 0;
    j.x = x; j.ld_x = ld_x; j.w = w; j.b = b; j.y = y; j.ld_y = ld_y;
    j.M = M; j.N = N; j.K = K;
    lin_batch(j, M, nthreads);
}

void kproj_oracle_backward_dx(int M, int N, int K, const float* dy, long ld_dy, const float* w, float* dx,
                              long ld_dx, int nthreads) {
    lin_job_t j;
    memset(&j, 0, sizeof j);
    j.kind = 1;
    j.dy = dy; j.ld_dy = ld_dy; j.w = w; j.dx = dx; j.ld_dx = ld_dx;
    j.M = M; j.N = N; j.K = K;
    lin_batch(j, M, nthreads);
}

void kproj_oracle_backward_dw(int M, int N, int K, const float* dy, long ld_dy, const float* x, long ld_x,
                              float* dw, float* db, int nthreads) {
    lin_job_t j;
    memset(&j, 0, sizeof j);
    j.kind = 2;
    j.dy = dy; j.ld_dy = ld_dy; j.x = x; j.ld_x = ld_x; j.dw = dw; j.db = db;
    j.M = M; j.N = N; j.K = K;
    lin_batch(j, N, nthreads);
}
