/*
 * ORACLE — test infrastructure only (see kattn_oracle.h).  Plain-C
 * restatement of kerr-engine's CPU LayerNorm, as used for LN1 / LN2 around
 * the attention sublayer (src/pipeline.rs:236, :250, :678, :743):
 *
 *   forward : CpuBackend::layer_norm, src/backend.rs:258-267, per row:
 *             mean = (sum x) / n, var = (sum (x - mean)^2) / n,
 *             inv_std = 1 / sqrt(var + 1e-5), y = (x - mean) * inv_std * w + b
 *             (sums left to right)
 *   backward: layer_norm_backward, src/backward.rs:93-128, per row:
 *             x_hat = (x - mean) * inv_std, g = dy * w,
 *             dx = inv_std / n * (n g - sum g - x_hat * sum(g x_hat)),
 *             dw_row = dy * x_hat, db_row = dy;
 *             layer_norm_backward_batch, src/backend.rs:195-206, sums dw_row /
 *             db_row over the positions in order from zero, and the caller
 *             adds them into the gradients (src/pipeline.rs:747-750).
 *
 * No fused multiply-add (built -ffp-contract=off), single thread: rows are
 * cheap.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "kattn_oracle.h"

static void row_stats(const float* x, int n, float* mean, float* inv_std) {
    const float nf = (float)n;
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += x[i];
    const float m = s / nf;
    float v = 0.0f;
    for (int i = 0; i < n; ++i) v += (x[i] - m) * (x[i] - m);
    v /= nf;
    *mean = m;
    *inv_std = 1.0f / sqrtf(v + 1e-5f);
}

void kln_oracle_forward(int M, int N, const float* x, long ld_x, const float* w, const float* b, float* y,
                        long ld_y) {
    for (int m = 0; m < M; ++m) {
        const float* xr = x + (long)m * ld_x;
        float* yr = y + (long)m * ld_y;
        float mean, inv_std;
        row_stats(xr, N, &mean, &inv_std);
        for (int i = 0; i < N; ++i) yr[i] = (xr[i] - mean) * inv_std * w[i] + b[i];
    }
}

void kln_oracle_backward(int M, int N, const float* dy, long ld_dy, const float* x, long ld_x, const float* w,
                         float* dx, long ld_dx, float* dw, float* db, int accumulate) {
    float* tw = (float*)calloc((size_t)N, sizeof(float));
    float* tb = (float*)calloc((size_t)N, sizeof(float));
    float* xh = (float*)malloc((size_t)N * sizeof(float));
    float* g = (float*)malloc((size_t)N * sizeof(float));
    if (!tw || !tb || !xh || !g) {
        free(tw);
        free(tb);
        free(xh);
        free(g);
        return;
    }
    const float nf = (float)N;
    for (int m = 0; m < M; ++m) {
        const float* xr = x + (long)m * ld_x;
        const float* dr = dy + (long)m * ld_dy;
        float* out = dx + (long)m * ld_dx;
        float mean, inv_std;
        row_stats(xr, N, &mean, &inv_std);
        for (int i = 0; i < N; ++i) xh[i] = (xr[i] - mean) * inv_std;
        for (int i = 0; i < N; ++i) g[i] = dr[i] * w[i];
        float s1 = 0.0f, s2 = 0.0f;
        for (int i = 0; i < N; ++i) s1 += g[i];
        for (int i = 0; i < N; ++i) s2 += g[i] * xh[i];
        for (int i = 0; i < N; ++i) out[i] = inv_std / nf * (nf * g[i] - s1 - xh[i] * s2);
        for (int i = 0; i < N; ++i) {
            tw[i] += dr[i] * xh[i];
            tb[i] += dr[i];
        }
    }
    for (int i = 0; i < N; ++i) {
        if (dw) dw[i] = accumulate ? dw[i] + tw[i] : tw[i];
        if (db) db[i] = accumulate ? db[i] + tb[i] : tb[i];
    }
    free(tw);
    free(tb);
    free(xh);
    free(g);
}
