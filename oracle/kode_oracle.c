/*
 * ORACLE — test infrastructure only (see kattn_oracle.h).  Plain-C
 * restatement of kerr-engine's CPU Kerr-ODE, the ODE core of the FFN
 * (KerrDualMaestro / KerrMaestroAdd), called per block at
 * src/pipeline.rs:504, :626, :1003, :1022, :1067, :1107:
 *
 *   forward : CpuBackend::kerr_ode -> kerr_ode_cpu (src/backend.rs:269-272,
 *             :387-417): deinterleave x into (r, s) bands, gamma =
 *             softplus(gamma_raw) (src/backend.rs:379-385), rk4_n_steps RK4
 *             steps of dt = 1/rk4_n_steps (rk4_step, src/model.rs:808-843,
 *             over kerr_derivative, src/model.rs:778-806), reinterleave.
 *             kerr_ode_batch (src/backend.rs:109-111) maps it over positions.
 *   backward: the trait's default kerr_ode_backward_batch (src/backend.rs:
 *             147-176): per position kerr_ode_backward (src/backward.rs:
 *             382-458), which recomputes the n_steps states, then runs
 *             rk4_step_backward (:295-379; kerr_derivative_with_cache_pub
 *             :184-214, kerr_derivative_backward_pub :222-286) from the last
 *             step to the first and chains d_gamma through softplus_backward
 *             (:150-153); the parameter gradients are summed over positions
 *             in order, from zero.
 *
 * Arithmetic as the reference writes it: f32 throughout, each expression
 * evaluated left to right, no fused multiply-add (built -ffp-contract=off,
 * as Rust never contracts), Rust's float Sum folding from -0.0, libm expf /
 * logf for exp / ln.
 *
 * Batched drivers may split positions over host threads.  The forward is
 * unchanged by that (positions are independent).  The backward's parameter
 * sums then run per thread over its contiguous range of positions and the
 * per-thread sums are added in thread order; with one thread they are the
 * reference's order exactly.
 */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "kattn_oracle.h"

/* src/backend.rs:379-385 (and src/model.rs:66-72). */
static float softplus(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

/* src/backward.rs:150-153. */
static float softplus_backward(float d_y, float x) {
    const float sig = x > 20.0f ? 1.0f : expf(x) / (1.0f + expf(x));
    return d_y * sig;
}

/* kerr_derivative (src/model.rs:778-806); with cache != NULL also
 * kerr_derivative_with_cache_pub (src/backward.rs:184-214): the cache keeps
 * mag_sq, ns and phi (r and s are the caller's arrays). */
typedef struct {
    float* mag_sq;
    float* ns;
    float* phi;
} deriv_cache;

static void kerr_derivative(int n, const float* r, const float* s, const float* gamma, const float* omega,
                            float alpha, float beta, float* dr, float* ds, deriv_cache* cache, float* scratch) {
    float* mag_sq = cache ? cache->mag_sq : scratch;
    float* ns = cache ? cache->ns : scratch + n;
    for (int k = 0; k < n; ++k) mag_sq[k] = r[k] * r[k] + s[k] * s[k];
    for (int k = 0; k < n; ++k) {
        float a = 0.0f;
        if (k >= 2) a += mag_sq[k - 2];
        if (k >= 1) a += mag_sq[k - 1];
        if (k + 1 < n) a += mag_sq[k + 1];
        if (k + 2 < n) a += mag_sq[k + 2];
        ns[k] = a;
    }
    for (int k = 0; k < n; ++k) {
        const float phi = omega[k] + alpha * mag_sq[k] + beta * ns[k];
        if (cache) cache->phi[k] = phi;
        dr[k] = -gamma[k] * r[k] - phi * s[k];
        ds[k] = -gamma[k] * s[k] + phi * r[k];
    }
}

/* rk4_step (src/model.rs:808-843): (r, s) -> (r_new, s_new).  w: 12 n floats. */
static void rk4_step(int n, const float* r, const float* s, float dt, const float* gamma, const float* omega,
                     float alpha, float beta, float* r_new, float* s_new, float* w) {
    float *dr1 = w, *ds1 = w + n, *dr2 = w + 2 * n, *ds2 = w + 3 * n, *dr3 = w + 4 * n, *ds3 = w + 5 * n;
    float *dr4 = w + 6 * n, *ds4 = w + 7 * n, *ri = w + 8 * n, *si = w + 9 * n;
    float* scratch = w + 10 * n;
    kerr_derivative(n, r, s, gamma, omega, alpha, beta, dr1, ds1, NULL, scratch);
    for (int k = 0; k < n; ++k) {
        ri[k] = r[k] + 0.5f * dt * dr1[k];
        si[k] = s[k] + 0.5f * dt * ds1[k];
    }
    kerr_derivative(n, ri, si, gamma, omega, alpha, beta, dr2, ds2, NULL, scratch);
    for (int k = 0; k < n; ++k) {
        ri[k] = r[k] + 0.5f * dt * dr2[k];
        si[k] = s[k] + 0.5f * dt * ds2[k];
    }
    kerr_derivative(n, ri, si, gamma, omega, alpha, beta, dr3, ds3, NULL, scratch);
    for (int k = 0; k < n; ++k) {
        ri[k] = r[k] + dt * dr3[k];
        si[k] = s[k] + dt * ds3[k];
    }
    kerr_derivative(n, ri, si, gamma, omega, alpha, beta, dr4, ds4, NULL, scratch);
    const float dt6 = dt / 6.0f;
    for (int k = 0; k < n; ++k) {
        r_new[k] = r[k] + dt6 * (dr1[k] + 2.0f * dr2[k] + 2.0f * dr3[k] + dr4[k]);
        s_new[k] = s[k] + dt6 * (ds1[k] + 2.0f * ds2[k] + 2.0f * ds3[k] + ds4[k]);
    }
}

/* kerr_ode_cpu (src/backend.rs:387-417) on one position. */
static void ode_forward_pos(int nb, int n_steps, const float* x, const float* gamma, const float* omega, float alpha,
                            float beta, float* y, float* w) {
    float *r = w, *s = w + nb, *rn = w + 2 * nb, *sn = w + 3 * nb, *rk = w + 4 * nb;
    const float dt = 1.0f / (float)n_steps;
    for (int k = 0; k < nb; ++k) {
        r[k] = x[2 * k];
        s[k] = x[2 * k + 1];
    }
    for (int st = 0; st < n_steps; ++st) {
        rk4_step(nb, r, s, dt, gamma, omega, alpha, beta, rn, sn, rk);
        memcpy(r, rn, sizeof(float) * nb);
        memcpy(s, sn, sizeof(float) * nb);
    }
    for (int k = 0; k < nb; ++k) {
        y[2 * k] = r[k];
        y[2 * k + 1] = s[k];
    }
}

/* kerr_derivative_backward_pub (src/backward.rs:222-286).  Adds d_gamma and
 * d_omega into dg_acc / dom_acc in the caller's order (the caller does
 * `acc[k] += dg[k]`), returns d_alpha / d_beta, writes d_r / d_s. */
static void deriv_backward(int n, const float* d_dr, const float* d_ds, const float* r, const float* s,
                           const deriv_cache* c, const float* gamma, float alpha, float beta, float* d_r, float* d_s,
                           float* dg_acc, float* dom_acc, float* d_alpha, float* d_beta, float* w) {
    float *d_phi = w, *d_mag = w + n, *d_ns = w + 2 * n;
    for (int k = 0; k < n; ++k) d_phi[k] = d_dr[k] * (-s[k]) + d_ds[k] * r[k];
    float da = -0.0f, db = -0.0f;
    for (int k = 0; k < n; ++k) da += d_phi[k] * c->mag_sq[k];
    for (int k = 0; k < n; ++k) db += d_phi[k] * c->ns[k];
    for (int k = 0; k < n; ++k) d_mag[k] = d_phi[k] * alpha;
    for (int k = 0; k < n; ++k) d_ns[k] = d_phi[k] * beta;
    for (int k = 0; k < n; ++k) {
        if (k >= 2) d_mag[k - 2] += d_ns[k];
        if (k >= 1) d_mag[k - 1] += d_ns[k];
        if (k + 1 < n) d_mag[k + 1] += d_ns[k];
        if (k + 2 < n) d_mag[k + 2] += d_ns[k];
    }
    for (int k = 0; k < n; ++k) {
        d_r[k] = d_dr[k] * (-gamma[k]) + d_ds[k] * c->phi[k] + d_mag[k] * 2.0f * r[k];
        d_s[k] = d_dr[k] * (-c->phi[k]) + d_ds[k] * (-gamma[k]) + d_mag[k] * 2.0f * s[k];
    }
    for (int k = 0; k < n; ++k) {
        dg_acc[k] += d_dr[k] * (-r[k]) + d_ds[k] * (-s[k]);
        dom_acc[k] += d_phi[k];
    }
    *d_alpha += da;
    *d_beta += db;
}

/* Working floats one position's backward needs for nb bands and n_steps. */
static size_t bwd_work_floats(int nb, int n_steps) { return (size_t)nb * (2 * (size_t)(n_steps + 1) + 64); }

/* kerr_ode_backward (src/backward.rs:382-458) on one position, with
 * rk4_step_backward (:295-379) inlined per step.  Writes d_input into dx and
 * adds the position's d_gamma_raw / d_omega into dgr / dom and its d_alpha /
 * d_beta into *da / *db (the per-position sums of src/backend.rs:163-172). */
static void ode_backward_pos(int nb, int n_steps, const float* dy, const float* x, const float* gamma_raw,
                             const float* gamma, const float* omega, float alpha, float beta, float* dx, float* dgr,
                             float* dom, float* da, float* db, float* w) {
    const int n = nb;
    const float dt = 1.0f / (float)n_steps;
    const float dt6 = dt / 6.0f;
    float* states = w;                       /* [n_steps + 1][2][n] */
    float* q = w + 2 * (size_t)(n_steps + 1) * n;
    float *d_r = q, *d_s = q + n, *g_acc = q + 2 * n, *om_acc = q + 3 * n;
    float *r2 = q + 4 * n, *s2 = q + 5 * n, *r3 = q + 6 * n, *s3 = q + 7 * n, *r4 = q + 8 * n, *s4 = q + 9 * n;
    float *dr1 = q + 10 * n, *ds1 = q + 11 * n, *dr2 = q + 12 * n, *ds2 = q + 13 * n, *dr3 = q + 14 * n,
          *ds3 = q + 15 * n, *dr4 = q + 16 * n, *ds4 = q + 17 * n;
    float *dn_r = q + 18 * n, *dn_s = q + 19 * n; /* d_r_new, d_s_new of the step */
    float *ddr = q + 20 * n, *dds = q + 21 * n, *dri = q + 22 * n, *dsi = q + 23 * n;
    deriv_cache c[4];
    for (int i = 0; i < 4; ++i) {
        c[i].mag_sq = q + (24 + 3 * i) * n;
        c[i].ns = q + (25 + 3 * i) * n;
        c[i].phi = q + (26 + 3 * i) * n;
    }
    float* bw = q + 36 * n;   /* 3 n for deriv_backward */
    float* rkw = q + 39 * n;  /* 12 n for rk4_step */
    float* scratch = q + 51 * n;

    for (int k = 0; k < n; ++k) {
        d_r[k] = dy[2 * k];
        d_s[k] = dy[2 * k + 1];
        states[k] = x[2 * k];
        states[n + k] = x[2 * k + 1];
    }
    for (int st = 0; st < n_steps; ++st) {
        const float* r = states + (size_t)st * 2 * n;
        float* nxt = states + (size_t)(st + 1) * 2 * n;
        rk4_step(n, r, r + n, dt, gamma, omega, alpha, beta, nxt, nxt + n, rkw);
    }
    for (int k = 0; k < n; ++k) g_acc[k] = om_acc[k] = 0.0f;
    float a_acc = 0.0f, b_acc = 0.0f;

    for (int st = n_steps - 1; st >= 0; --st) {
        const float* r = states + (size_t)st * 2 * n;
        const float* s = r + n;
        /* rk4_step_backward: recompute the four evaluations with caches. */
        kerr_derivative(n, r, s, gamma, omega, alpha, beta, dr1, ds1, &c[0], scratch);
        for (int k = 0; k < n; ++k) {
            r2[k] = r[k] + 0.5f * dt * dr1[k];
            s2[k] = s[k] + 0.5f * dt * ds1[k];
        }
        kerr_derivative(n, r2, s2, gamma, omega, alpha, beta, dr2, ds2, &c[1], scratch);
        for (int k = 0; k < n; ++k) {
            r3[k] = r[k] + 0.5f * dt * dr2[k];
            s3[k] = s[k] + 0.5f * dt * ds2[k];
        }
        kerr_derivative(n, r3, s3, gamma, omega, alpha, beta, dr3, ds3, &c[2], scratch);
        for (int k = 0; k < n; ++k) {
            r4[k] = r[k] + dt * dr3[k];
            s4[k] = s[k] + dt * ds3[k];
        }
        kerr_derivative(n, r4, s4, gamma, omega, alpha, beta, dr4, ds4, &c[3], scratch);

        float sg[1024], so[1024];
        float* stg = n <= 1024 ? sg : (float*)malloc(sizeof(float) * n);
        float* sto = n <= 1024 ? so : (float*)malloc(sizeof(float) * n);
        for (int k = 0; k < n; ++k) stg[k] = sto[k] = 0.0f;
        float sa = 0.0f, sb = 0.0f;

        memcpy(dn_r, d_r, sizeof(float) * n);
        memcpy(dn_s, d_s, sizeof(float) * n);
        /* d_r / d_s keep the direct path (r_new = r + ...): already equal. */
        for (int k = 0; k < n; ++k) {
            ddr[k] = dn_r[k] * dt6;
            dds[k] = dn_s[k] * dt6;
        }
        /* k4 = f(r4, s4) */
        deriv_backward(n, ddr, dds, r4, s4, &c[3], gamma, alpha, beta, dri, dsi, stg, sto, &sa, &sb, bw);
        for (int k = 0; k < n; ++k) {
            d_r[k] += dri[k];
            d_s[k] += dsi[k];
        }
        for (int k = 0; k < n; ++k) {
            ddr[k] = dri[k] * dt + dn_r[k] * dt6 * 2.0f;
            dds[k] = dsi[k] * dt + dn_s[k] * dt6 * 2.0f;
        }
        /* k3 = f(r3, s3) */
        deriv_backward(n, ddr, dds, r3, s3, &c[2], gamma, alpha, beta, dri, dsi, stg, sto, &sa, &sb, bw);
        for (int k = 0; k < n; ++k) {
            d_r[k] += dri[k];
            d_s[k] += dsi[k];
        }
        for (int k = 0; k < n; ++k) {
            ddr[k] = dri[k] * 0.5f * dt + dn_r[k] * dt6 * 2.0f;
            dds[k] = dsi[k] * 0.5f * dt + dn_s[k] * dt6 * 2.0f;
        }
        /* k2 = f(r2, s2) */
        deriv_backward(n, ddr, dds, r2, s2, &c[1], gamma, alpha, beta, dri, dsi, stg, sto, &sa, &sb, bw);
        for (int k = 0; k < n; ++k) {
            d_r[k] += dri[k];
            d_s[k] += dsi[k];
        }
        for (int k = 0; k < n; ++k) {
            ddr[k] = dri[k] * 0.5f * dt + dn_r[k] * dt6;
            dds[k] = dsi[k] * 0.5f * dt + dn_s[k] * dt6;
        }
        /* k1 = f(r, s) */
        deriv_backward(n, ddr, dds, r, s, &c[0], gamma, alpha, beta, dri, dsi, stg, sto, &sa, &sb, bw);
        for (int k = 0; k < n; ++k) {
            d_r[k] += dri[k];
            d_s[k] += dsi[k];
        }
        /* kerr_ode_backward (:436-443): the step's sums into the totals. */
        for (int k = 0; k < n; ++k) {
            g_acc[k] += stg[k];
            om_acc[k] += sto[k];
        }
        a_acc += sa;
        b_acc += sb;
        if (stg != sg) free(stg);
        if (sto != so) free(sto);
    }
    for (int k = 0; k < n; ++k) {
        dx[2 * k] = d_r[k];
        dx[2 * k + 1] = d_s[k];
        dgr[k] += softplus_backward(g_acc[k], gamma_raw[k]);
        dom[k] += om_acc[k];
    }
    *da += a_acc;
    *db += b_acc;
}

/* ---------------------------------------------------------------- drivers */

typedef struct {
    int lo, hi, nb, n_steps;
    const float *x, *dy, *gamma_raw, *gamma, *omega;
    long ld_x, ld_y, ld_dy, ld_dx;
    float alpha, beta;
    float *y, *dx;
    float *dgr, *dom, da, db; /* per-thread parameter sums (backward) */
} ode_job;

static void* fwd_job(void* p) {
    ode_job* j = (ode_job*)p;
    float* w = (float*)malloc(sizeof(float) * (size_t)j->nb * 16);
    for (int m = j->lo; m < j->hi; ++m)
        ode_forward_pos(j->nb, j->n_steps, j->x + (long)m * j->ld_x, j->gamma, j->omega, j->alpha, j->beta,
                        j->y + (long)m * j->ld_y, w);
    free(w);
    return NULL;
}

static void* bwd_job(void* p) {
    ode_job* j = (ode_job*)p;
    float* w = (float*)malloc(sizeof(float) * bwd_work_floats(j->nb, j->n_steps));
    for (int m = j->lo; m < j->hi; ++m)
        ode_backward_pos(j->nb, j->n_steps, j->dy + (long)m * j->ld_dy, j->x + (long)m * j->ld_x, j->gamma_raw,
                         j->gamma, j->omega, j->alpha, j->beta, j->dx + (long)m * j->ld_dx, j->dgr, j->dom, &j->da,
                         &j->db, w);
    free(w);
    return NULL;
}

static int resolve_threads(int nthreads, int M) {
    if (nthreads <= 0) {
        const long cores = sysconf(_SC_NPROCESSORS_ONLN);
        nthreads = cores > 0 ? (int)cores : 1;
    }
    if (nthreads > M) nthreads = M;
    return nthreads < 1 ? 1 : nthreads;
}

static void run_jobs(ode_job* jobs, int nt, void* (*fn)(void*)) {
    if (nt == 1) {
        fn(&jobs[0]);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nt);
    for (int t = 0; t < nt; ++t) pthread_create(&th[t], NULL, fn, &jobs[t]);
    for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
    free(th);
}

void kode_oracle_forward(int M, int nb, int n_steps, const float* x, long ld_x, const float* gamma_raw,
                         const float* omega, float alpha, float beta, float* y, long ld_y, int nthreads) {
    if (M <= 0 || nb <= 0) return;
    float* gamma = (float*)malloc(sizeof(float) * (size_t)nb);
    for (int k = 0; k < nb; ++k) gamma[k] = softplus(gamma_raw[k]);
    const int nt = resolve_threads(nthreads, M);
    ode_job* jobs = (ode_job*)calloc((size_t)nt, sizeof(ode_job));
    for (int t = 0; t < nt; ++t) {
        ode_job* j = &jobs[t];
        j->lo = (int)((long)M * t / nt);
        j->hi = (int)((long)M * (t + 1) / nt);
        j->nb = nb;
        j->n_steps = n_steps;
        j->x = x;
        j->ld_x = ld_x;
        j->y = y;
        j->ld_y = ld_y;
        j->gamma = gamma;
        j->omega = omega;
        j->alpha = alpha;
        j->beta = beta;
    }
    run_jobs(jobs, nt, fwd_job);
    free(jobs);
    free(gamma);
}

void kode_oracle_backward(int M, int nb, int n_steps, const float* dy, long ld_dy, const float* x, long ld_x,
                          const float* gamma_raw, const float* omega, float alpha, float beta, float* dx, long ld_dx,
                          float* d_gamma_raw, float* d_omega, float* d_alpha_beta, int nthreads) {
    for (int k = 0; k < nb; ++k) d_gamma_raw[k] = d_omega[k] = 0.0f;
    d_alpha_beta[0] = d_alpha_beta[1] = 0.0f;
    if (M <= 0 || nb <= 0) return;
    float* gamma = (float*)malloc(sizeof(float) * (size_t)nb);
    for (int k = 0; k < nb; ++k) gamma[k] = softplus(gamma_raw[k]);
    const int nt = resolve_threads(nthreads, M);
    ode_job* jobs = (ode_job*)calloc((size_t)nt, sizeof(ode_job));
    for (int t = 0; t < nt; ++t) {
        ode_job* j = &jobs[t];
        j->lo = (int)((long)M * t / nt);
        j->hi = (int)((long)M * (t + 1) / nt);
        j->nb = nb;
        j->n_steps = n_steps;
        j->x = x;
        j->ld_x = ld_x;
        j->dy = dy;
        j->ld_dy = ld_dy;
        j->dx = dx;
        j->ld_dx = ld_dx;
        j->gamma_raw = gamma_raw;
        j->gamma = gamma;
        j->omega = omega;
        j->alpha = alpha;
        j->beta = beta;
        j->dgr = (float*)calloc((size_t)nb, sizeof(float));
        j->dom = (float*)calloc((size_t)nb, sizeof(float));
    }
    run_jobs(jobs, nt, bwd_job);
    for (int t = 0; t < nt; ++t) {
        for (int k = 0; k < nb; ++k) {
            d_gamma_raw[k] += jobs[t].dgr[k];
            d_omega[k] += jobs[t].dom[k];
        }
        d_alpha_beta[0] += jobs[t].da;
        d_alpha_beta[1] += jobs[t].db;
        free(jobs[t].dgr);
        free(jobs[t].dom);
    }
    free(jobs);
    free(gamma);
}
