/*
 * ORACLE — test infrastructure only (see kattn_oracle.h).  PARITY UNPINNED:
 * the reference has no attention golden vectors; this restatement follows its
 * loops statement by statement and is cross-checked against float64 autograd.
 *
 * Build with -ffp-contract=off: Rust never fuses a*b+c into an FMA, and gcc
 * would otherwise contract the dot products below on an FMA-capable -march.
 */
#include "kattn_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* src/pipeline.rs:305-347 (forward head loop of attention_with_cache). */
void kattn_oracle_forward_seq(int T, int C, int H,
                              const float* q, const float* k, const float* v, long ld_qkv,
                              float* out, long ld_o, float* att_cache, float* lse) {
    const int hd = C / H;
    /* src/pipeline.rs:285: let scale = 1.0 / (head_dim as f32).sqrt(); */
    const float scale = 1.0f / sqrtf((float)hd);
    float* att = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));

    for (int qi = 0; qi < T; ++qi)
        for (int c = 0; c < C; ++c) out[(long)qi * ld_o + c] = 0.0f;

    for (int head = 0; head < H; ++head) {
        const int offset = head * hd;
        for (int qi = 0; qi < T; ++qi) {
            /* :318 reset to -inf for causal masking */
            for (int ki = 0; ki < T; ++ki) att[ki] = -INFINITY;
            /* :320-327 scores for ki <= qi */
            for (int ki = 0; ki <= qi; ++ki) {
                float dot = 0.0f;
                for (int d = 0; d < hd; ++d)
                    dot += q[(long)qi * ld_qkv + offset + d] * k[(long)ki * ld_qkv + offset + d];
                att[ki] = dot * scale;
            }
            /* :329 max via f32::max fold from -inf (fmaxf has the same NaN rule) */
            float max_att = -INFINITY;
            for (int ki = 0; ki <= qi; ++ki) max_att = fmaxf(max_att, att[ki]);
            /* :330-334 exp and running sum, then :335-337 normalise */
            float exp_sum = 0.0f;
            for (int ki = 0; ki <= qi; ++ki) {
                att[ki] = expf(att[ki] - max_att);
                exp_sum += att[ki];
            }
            for (int ki = 0; ki <= qi; ++ki) att[ki] /= exp_sum;
            if (lse) lse[(long)head * T + qi] = (float)((double)max_att + log((double)exp_sum));
            /* :340 copy the whole row (above-diagonal entries stay -inf) */
            if (att_cache) memcpy(att_cache + ((long)head * T + qi) * T, att, sizeof(float) * (size_t)T);
            /* :342-348 weighted sum of values */
            for (int d = 0; d < hd; ++d) {
                float sum = 0.0f;
                for (int ki = 0; ki <= qi; ++ki) sum += att[ki] * v[(long)ki * ld_qkv + offset + d];
                out[(long)qi * ld_o + offset + d] = sum;
            }
        }
    }
    free(att);
}

/* src/backward.rs:464-514 (attention_backward_single) for one query position. */
static void attention_backward_single(int T, int C, int H, const float* d_out,
                                      const float* q, const float* k, const float* v, long ld_qkv,
                                      const float* att_all, int pos,
                                      float* d_q, float* d_k, float* d_v, long ld_d,
                                      float* d_att, float* d_score) {
    const int hd = C / H;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int head = 0; head < H; ++head) {
        const int offset = head * hd;
        /* src/backend.rs:360-361: att_for_pos[head] = att_weights[head][pos] */
        const float* att = att_all + ((long)head * T + pos) * T;
        /* :488-497 d_att[ki] = d_out . v[ki]; d_v[ki] += att[ki] * d_out */
        for (int ki = 0; ki <= pos; ++ki) {
            float dot = 0.0f;
            for (int d = 0; d < hd; ++d) {
                dot += d_out[offset + d] * v[(long)ki * ld_qkv + offset + d];
                d_v[(long)ki * ld_d + offset + d] += att[ki] * d_out[offset + d];
            }
            d_att[ki] = dot;
        }
        /* :501 iterator sum; Rust's float Sum folds from -0.0 */
        float att_d_att_sum = -0.0f;
        for (int j = 0; j <= pos; ++j) att_d_att_sum += att[j] * d_att[j];
        /* :502-505 */
        for (int ki = 0; ki <= pos; ++ki) d_score[ki] = att[ki] * (d_att[ki] - att_d_att_sum);
        /* :510-515, products evaluated left to right as written */
        for (int ki = 0; ki <= pos; ++ki) {
            for (int d = 0; d < hd; ++d) {
                d_q[(long)pos * ld_d + offset + d] += d_score[ki] * k[(long)ki * ld_qkv + offset + d] * scale;
                d_k[(long)ki * ld_d + offset + d] += d_score[ki] * q[(long)pos * ld_qkv + offset + d] * scale;
            }
        }
    }
}

/* src/backend.rs:344-373 (CpuBackend::attention_backward). */
void kattn_oracle_backward_seq(int T, int C, int H,
                               const float* d_out, long ld_o,
                               const float* q, const float* k, const float* v, long ld_qkv,
                               const float* att,
                               float* dq, float* dk, float* dv, long ld_d) {
    for (int t = 0; t < T; ++t)
        for (int c = 0; c < C; ++c) {
            dq[(long)t * ld_d + c] = 0.0f;
            dk[(long)t * ld_d + c] = 0.0f;
            dv[(long)t * ld_d + c] = 0.0f;
        }
    float* d_att = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
    float* d_score = (float*)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
    for (int pos = 0; pos < T; ++pos)
        attention_backward_single(T, C, H, d_out + (long)pos * ld_o, q, k, v, ld_qkv, att, pos,
                                  dq, dk, dv, ld_d, d_att, d_score);
    free(d_att);
    free(d_score);
}

/* ---- batched drivers: src/train.rs:241-255 runs one sequence per host thread ---- */

typedef struct {
    int fwd, B, T, C, H, tid, nthreads;
    const float *q, *k, *v, *d_out, *att_in;
    long ld_qkv, ld_o, ld_d;
    float *out, *att, *lse, *dq, *dk, *dv;
} job_t;

static void* run_job(void* p) {
    job_t* j = (job_t*)p;
    for (int b = j->tid; b < j->B; b += j->nthreads) {
        const long so = (long)b * j->T;
        const long sa = (long)b * j->H * j->T * j->T;
        if (j->fwd) {
            kattn_oracle_forward_seq(j->T, j->C, j->H, j->q + so * j->ld_qkv, j->k + so * j->ld_qkv,
                                     j->v + so * j->ld_qkv, j->ld_qkv, j->out + so * j->ld_o, j->ld_o,
                                     j->att ? j->att + sa : NULL,
                                     j->lse ? j->lse + (long)b * j->H * j->T : NULL);
        } else {
            kattn_oracle_backward_seq(j->T, j->C, j->H, j->d_out + so * j->ld_o, j->ld_o,
                                      j->q + so * j->ld_qkv, j->k + so * j->ld_qkv,
                                      j->v + so * j->ld_qkv, j->ld_qkv, j->att_in + sa,
                                      j->dq + so * j->ld_d, j->dk + so * j->ld_d,
                                      j->dv + so * j->ld_d, j->ld_d);
        }
    }
    return NULL;
}

int kattn_oracle_default_threads(int B) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    return (int)(n < B ? n : (B > 0 ? B : 1));
}

static void run_batch(job_t proto, int nthreads) {
    if (nthreads <= 0) nthreads = kattn_oracle_default_threads(proto.B);
    if (nthreads > proto.B) nthreads = proto.B > 0 ? proto.B : 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    job_t* jobs = (job_t*)malloc(sizeof(job_t) * (size_t)nthreads);
    for (int i = 0; i < nthreads; ++i) {
        jobs[i] = proto;
        jobs[i].tid = i;
        jobs[i].nthreads = nthreads;
        if (i > 0) pthread_create(&th[i], NULL, run_job, &jobs[i]);
    }
    run_job(&jobs[0]);
    for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
}

void kattn_oracle_forward_batch(int B, int T, int C, int H,
                                const float* q, const float* k, const float* v, long ld_qkv,
                                float* out, long ld_o, float* att, float* lse, int nthreads) {
    job_t j;
    memset(&j, 0, sizeof j);
    j.fwd = 1; j.B = B; j.T = T; j.C = C; j.H = H;
    j.q = q; j.k = k; j.v = v; j.ld_qkv = ld_qkv;
    j.out = out; j.ld_o = ld_o; j.att = att; j.lse = lse;
    run_batch(j, nthreads);
}

void kattn_oracle_backward_batch(int B, int T, int C, int H,
                                 const float* d_out, long ld_o,
                                 const float* q, const float* k, const float* v, long ld_qkv,
                                 const float* att,
                                 float* dq, float* dk, float* dv, long ld_d, int nthreads) {
    job_t j;
    memset(&j, 0, sizeof j);
    j.fwd = 0; j.B = B; j.T = T; j.C = C; j.H = H;
    j.d_out = d_out; j.ld_o = ld_o;
    j.q = q; j.k = k; j.v = v; j.ld_qkv = ld_qkv; j.att_in = att;
    j.dq = dq; j.dk = dk; j.dv = dv; j.ld_d = ld_d;
    run_batch(j, nthreads);
}
