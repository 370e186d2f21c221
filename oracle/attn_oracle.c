/*
 * attn_oracle.c -- TEST INFRASTRUCTURE ONLY (see attn_oracle.h).
 *
 * CPU restatement of the reference engine's attention step, written from the
 * reference's behaviour, in the reference's operation order, so that results
 * are bit-identical to the reference compiled without FP contraction.  Built
 * with -ffp-contract=off so that every a*b+c below is two rounded operations,
 * as in the reference's scalar code.  Each function cites the reference
 * file:line it follows.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load the library built from this file.
 */
#include "attn_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32, cpp/quant.hpp:73-135 (= picolm/quant.c:11-78)             */
/* ------------------------------------------------------------------------ */

/*
 * The reference rounds the magnitude half-up (adds half an ulp, then
 * truncates), not round-to-nearest-even, and flushes f32 subnormals to a
 * signed zero (cpp/quant.hpp:110-134).  Adding half an ulp to the rebiased
 * (exponent|fraction) word lets the carry bump the exponent, which is the same
 * as the reference's explicit overflow branch, including overflow to inf.
 */
uint16_t ora_f32_to_f16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    const uint16_t sgn = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t be = (u >> 23) & 0xFFu;
    const uint32_t frac = u & 0x7FFFFFu;
    if (be == 0) return sgn;                                   /* quant.hpp:110-112 */
    if (be == 0xFF) return (uint16_t)(sgn | 0x7C00u | (frac ? 0x200u : 0u)); /* :113-115 */
    const int e = (int)be - 112;                               /* 127 -> 15 rebias */
    if (e >= 31) return (uint16_t)(sgn | 0x7C00u);             /* :116-118 */
    if (e <= 0) {                                              /* :119-126 */
        if (e < -10) return sgn;
        const uint32_t sig = frac | 0x800000u;
        const uint32_t sh = (uint32_t)(14 - e);
        return (uint16_t)(sgn | ((sig + (1u << (sh - 1))) >> sh));
    }
    const uint32_t word = (((uint32_t)e << 23) | frac) + 0x1000u; /* :128-134 */
    return (uint16_t)(sgn | (word >> 13));
}

/* Exact widening; subnormals are mant * 2^-24 (cpp/quant.hpp:73-100). */
float ora_f16_to_f32(uint16_t h) {
    const uint32_t sgn = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    uint32_t u;
    if (e == 0) {
        float mag = (float)m * 5.9604644775390625e-8f;        /* 2^-24, exact */
        memcpy(&u, &mag, sizeof u);
        u |= sgn;
    } else if (e == 31) {
        u = sgn | 0x7F800000u | (m << 13);
    } else {
        u = sgn | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

void ora_f32_to_f16_n(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = ora_f32_to_f16(in[i]);
}

void ora_f16_to_f32_n(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = ora_f16_to_f32(in[i]);
}

/* ------------------------------------------------------------------------ */
/* RMSNorm, cpp/tensor.hpp:146-176 (SSE2 path, the one x86 builds take)     */
/* ------------------------------------------------------------------------ */

/*
 * Sum of squares in four interleaved lanes (element i goes to lane i%4), the
 * lanes folded as (l0+l2)+(l1+l3) (hsum_sse, cpp/quant.hpp:296-302), then any
 * tail elements added one by one.  scale = 1/sqrtf(ss/n + eps); out = x*scale*w.
 */
void ora_rmsnorm_inplace(float* x, const float* w, int n, float eps) {
    float lane[4] = {0.f, 0.f, 0.f, 0.f};
    int i = 0;
    for (; i + 3 < n; i += 4)
        for (int j = 0; j < 4; j++) {
            const float sq = x[i + j] * x[i + j];
            lane[j] = lane[j] + sq;
        }
    float ss = (lane[0] + lane[2]) + (lane[1] + lane[3]);
    for (; i < n; i++) {
        const float sq = x[i] * x[i];
        ss = ss + sq;
    }
    const float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int d = 0; d < n; d++) {
        const float t = x[d] * scale;
        x[d] = t * w[d];
    }
}

/* ------------------------------------------------------------------------ */
/* RoPE                                                                     */
/* ------------------------------------------------------------------------ */

static void rot_pair(float* a, float* b, float c, float s) {
    const float x0 = *a, x1 = *b;
    const float p0 = x0 * c, p1 = x1 * s, p2 = x0 * s, p3 = x1 * c;
    *a = p0 - p1;
    *b = p2 + p3;
}

/* NeoX: element i pairs with i + hd/2 (cpp/tensor.hpp:201-283). */
void ora_rope_neox(float* q, float* k, int hd, int hq, int hkv,
                   const float* c, const float* s) {
    const int half = hd / 2;
    for (int h = 0; h < hq; h++)
        for (int i = 0; i < half; i++) rot_pair(q + h * hd + i, q + h * hd + i + half, c[i], s[i]);
    for (int h = 0; h < hkv; h++)
        for (int i = 0; i < half; i++) rot_pair(k + h * hd + i, k + h * hd + i + half, c[i], s[i]);
}

/* Interleaved: element 2i pairs with 2i+1 (picolm/tensor.c:247-293). */
void ora_rope_interleaved(float* q, float* k, int hd, int hq, int hkv,
                          const float* c, const float* s) {
    const int half = hd / 2;
    for (int h = 0; h < hq; h++)
        for (int i = 0; i < half; i++) rot_pair(q + h * hd + 2 * i, q + h * hd + 2 * i + 1, c[i], s[i]);
    for (int h = 0; h < hkv; h++)
        for (int i = 0; i < half; i++) rot_pair(k + h * hd + 2 * i, k + h * hd + 2 * i + 1, c[i], s[i]);
}

/* theta = (float)pos / powf(base, (float)(2i)/(float)hd) (cpp/model.hpp:1008-1017). */
void ora_rope_table(float* cos_t, float* sin_t, int max_seq, int hd, float base) {
    const int half = hd / 2;
    for (int p = 0; p < max_seq; p++)
        for (int i = 0; i < half; i++) {
            const float theta = (float)p / powf(base, (float)(2 * i) / (float)hd);
            cos_t[(size_t)p * half + i] = cosf(theta);
            sin_t[(size_t)p * half + i] = sinf(theta);
        }
}

/* ------------------------------------------------------------------------ */
/* Attention                                                                */
/* ------------------------------------------------------------------------ */

/* Online-softmax scan of one q head over cache rows [b, e), C++ engine order
 * (cpp/model.hpp:378-413).  State (m, l, acc) is updated in place. */
static void scan_rows_cpp(const float* qh, const uint16_t* kc, const uint16_t* vc,
                          int kvd, int kvh, int hd, int b, int e,
                          float* m, float* l, float* acc) {
    const float rs = sqrtf((float)hd);
    for (int t = b; t < e; t++) {
        const uint16_t* kt = kc + (size_t)t * kvd + (size_t)kvh * hd;
        const uint16_t* vt = vc + (size_t)t * kvd + (size_t)kvh * hd;
        float score = 0.0f;
        for (int d = 0; d < hd; d++) {
            const float p = qh[d] * ora_f16_to_f32(kt[d]);
            score = score + p;
        }
        score = score / rs;
        if (score > *m) {
            const float corr = expf(*m - score);
            *l = *l * corr;
            for (int d = 0; d < hd; d++) acc[d] = acc[d] * corr;
            *l = *l + 1.0f;
            for (int d = 0; d < hd; d++) acc[d] = acc[d] + ora_f16_to_f32(vt[d]);
            *m = score;
        } else {
            const float w = expf(score - *m);
            *l = *l + w;
            for (int d = 0; d < hd; d++) {
                const float p = w * ora_f16_to_f32(vt[d]);
                acc[d] = acc[d] + p;
            }
        }
    }
}

/* Same scan in the C engine's fused order (picolm/model.c:790-817). */
static void scan_rows_c(const float* qh, const uint16_t* kc, const uint16_t* vc,
                        int kvd, int kvh, int hd, int b, int e,
                        float* m, float* l, float* acc) {
    const float rs = sqrtf((float)hd);
    for (int t = b; t < e; t++) {
        const uint16_t* kt = kc + (size_t)t * kvd + (size_t)kvh * hd;
        const uint16_t* vt = vc + (size_t)t * kvd + (size_t)kvh * hd;
        float score = 0.0f;
        for (int d = 0; d < hd; d++) {
            const float p = qh[d] * ora_f16_to_f32(kt[d]);
            score = score + p;
        }
        score = score / rs;
        if (score > *m) {
            const float corr = expf(*m - score);
            *l = *l * corr + 1.0f;
            for (int d = 0; d < hd; d++) {
                const float p = acc[d] * corr;
                acc[d] = p + ora_f16_to_f32(vt[d]);
            }
            *m = score;
        } else {
            const float w = expf(score - *m);
            *l = *l + w;
            for (int d = 0; d < hd; d++) {
                const float p = w * ora_f16_to_f32(vt[d]);
                acc[d] = acc[d] + p;
            }
        }
    }
}

void ora_attend_rows(int hq, int hkv, int hd, const float* q_rot,
                     const uint16_t* kc, const uint16_t* vc,
                     int row_begin, int row_end,
                     float* m, float* l, float* acc) {
    const int g = hq / hkv, kvd = hkv * hd;
    for (int h = 0; h < hq; h++) {
        m[h] = -1e30f;
        l[h] = 0.0f;
        memset(acc + (size_t)h * hd, 0, sizeof(float) * (size_t)hd);
        scan_rows_cpp(q_rot + (size_t)h * hd, kc, vc, kvd, h / g, hd, row_begin, row_end,
                      &m[h], &l[h], acc + (size_t)h * hd);
    }
}

static int bad_shape(int hq, int hkv, int hd) {
    return hq <= 0 || hkv <= 0 || hq % hkv != 0 || hd <= 0 || hd % 2 != 0 || hd > 512;
}

/* Norm + RoPE + cache store for one token (cpp/model.hpp:326-373). */
static void prep_token(int hq, int hkv, int hd, int rope_mode, float eps,
                       float* q, float* k, const float* v,
                       const float* qn_w, const float* kn_w,
                       const float* c, const float* s,
                       uint16_t* kc, uint16_t* vc, int pos) {
    const int kvd = hkv * hd;
    if (qn_w)
        for (int h = 0; h < hq; h++) ora_rmsnorm_inplace(q + (size_t)h * hd, qn_w, hd, eps);
    if (kn_w)
        for (int h = 0; h < hkv; h++) ora_rmsnorm_inplace(k + (size_t)h * hd, kn_w, hd, eps);
    if (rope_mode == 0) ora_rope_neox(q, k, hd, hq, hkv, c, s);
    else ora_rope_interleaved(q, k, hd, hq, hkv, c, s);
    ora_f32_to_f16_n(k, kc + (size_t)pos * kvd, (size_t)kvd);
    ora_f32_to_f16_n(v, vc + (size_t)pos * kvd, (size_t)kvd);
}

/* Attention of one token over rows [0, pos] (cpp/model.hpp:375-418). */
static void attend_token(int hq, int hkv, int hd, const float* q,
                         const uint16_t* kc, const uint16_t* vc, int pos,
                         float* out, int variant, int h_begin, int h_end) {
    const int g = hq / hkv, kvd = hkv * hd;
    float* acc = (float*)malloc(sizeof(float) * (size_t)hd);
    for (int h = h_begin; h < h_end; h++) {
        float m = -1e30f, l = 0.0f;
        memset(acc, 0, sizeof(float) * (size_t)hd);
        if (variant == 0) {
            scan_rows_cpp(q + (size_t)h * hd, kc, vc, kvd, h / g, hd, 0, pos + 1, &m, &l, acc);
            for (int d = 0; d < hd; d++) out[(size_t)h * hd + d] = acc[d] / l;
        } else {
            scan_rows_c(q + (size_t)h * hd, kc, vc, kvd, h / g, hd, 0, pos + 1, &m, &l, acc);
            const float inv = 1.0f / l;
            for (int d = 0; d < hd; d++) out[(size_t)h * hd + d] = acc[d] * inv;
        }
    }
    free(acc);
}

int ora_decode_step(int hq, int hkv, int hd, int rope_mode, float eps,
                    float* q, float* k, const float* v,
                    const float* qn_w, const float* kn_w,
                    const float* cos_row, const float* sin_row,
                    uint16_t* kc, uint16_t* vc, int pos, float* out, int variant) {
    if (bad_shape(hq, hkv, hd) || pos < 0 || !q || !k || !v || !kc || !vc || !out) return -1;
    prep_token(hq, hkv, hd, rope_mode, eps, q, k, v, qn_w, kn_w, cos_row, sin_row, kc, vc, pos);
    attend_token(hq, hkv, hd, q, kc, vc, pos, out, variant, 0, hq);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Threaded drivers (same arithmetic per head; tasks are independent)       */
/* ------------------------------------------------------------------------ */

typedef struct {
    int (*fn)(void* ctx, int task);
    void* ctx;
    int n_tasks;
    int next;
    pthread_mutex_t mu;
} pool_t;

static void* pool_worker(void* arg) {
    pool_t* p = (pool_t*)arg;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        const int t = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (t >= p->n_tasks) break;
        p->fn(p->ctx, t);
    }
    return NULL;
}

static void run_tasks(int (*fn)(void*, int), void* ctx, int n_tasks, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_tasks) n_threads = n_tasks;
    pool_t p = {fn, ctx, n_tasks, 0, PTHREAD_MUTEX_INITIALIZER};
    if (n_threads <= 1) {
        pool_worker(&p);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, pool_worker, &p);
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    free(th);
}

typedef struct {
    int hq, hkv, hd;
    const float* qrot;       /* [n_tok][hq*hd] rotated */
    const uint16_t *kc, *vc;
    int start_pos;
    float* out;
} prefill_ctx_t;

static int prefill_task(void* vctx, int task) {
    prefill_ctx_t* c = (prefill_ctx_t*)vctx;
    const int qd = c->hq * c->hd;
    attend_token(c->hq, c->hkv, c->hd, c->qrot + (size_t)task * qd, c->kc, c->vc,
                 c->start_pos + task, c->out + (size_t)task * qd, 0, 0, c->hq);
    return 0;
}

int ora_prefill(int hq, int hkv, int hd, int rope_mode, float eps,
                const float* q, const float* k, const float* v,
                const float* qn_w, const float* kn_w,
                const float* cos_t, const float* sin_t,
                uint16_t* kc, uint16_t* vc, int start_pos, int n_tok,
                float* out, int n_threads) {
    if (bad_shape(hq, hkv, hd) || start_pos < 0 || n_tok < 0) return -1;
    const int qd = hq * hd, kvd = hkv * hd, half = hd / 2;
    float* qrot = (float*)malloc(sizeof(float) * (size_t)n_tok * qd + 1);
    float* kt = (float*)malloc(sizeof(float) * (size_t)kvd);
    /* Every token's k/v row is stored before any token reads rows beyond its
     * own position, so storing all rows first and then attending (in parallel)
     * reads exactly what the reference's token-by-token loop reads. */
    for (int i = 0; i < n_tok; i++) {
        const int pos = start_pos + i;
        memcpy(qrot + (size_t)i * qd, q + (size_t)i * qd, sizeof(float) * (size_t)qd);
        memcpy(kt, k + (size_t)i * kvd, sizeof(float) * (size_t)kvd);
        prep_token(hq, hkv, hd, rope_mode, eps, qrot + (size_t)i * qd, kt, v + (size_t)i * kvd,
                   qn_w, kn_w, cos_t + (size_t)pos * half, sin_t + (size_t)pos * half, kc, vc, pos);
    }
    prefill_ctx_t ctx = {hq, hkv, hd, qrot, kc, vc, start_pos, out};
    run_tasks(prefill_task, &ctx, n_tok, n_threads);
    free(kt);
    free(qrot);
    return 0;
}

typedef struct {
    int hq, hkv, hd, rope_mode;
    float eps;
    const float *q, *k, *v, *qn_w, *kn_w, *cos_t, *sin_t;
    uint16_t* const* kc;
    uint16_t* const* vc;
    const int* pos;
    float* out;
} batch_ctx_t;

static int batch_task(void* vctx, int b) {
    batch_ctx_t* c = (batch_ctx_t*)vctx;
    const int qd = c->hq * c->hd, kvd = c->hkv * c->hd, half = c->hd / 2;
    float* qb = (float*)malloc(sizeof(float) * (size_t)(qd + kvd));
    float* kb = qb + qd;
    memcpy(qb, c->q + (size_t)b * qd, sizeof(float) * (size_t)qd);
    memcpy(kb, c->k + (size_t)b * kvd, sizeof(float) * (size_t)kvd);
    const int p = c->pos[b];
    ora_decode_step(c->hq, c->hkv, c->hd, c->rope_mode, c->eps, qb, kb, c->v + (size_t)b * kvd,
                    c->qn_w, c->kn_w, c->cos_t + (size_t)p * half, c->sin_t + (size_t)p * half,
                    c->kc[b], c->vc[b], p, c->out + (size_t)b * qd, 0);
    free(qb);
    return 0;
}

int ora_decode_batch(int B, int hq, int hkv, int hd, int rope_mode, float eps,
                     const float* q, const float* k, const float* v,
                     const float* qn_w, const float* kn_w,
                     const float* cos_t, const float* sin_t,
                     uint16_t* const* kc, uint16_t* const* vc,
                     const int* pos, float* out, int n_threads) {
    if (bad_shape(hq, hkv, hd) || B < 0) return -1;
    batch_ctx_t ctx = {hq, hkv, hd, rope_mode, eps, q, k, v, qn_w, kn_w, cos_t, sin_t, kc, vc, pos, out};
    run_tasks(batch_task, &ctx, B, n_threads);
    return 0;
}

typedef struct {
    int hq, hkv, hd, n_parts;
    const float* qrot;
    const uint16_t *kc, *vc;
    int pos;
    float* out;
} heads_ctx_t;

static int heads_task(void* vctx, int task) {
    heads_ctx_t* c = (heads_ctx_t*)vctx;
    const int h0 = (int)((long long)task * c->hq / c->n_parts), h1 = (int)((long long)(task + 1) * c->hq / c->n_parts);
    attend_token(c->hq, c->hkv, c->hd, c->qrot, c->kc, c->vc, c->pos, c->out, 0, h0, h1);
    return 0;
}

/* ora_decode_step (variant 0) with the q heads spread over n_threads host
 * threads: the same per-head arithmetic, for one long sequence. */
int ora_decode_step_mt(int hq, int hkv, int hd, int rope_mode, float eps,
                       float* q, float* k, const float* v,
                       const float* qn_w, const float* kn_w,
                       const float* cos_row, const float* sin_row,
                       uint16_t* kc, uint16_t* vc, int pos, float* out, int n_threads) {
    if (bad_shape(hq, hkv, hd) || pos < 0 || !q || !k || !v || !kc || !vc || !out) return -1;
    prep_token(hq, hkv, hd, rope_mode, eps, q, k, v, qn_w, kn_w, cos_row, sin_row, kc, vc, pos);
    heads_ctx_t ctx = {hq, hkv, hd, hq, q, kc, vc, pos, out};
    run_tasks(heads_task, &ctx, hq, n_threads);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Projections: GGUF block dequantisation and the mat-vec                   */
/* ------------------------------------------------------------------------ */

/* gguf_type_block_size / gguf_type_quant_size, cpp/quant.hpp:137-166 */
int ora_weight_block(int type, int* elems, int* bytes) {
    int e = 0, b = 0;
    switch (type) {
        case 1: e = 1; b = 4; break;     /* F32 */
        case 2: e = 1; b = 2; break;     /* F16 */
        case 3: e = 32; b = 18; break;   /* Q4_0: fp16 d, 16 bytes of nibbles */
        case 9: e = 32; b = 34; break;   /* Q8_0: fp16 d, 32 int8 */
        case 13: e = 256; b = 144; break; /* Q4_K: d, dmin, 12 scale bytes, 128 nibble bytes */
        case 15: e = 256; b = 210; break; /* Q6_K: 128 low, 64 high bytes, 16 int8 scales, d */
        default: return 0;
    }
    if (elems) *elems = e;
    if (bytes) *bytes = b;
    return 1;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* get_scale_min_k4, cpp/quant.hpp:210-218 */
static void scale_min_k4(int j, const uint8_t* q, int* sc, int* mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

void ora_dequant_row(const void* src, float* dst, int n, int type) {
    const uint8_t* p = (const uint8_t*)src;
    switch (type) {
        case 1: memcpy(dst, src, (size_t)n * sizeof(float)); return;        /* quant.hpp:175-177 */
        case 2:                                                           /* quant.hpp:180-185 */
            for (int i = 0; i < n; i++) dst[i] = ora_f16_to_f32(rd16(p + 2 * i));
            return;
        case 3:                                                           /* quant.hpp:197-207 */
            for (int b = 0; b < n / 32; b++, p += 18) {
                const float d = ora_f16_to_f32(rd16(p));
                for (int j = 0; j < 32; j++) {
                    const int nib = j < 16 ? (p[2 + j] & 0xF) : (p[2 + j - 16] >> 4);
                    dst[32 * b + j] = d * ((float)nib - 8.0f);
                }
            }
            return;
        case 9:                                                           /* quant.hpp:187-195 */
            for (int b = 0; b < n / 32; b++, p += 34) {
                const float d = ora_f16_to_f32(rd16(p));
                for (int j = 0; j < 32; j++) dst[32 * b + j] = d * (float)(int8_t)p[2 + j];
            }
            return;
        case 13:                                                          /* quant.hpp:220-251 */
            for (int b = 0; b < n / 256; b++, p += 144) {
                const float d = ora_f16_to_f32(rd16(p)), dmin = ora_f16_to_f32(rd16(p + 2));
                const uint8_t* q = p + 16;
                float* y = dst + 256 * b;
                for (int j = 0; j < 4; j++, y += 64, q += 32) {
                    int sc, mn;
                    scale_min_k4(2 * j, p + 4, &sc, &mn);
                    const float d1 = d * (float)sc, m1 = dmin * (float)mn;
                    scale_min_k4(2 * j + 1, p + 4, &sc, &mn);
                    const float d2 = d * (float)sc, m2 = dmin * (float)mn;
                    for (int l = 0; l < 32; l++) y[l] = d1 * (float)(q[l] & 0xF) - m1;
                    for (int l = 0; l < 32; l++) y[l + 32] = d2 * (float)(q[l] >> 4) - m2;
                }
            }
            return;
        case 15:                                                          /* quant.hpp:253-281 */
            for (int b = 0; b < n / 256; b++, p += 210) {
                const uint8_t* ql = p;
                const uint8_t* qh = p + 128;
                const int8_t* sc = (const int8_t*)(p + 192);
                const float d = ora_f16_to_f32(rd16(p + 208));
                float* y = dst + 256 * b;
                for (int c = 0; c < 2; c++, y += 128, ql += 64, qh += 32) {
                    const int is = 8 * c;
                    for (int l = 0; l < 32; l++) {
                        const int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                        const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                        const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                        const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                        const int il = is + l / 16;
                        y[l] = d * (float)sc[il] * (float)q1;
                        y[l + 32] = d * (float)sc[il + 2] * (float)q2;
                        y[l + 64] = d * (float)sc[il + 4] * (float)q3;
                        y[l + 96] = d * (float)sc[il + 6] * (float)q4;
                    }
                }
            }
            return;
        default:
            for (int i = 0; i < n; i++) dst[i] = 0.f;
    }
}

/* vec_dot_f32_f32 with PICOLM_SSE2 (cpp/quant.hpp:296-323): two 4-lane
 * accumulators over 8 elements per step (product rounded, then added), the
 * lanes summed (v0+v2)+(v1+v3) (hsum_sse), then the tail in order. */
static float dot_f32(const float* w, const float* x, int n) {
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
    int i = 0;
    for (; i + 7 < n; i += 8)
        for (int j = 0; j < 4; j++) {
            a0[j] = a0[j] + w[i + j] * x[i + j];
            a1[j] = a1[j] + w[i + 4 + j] * x[i + 4 + j];
        }
    float v[4];
    for (int j = 0; j < 4; j++) v[j] = a0[j] + a1[j];
    float sum = (v[0] + v[2]) + (v[1] + v[3]);
    for (; i < n; i++) sum += w[i] * x[i];
    return sum;
}

float ora_vec_dot(const void* row, const float* x, int n, int type) {
    if (type == 1) return dot_f32((const float*)row, x, n);
    if (type == 9) {  /* vec_dot_q8_0_f32, cpp/quant.hpp:325-343 */
        const uint8_t* p = (const uint8_t*)row;
        float sumf = 0.0f;
        for (int b = 0; b < n / 32; b++, p += 34) {
            const float d = ora_f16_to_f32(rd16(p));
            float sum = 0.0f;
            for (int j = 0; j < 32; j++) sum += (float)(int8_t)p[2 + j] * x[32 * b + j];
            sumf += d * sum;
        }
        return sumf;
    }
    float* buf = (float*)malloc((size_t)n * sizeof(float));   /* cpp/quant.hpp:349-355 */
    if (!buf) return 0.0f;
    ora_dequant_row(row, buf, n, type);
    const float s = dot_f32(buf, x, n);
    free(buf);
    return s;
}

void ora_matvec(const void* w, int type, const float* bias, int n_in, int n_out, int n_vec,
                const float* x, float* out, int accumulate) {
    int e = 0, b = 0;
    if (!ora_weight_block(type, &e, &b)) return;
    const size_t row_bytes = (size_t)(n_in / e) * (size_t)b;
    for (int v = 0; v < n_vec; v++)
        for (int d = 0; d < n_out; d++) {
            float y = ora_vec_dot((const uint8_t*)w + (size_t)d * row_bytes, x + (size_t)v * n_in, n_in, type);
            if (bias) y += bias[d];                              /* matmul_bias: vec_add of the bias */
            float* o = out + (size_t)v * n_out + d;
            *o = accumulate ? *o + y : y;                        /* the residual add, cpp/model.hpp:427 */
        }
}
