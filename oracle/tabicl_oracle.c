/*
 * TEST INFRASTRUCTURE ONLY - the parity oracle and timed CPU baseline.
 *
 * A plain-C restatement of tabicl-anywhere's CPU prediction path (the Rust crate cannot be built here: no Rust
 * toolchain), used by tests/ as the checker and by bench.py as the CPU baseline. Nothing in the product links,
 * loads or calls this file. Every function cites the reference file:line it restates (paths inside the
 * tabicl-anywhere repository). Arithmetic is f32 as in the reference; compiled with -ffp-contract=off so that no
 * multiply-add is fused unless written as fmaf (the reference's `mul_add_e` inner loops), as Rust never fuses on
 * its own.
 *
 * Parity is pinned by tests/test_oracle_golden.py against the reference's committed golden vectors
 * (tests/data/tiny-raw.tirs: PyTorch TabICL's row representations, in-context keys/values and logits).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>

#define EXPORT __attribute__((visibility("default")))

/* ---- a small parallel-for over host threads (the reference's rayon `each`, predict.rs:270-278) ---------- */

static int g_threads = 0;

EXPORT void or_set_threads(int n) { g_threads = n; }

EXPORT int or_threads(void) {
    if (g_threads > 0) return g_threads;
    const char *e = getenv("ORACLE_THREADS");
    if (e && atoi(e) > 0) return atoi(e);
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef struct {
    void (*fn)(void *, int);
    void *ctx;
    int n;
    atomic_int next;
} par_job;

static void *par_worker(void *arg) {
    par_job *j = (par_job *)arg;
    for (;;) {
        int i = atomic_fetch_add(&j->next, 1);
        if (i >= j->n) break;
        j->fn(j->ctx, i);
    }
    return NULL;
}

static void par_for(int n, void (*fn)(void *, int), void *ctx) {
    int t = or_threads();
    if (t > n) t = n;
    if (t <= 1) {
        for (int i = 0; i < n; i++) fn(ctx, i);
        return;
    }
    par_job j;
    j.fn = fn, j.ctx = ctx, j.n = n;
    atomic_init(&j.next, 0);
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * t);
    for (int k = 1; k < t; k++) pthread_create(&th[k], NULL, par_worker, &j);
    par_worker(&j);
    for (int k = 1; k < t; k++) pthread_join(th[k], NULL);
    free(th);
}

/* ---- kern.rs: scalar restatements of the inner loops ---------------------------------------------------- */

/* kern.rs:214-216 */
static const float OR_LOG2E = 1.44269504088896340736f;
static const float OR_LN2_HI = 0.6933594f;
static const float OR_LN2_LO = -2.1219444e-4f;

static inline float clampf(float x, float lo, float hi) {
    /* Rust f32::clamp: NaN stays NaN */
    if (x < lo) return lo;
    if (x > hi) return hi;
    return x;
}

static inline float f32_from_bits(uint32_t b) {
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* kern.rs:220-235 - the reference's own exponential: Cody-Waite reduction and a degree-7 Taylor polynomial,
 * clamped to [-87, 88]. */
EXPORT float or_exp1(float x) {
    x = clampf(x, -87.0f, 88.0f);
    float n = floorf(x * OR_LOG2E + 0.5f);
    float r = (x - n * OR_LN2_HI) - n * OR_LN2_LO;
    float p = 1.0f / 5040.0f;
    p = p * r + 1.0f / 720.0f;
    p = p * r + 1.0f / 120.0f;
    p = p * r + 1.0f / 24.0f;
    p = p * r + 1.0f / 6.0f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    return p * f32_from_bits(((uint32_t)((int32_t)n + 127)) << 23);
}

/* kern.rs:256-282 - erf by Abramowitz and Stegun 7.1.26, and its power series below 0.5. */
EXPORT float or_erf1(float x) {
    float a = fabsf(x);
    float t = 1.0f / (1.0f + 0.3275911f * a);
    float p = 1.0614054f;
    p = p * t - 1.4531521f;
    p = p * t + 1.4214138f;
    p = p * t - 0.28449674f;
    p = p * t + 0.2548296f;
    float far = copysignf(1.0f - p * t * or_exp1(-a * a), x);
    float x2 = x * x;
    float q = -1.0f / 1320.0f;
    q = q * x2 + 1.0f / 216.0f;
    q = q * x2 - 1.0f / 42.0f;
    q = q * x2 + 0.1f;
    q = q * x2 - 1.0f / 3.0f;
    q = q * x2 + 1.0f;
    float near = q * x * 1.12837916709551257390f; /* FRAC_2_SQRT_PI */
    return a < 0.5f ? near : far;
}

/* kern.rs:285-290 */
EXPORT float or_gelu1(float v) { return 0.5f * v * (1.0f + or_erf1(v * 0.70710678118654752440f)); }

static void gelu_inplace(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] = or_gelu1(x[i]);
}

/* kern.rs:292-297 */
EXPORT float or_tanh1(float x) {
    float e = or_exp1(2.0f * clampf(x, -10.0f, 10.0f));
    return (e - 1.0f) / (e + 1.0f);
}

/* kern.rs:42-61 - dot with four running sums (lane order simplified to one chain per sum) */
static float dot(const float *a, const float *b, int n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int i = 0;
    for (; i + 4 <= n; i += 4) {
        s0 = fmaf(a[i], b[i], s0);
        s1 = fmaf(a[i + 1], b[i + 1], s1);
        s2 = fmaf(a[i + 2], b[i + 2], s2);
        s3 = fmaf(a[i + 3], b[i + 3], s3);
    }
    float s = (s0 + s1) + (s2 + s3);
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

/* kern.rs:95-150 matvec, kern.rs:154-159 linear: y = w x (+ b), w is [out][in] */
static void linear(const float *w, const float *b, const float *x, int in, int out, float *y) {
    for (int o = 0; o < out; o++) {
        float v = dot(w + (size_t)o * in, x, in);
        y[o] = b ? v + b[o] : v;
    }
}

/* kern.rs:357-376 - layer norm over the whole vector, eps 1e-5, biased variance */
static void layer_norm(const float *x, const float *w, const float *b, int n, float *y) {
    float s = 0;
    for (int i = 0; i < n; i++) s += x[i];
    float mean = s / (float)n;
    float q = 0;
    for (int i = 0; i < n; i++) {
        float d = x[i] - mean;
        q = fmaf(d, d, q);
    }
    float var = q / (float)n;
    float inv = 1.0f / sqrtf(var + 1e-5f);
    for (int i = 0; i < n; i++) y[i] = (x[i] - mean) * inv * w[i] + b[i];
}

/* kern.rs:163-197 weighted_sum: acc[i] += sum_r wts[r] * rows[r][i], rows taken four at a time */
static void weighted_sum(const float *wts, const float *rows, int nrows, int n, float *acc) {
    int r = 0;
    for (; r + 4 <= nrows; r += 4) {
        const float *r0 = rows + (size_t)r * n, *r1 = r0 + n, *r2 = r1 + n, *r3 = r2 + n;
        for (int i = 0; i < n; i++) {
            float a = fmaf(wts[r], r0[i], acc[i]);
            float bb = wts[r + 1] * r1[i];
            a = fmaf(wts[r + 2], r2[i], a);
            bb = fmaf(wts[r + 3], r3[i], bb);
            acc[i] = a + bb;
        }
    }
    for (; r < nrows; r++)
        for (int i = 0; i < n; i++) acc[i] = fmaf(wts[r], rows[(size_t)r * n + i], acc[i]);
}

/* kern.rs:302-323 weighted_sum_int, for 16- and 8-bit rows */
#define WEIGHTED_SUM_INT(NAME, T)                                                                                 \
    static void NAME(const float *wts, const T *rows, int nrows, int n, float *acc) {                             \
        int r = 0;                                                                                                \
        for (; r + 4 <= nrows; r += 4) {                                                                          \
            const T *r0 = rows + (size_t)r * n, *r1 = r0 + n, *r2 = r1 + n, *r3 = r2 + n;                        \
            for (int i = 0; i < n; i++)                                                                           \
                acc[i] += (wts[r] * (float)r0[i] + wts[r + 1] * (float)r1[i]) +                                    \
                          (wts[r + 2] * (float)r2[i] + wts[r + 3] * (float)r3[i]);                                 \
        }                                                                                                         \
        for (; r < nrows; r++)                                                                                    \
            for (int i = 0; i < n; i++) acc[i] += wts[r] * (float)rows[(size_t)r * n + i];                       \
    }
WEIGHTED_SUM_INT(weighted_sum_i16, int16_t)
WEIGHTED_SUM_INT(weighted_sum_i8, int8_t)

/* kern.rs:328-353 matvec_int: y[j] = rows[j] . x with sixteen running sums */
#define MATVEC_INT(NAME, T)                                                                                       \
    static void NAME(const T *rows, const float *x, int n, int nout, float *y) {                                  \
        for (int j = 0; j < nout; j++) {                                                                          \
            const T *row = rows + (size_t)j * n;                                                                  \
            float a[16] = {0};                                                                                    \
            int i = 0;                                                                                            \
            for (; i + 16 <= n; i += 16)                                                                          \
                for (int l = 0; l < 16; l++) a[l] += (float)row[i + l] * x[i + l];                                \
            float s = 0;                                                                                          \
            for (int l = 0; l < 8; l++) s += a[l] + a[l + 8];                                                     \
            for (; i < n; i++) s += (float)row[i] * x[i];                                                         \
            y[j] = s;                                                                                             \
        }                                                                                                         \
    }
MATVEC_INT(matvec_i16, int16_t)
MATVEC_INT(matvec_i8, int8_t)

/* kern.rs:95-150 matvec over f32 rows (values [hd][r] times weights [r]) */
static void matvec(const float *w, const float *x, int n, int nout, float *y) {
    for (int j = 0; j < nout; j++) y[j] = dot(w + (size_t)j * n, x, n);
}

/* kern.rs:201-212 */
static float vmax(const float *x, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = x[i] > m ? x[i] : m;
    return m;
}

/* kern.rs:239-254 exp_shift_sum: x[i] = e^(x[i] - shift), eight lane sums */
static float exp_shift_sum(float *x, int n, float shift) {
    float s[8] = {0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) {
            x[i + l] = or_exp1(x[i + l] - shift);
            s[l] += x[i + l];
        }
    float t = 0;
    for (int l = 0; l < 8; l++) t += s[l];
    for (; i < n; i++) {
        x[i] = or_exp1(x[i] - shift);
        t += x[i];
    }
    return t;
}

/* ---- the model as the oracle sees it ----------------------------------------------------------------------- */

/* One in-context block (model.rs:27-98); `wkv`/`bkv` are in_proj rows d..3d (fit only), `sb*` the scalable
 * softmax's base MLP (model.rs:15-24; fit-time query_scale only). */
typedef struct {
    const float *n1w, *n1b, *wq, *bq, *q0w, *q0b, *q2w, *q2b, *wo, *bo, *n2w, *n2b, *w1, *b1, *w2, *b2;
    const float *wkv, *bkv, *sb0w, *sb0b, *sb2w, *sb2b;
} or_layer;

typedef struct {
    int d, heads, ff, hid, layers, dff, outs, max_classes;
    const or_layer *layer;
    const float *lnw, *lnb, *dec0w, *dec0b, *dec2w, *dec2b;
    const float *icl_y; /* classifier: [classes][d] (model.rs:163-177); regression: [weight d][bias d] */
} or_model;

/* fit.rs:103-127: bytes of one stored chunk of `rc` rows */
EXPORT size_t or_record(int kv, int d, int rc) {
    int w = kv == 0 ? 4 : (kv == 1 ? 2 : 1);
    return (size_t)2 * d * rc * w + (kv == 0 ? 0 : (size_t)8 * d);
}

/* nn.rs:97-107 Block::query_scale: the scalable softmax's length term times 1/sqrt(head width) */
EXPORT void or_query_scale(const or_model *m, int l, int n, float *out) {
    const or_layer *b = &m->layer[l];
    int d = m->d, hd = d / m->heads, hid = m->hid;
    float inv = 1.0f / sqrtf((float)hd);
    float logn = logf((float)(n > 1 ? n : 1));
    float *h = (float *)malloc(sizeof(float) * hid);
    for (int i = 0; i < hid; i++) h[i] = b->sb0w[i] * logn + b->sb0b[i];
    gelu_inplace(h, hid);
    linear(b->sb2w, b->sb2b, h, hid, d, out);
    for (int i = 0; i < d; i++) out[i] *= inv;
    free(h);
}

/* nn.rs:130-152 query: q = scale * (Wq norm1(x) + bq), modulated per head by the query MLP */
static void query(const or_model *m, int l, const float *scale, const float *x, float *q, float *t, float *h64, float *mm) {
    const or_layer *b = &m->layer[l];
    int d = m->d, hd = d / m->heads;
    layer_norm(x, b->n1w, b->n1b, d, t);
    linear(b->wq, b->bq, t, d, d, q);
    for (int h = 0; h < m->heads; h++) {
        float *qh = q + h * hd;
        const float *sh = scale + h * hd;
        linear(b->q0w, b->q0b, qh, hd, m->hid, h64);
        gelu_inplace(h64, m->hid);
        linear(b->q2w, b->q2b, h64, m->hid, hd, mm);
        for (int i = 0; i < hd; i++) qh[i] *= sh[i] * (1.0f + or_tanh1(mm[i]));
    }
}

EXPORT void or_query(const or_model *m, int l, const float *scale, const float *x, float *q) {
    float *t = malloc(sizeof(float) * m->d), *h64 = malloc(sizeof(float) * m->hid), *mm = malloc(sizeof(float) * m->d);
    query(m, l, scale, x, q, t, h64, mm);
    free(t), free(h64), free(mm);
}

/* ---- nn.rs:166-287 Soft: the streaming softmax ------------------------------------------------------------- */

typedef struct {
    int heads, d;
    float *m, *s, *acc;
} soft;

static void soft_reset(soft *s) {
    for (int h = 0; h < s->heads; h++) s->m[h] = -INFINITY, s->s[h] = 0;
    memset(s->acc, 0, sizeof(float) * s->d);
}

/* rescale for a new running maximum (nn.rs:207-215) */
static void soft_top(soft *st, int h, int hd, float top) {
    if (top > st->m[h]) {
        if (st->s[h] > 0) {
            float f = or_exp1(st->m[h] - top);
            st->s[h] *= f;
            for (int i = 0; i < hd; i++) st->acc[h * hd + i] *= f;
        }
        st->m[h] = top;
    }
}

/* nn.rs:194-228 update_scaled for float keys/values (vs = NULL) */
static void soft_update_f32(soft *st, const float *q, const float *kt, const float *vt, int r, float *sc, float *tmp) {
    int hd = st->d / st->heads;
    for (int h = 0; h < st->heads; h++) {
        const float *k = kt + (size_t)h * hd * r, *v = vt + (size_t)h * hd * r;
        memset(sc, 0, sizeof(float) * r);
        weighted_sum(q + h * hd, k, hd, r, sc);
        soft_top(st, h, hd, vmax(sc, r));
        st->s[h] += exp_shift_sum(sc, r, st->m[h]);
        matvec(v, sc, r, hd, tmp);
        for (int i = 0; i < hd; i++) st->acc[h * hd + i] += tmp[i];
    }
}

/* nn.rs:233-258 update_int: q already multiplied by the keys' scales, vs the values' scales */
#define SOFT_UPDATE_INT(NAME, T, WS, MV)                                                                          \
    static void NAME(soft *st, const float *q, const T *kt, const T *vt, const float *vs, int r, float *sc,       \
                     float *tmp) {                                                                                \
        int hd = st->d / st->heads;                                                                               \
        for (int h = 0; h < st->heads; h++) {                                                                     \
            const T *k = kt + (size_t)h * hd * r, *v = vt + (size_t)h * hd * r;                                   \
            memset(sc, 0, sizeof(float) * r);                                                                     \
            WS(q + h * hd, k, hd, r, sc);                                                                         \
            soft_top(st, h, hd, vmax(sc, r));                                                                     \
            st->s[h] += exp_shift_sum(sc, r, st->m[h]);                                                           \
            MV(v, sc, r, hd, tmp);                                                                                \
            for (int i = 0; i < hd; i++) st->acc[h * hd + i] += tmp[i] * vs[h * hd + i];                          \
        }                                                                                                         \
    }
SOFT_UPDATE_INT(soft_update_i16, int16_t, weighted_sum_i16, matvec_i16)
SOFT_UPDATE_INT(soft_update_i8, int8_t, weighted_sum_i8, matvec_i8)

/* nn.rs:261-276 merge */
static void soft_merge(soft *a, const soft *o) {
    int hd = a->d / a->heads;
    for (int h = 0; h < a->heads; h++) {
        if (o->s[h] <= 0) continue;
        float top = a->m[h] > o->m[h] ? a->m[h] : o->m[h];
        float fa = a->s[h] > 0 ? or_exp1(a->m[h] - top) : 0.0f;
        float fb = or_exp1(o->m[h] - top);
        a->s[h] = a->s[h] * fa + o->s[h] * fb;
        for (int i = h * hd; i < (h + 1) * hd; i++) a->acc[i] = a->acc[i] * fa + o->acc[i] * fb;
        a->m[h] = top;
    }
}

/* nn.rs:280-286 finish */
static void soft_finish(soft *st) {
    int hd = st->d / st->heads;
    for (int h = 0; h < st->heads; h++) {
        float inv = 1.0f / st->s[h];
        for (int i = 0; i < hd; i++) st->acc[h * hd + i] *= inv;
    }
}

/* One stored chunk seen in place (predict.rs:459-480): feed it to a running softmax. `qs` is scratch for the
 * query times the keys' scales (predict.rs:486-497). */
static void soft_chunk(soft *st, int kv, const uint8_t *rec, int rc, const float *q, float *qs, float *sc, float *tmp) {
    int d = st->d;
    if (kv == 0) {
        const float *kt = (const float *)rec;
        soft_update_f32(st, q, kt, kt + (size_t)d * rc, rc, sc, tmp);
        return;
    }
    const float *scales = (const float *)rec;
    for (int i = 0; i < d; i++) qs[i] = q[i] * scales[i];
    const uint8_t *body = rec + (size_t)8 * d;
    if (kv == 1) {
        const int16_t *kt = (const int16_t *)body;
        soft_update_i16(st, qs, kt, kt + (size_t)d * rc, scales + d, rc, sc, tmp);
    } else {
        const int8_t *kt = (const int8_t *)body;
        soft_update_i8(st, qs, kt, kt + (size_t)d * rc, scales + d, rc, sc, tmp);
    }
}

/* Attention of one query against one layer's stored cache, chunks [c0, c1) (predict.rs:431-520 for one reader).
 * Leaves the running state unfinished so ranges can be merged (predict.rs:521-532). */
static void attend_range(soft *st, int kv, const uint8_t *layer, int rows, int chunk, int c0, int c1, const float *q,
                         float *qs, float *sc, float *tmp) {
    size_t full = or_record(kv, st->d, chunk);
    for (int ci = c0; ci < c1; ci++) {
        int rc = rows - ci * chunk < chunk ? rows - ci * chunk : chunk;
        soft_chunk(st, kv, layer + (size_t)ci * full, rc, q, qs, sc, tmp);
    }
}

/* AttendCached::attend semantics (predict.rs:63-66): attention outputs [n][d] for scaled queries [n][d] against
 * one layer of the cache, split over `parts` readers merged as key_threads does (predict.rs:398-409, 521-532). */
typedef struct {
    int kv, d, heads, rows, chunk, parts, n_chunks;
    const uint8_t *layer;
    const float *q;
    float *out;
} attend_job;

static void attend_one(void *ctx, int r) {
    const attend_job *j = (const attend_job *)ctx;
    int d = j->d, heads = j->heads;
    soft a, b;
    a.heads = b.heads = heads, a.d = b.d = d;
    a.m = malloc(sizeof(float) * heads), a.s = malloc(sizeof(float) * heads), a.acc = malloc(sizeof(float) * d);
    b.m = malloc(sizeof(float) * heads), b.s = malloc(sizeof(float) * heads), b.acc = malloc(sizeof(float) * d);
    float *qs = malloc(sizeof(float) * d), *sc = malloc(sizeof(float) * j->chunk), *tmp = malloc(sizeof(float) * d);
    soft_reset(&a);
    int per = (j->n_chunks + j->parts - 1) / j->parts;
    for (int p = 0; p < j->parts; p++) {
        int c0 = p * per, c1 = (p + 1) * per < j->n_chunks ? (p + 1) * per : j->n_chunks;
        if (c0 >= c1) continue;
        if (p == 0) {
            attend_range(&a, j->kv, j->layer, j->rows, j->chunk, c0, c1, j->q + (size_t)r * d, qs, sc, tmp);
        } else {
            soft_reset(&b);
            attend_range(&b, j->kv, j->layer, j->rows, j->chunk, c0, c1, j->q + (size_t)r * d, qs, sc, tmp);
            soft_merge(&a, &b);
        }
    }
    soft_finish(&a);
    memcpy(j->out + (size_t)r * d, a.acc, sizeof(float) * d);
    free(a.m), free(a.s), free(a.acc), free(b.m), free(b.s), free(b.acc), free(qs), free(sc), free(tmp);
}

EXPORT void or_attend(int kv, int d, int heads, const uint8_t *layer, int rows, int chunk, const float *q, int n,
                      int parts, float *out) {
    attend_job j;
    j.kv = kv, j.d = d, j.heads = heads, j.rows = rows, j.chunk = chunk, j.layer = layer, j.q = q, j.out = out;
    j.n_chunks = (rows + chunk - 1) / chunk;
    j.parts = parts < 1 ? 1 : (parts > j.n_chunks ? j.n_chunks : parts);
    par_for(n, attend_one, &j);
}

/* ---- predict.rs:381-586 in_context: the whole in-context stage ------------------------------------------- */

typedef struct {
    const or_model *m;
    int l;
    const float *scale, *att;
    float *h, *q, *logits;
    int out_n;
} rows_job;

/* nn.rs:130-152 for one row */
static void query_one(void *ctx, int r) {
    const rows_job *j = (const rows_job *)ctx;
    const or_model *m = j->m;
    float *t = malloc(sizeof(float) * m->d), *h64 = malloc(sizeof(float) * m->hid), *mm = malloc(sizeof(float) * m->d);
    query(m, j->l, j->scale, j->h + (size_t)r * m->d, j->q + (size_t)r * m->d, t, h64, mm);
    free(t), free(h64), free(mm);
}

/* predict.rs:542-568 for one row: out-projection and residual, then feed-forward and residual */
static void tail_one(void *ctx, int r) {
    const rows_job *j = (const rows_job *)ctx;
    const or_model *m = j->m;
    const or_layer *b = &m->layer[j->l];
    int d = m->d, ff = m->ff;
    float *hr = j->h + (size_t)r * d;
    float *t = malloc(sizeof(float) * (d > ff ? d : ff)), *mid = malloc(sizeof(float) * ff);
    linear(b->wo, b->bo, j->att + (size_t)r * d, d, d, t);
    for (int i = 0; i < d; i++) hr[i] += t[i];
    layer_norm(hr, b->n2w, b->n2b, d, t);
    linear(b->w1, b->b1, t, d, ff, mid);
    gelu_inplace(mid, ff);
    linear(b->w2, b->b2, mid, ff, d, t);
    for (int i = 0; i < d; i++) hr[i] += t[i];
    free(t), free(mid);
}

/* predict.rs:570-584 decoder for one row */
static void decode_one(void *ctx, int r) {
    const rows_job *j = (const rows_job *)ctx;
    const or_model *m = j->m;
    int d = m->d, dff = m->dff;
    float *t = malloc(sizeof(float) * d), *hid = malloc(sizeof(float) * dff), *all = malloc(sizeof(float) * m->outs);
    layer_norm(j->h + (size_t)r * d, m->lnw, m->lnb, d, t);
    linear(m->dec0w, m->dec0b, t, d, dff, hid);
    gelu_inplace(hid, dff);
    linear(m->dec2w, m->dec2b, hid, dff, m->outs, all);
    memcpy(j->logits + (size_t)r * j->out_n, all, sizeof(float) * j->out_n);
    free(t), free(hid), free(all);
}

/* Row representations h [n][d] (consumed) to the first `out_n` decoder outputs per row. `layers[l]` is the
 * stored n{node}_kv{l} tensor, `scales` the stored n{node}_scale [L][d]. `parts` > 1 splits the training rows as
 * key_threads does. */
EXPORT void or_in_context(const or_model *m, int kv, const uint8_t *const *layers, const float *scales, int rows,
                          int chunk, float *h, int n, int out_n, int parts, float *logits) {
    int d = m->d;
    float *q = malloc(sizeof(float) * (size_t)n * d);
    float *att = malloc(sizeof(float) * (size_t)n * d);
    rows_job j;
    j.m = m, j.h = h, j.q = q, j.att = att, j.logits = logits, j.out_n = out_n;
    for (int l = 0; l < m->layers; l++) {
        j.l = l, j.scale = scales + (size_t)l * d;
        par_for(n, query_one, &j);
        or_attend(kv, d, m->heads, layers[l], rows, chunk, q, n, parts, att);
        par_for(n, tail_one, &j);
    }
    par_for(n, decode_one, &j);
    free(q), free(att);
}

/* ---- fit.rs:549-576 pack: one chunk of keys and values in its stored form --------------------------------- */

static inline int16_t sat_i16(float v) {
    if (v != v) return 0; /* Rust `as` maps NaN to 0 and saturates */
    if (v >= 32767.0f) return 32767;
    if (v <= -32768.0f) return -32768;
    return (int16_t)v;
}
static inline int8_t sat_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}

/* `c` is [2d][rc] floats (keys then values, dimension-major); writes or_record(kv, d, rc) bytes. */
EXPORT void or_pack(int kv, int d, int rc, const float *c, uint8_t *rec) {
    if (kv == 0) {
        memcpy(rec, c, sizeof(float) * 2 * (size_t)d * rc);
        return;
    }
    float top = kv == 1 ? 32767.0f : 127.0f;
    float *scales = (float *)malloc(sizeof(float) * 2 * d);
    uint8_t *body = rec + (size_t)8 * d;
    for (int j = 0; j < 2 * d; j++) {
        const float *row = c + (size_t)j * rc;
        float big = 0.0f;
        for (int i = 0; i < rc; i++) {
            float a = fabsf(row[i]);
            big = a > big ? a : big; /* f32::max ignores NaN */
        }
        float s = big > 0.0f ? big / top : 1.0f;
        scales[j] = s;
        float inv = 1.0f / s;
        if (kv == 1) {
            int16_t *o = (int16_t *)(body + (size_t)2 * j * rc);
            for (int i = 0; i < rc; i++) o[i] = sat_i16(roundf(row[i] * inv));
        } else {
            int8_t *o = (int8_t *)(body + (size_t)j * rc);
            for (int i = 0; i < rc; i++) o[i] = sat_i8(roundf(row[i] * inv));
        }
    }
    memcpy(rec, scales, sizeof(float) * 2 * d);
    free(scales);
}

/* predict.rs:590-629 layer_rows: one layer's cache widened to floats, row by row: k, v [rows][d] */
EXPORT void or_layer_rows(int kv, int d, const uint8_t *layer, int rows, int chunk, float *k, float *v) {
    size_t full = or_record(kv, d, chunk);
    for (int ci = 0, r0 = 0; r0 < rows; ci++, r0 += chunk) {
        int rc = rows - r0 < chunk ? rows - r0 : chunk;
        const uint8_t *rec = layer + (size_t)ci * full;
        for (int j = 0; j < 2 * d; j++)
            for (int r = 0; r < rc; r++) {
                size_t i = (size_t)j * rc + r;
                float val;
                if (kv == 0)
                    val = ((const float *)rec)[i];
                else {
                    const float *sc = (const float *)rec;
                    const uint8_t *body = rec + (size_t)8 * d;
                    float in = kv == 1 ? (float)((const int16_t *)body)[i] : (float)((const int8_t *)body)[i];
                    val = in * sc[j];
                }
                if (j < d)
                    k[(size_t)(r0 + r) * d + j] = val;
                else
                    v[(size_t)(r0 + r) * d + j - d] = val;
            }
    }
}

/* ---- fit.rs:577-747: the in-context stage of fitting (the producer of the cache) ------------------------- */

/* model.rs:185-200 add_y */
EXPORT void or_add_y(const or_model *m, const float *y, int n, float *h) {
    int d = m->d;
    for (int r = 0; r < n; r++) {
        float *cell = h + (size_t)r * d;
        if (m->max_classes > 0) {
            const float *row = m->icl_y + (size_t)((int)y[r]) * d;
            for (int i = 0; i < d; i++) cell[i] += row[i];
        } else {
            for (int i = 0; i < d; i++) cell[i] += m->icl_y[i] * y[r] + m->icl_y[d + i];
        }
    }
}

typedef struct {
    const or_model *m;
    const or_layer *b;
    const float *h;
    float *kvf;
    uint8_t *out;
    int rows, chunk, kv;
    size_t full;
} kv_job;

/* fit.rs:633-653 for one chunk: keys and values of its rows, dimension-major, then packed */
static void kv_chunk(void *ctx, int ci) {
    const kv_job *j = (const kv_job *)ctx;
    int d = j->m->d, r0 = ci * j->chunk, rc = j->rows - r0 < j->chunk ? j->rows - r0 : j->chunk;
    float *kt = j->kvf + 2 * (size_t)d * r0, *vt = kt + (size_t)d * rc;
    float *t = malloc(sizeof(float) * d), *two = malloc(sizeof(float) * 2 * d);
    for (int r = 0; r < rc; r++) {
        layer_norm(j->h + (size_t)(r0 + r) * d, j->b->n1w, j->b->n1b, d, t);
        linear(j->b->wkv, j->b->bkv, t, d, 2 * d, two);
        for (int c = 0; c < d; c++) kt[(size_t)c * rc + r] = two[c], vt[(size_t)c * rc + r] = two[d + c];
    }
    or_pack(j->kv, d, rc, kt, j->out + (size_t)ci * j->full);
    free(t), free(two);
}

/* Training rows h [rows][d] (target embedding already added, consumed) to every layer's stored keys and values
 * (`out[l]` receives the whole n{j}_kv{l} tensor) and the query scales [L][d] (n{j}_scale). The in-memory
 * path of fit.rs:627-745: keys/values of each chunk packed as written, the layer's attention over the exact
 * float keys/values. */
EXPORT void or_icl_fit(const or_model *m, float *h, int rows, int chunk, int kv, uint8_t *const *out, float *scales) {
    int d = m->d;
    float *kvf = malloc(sizeof(float) * 2 * (size_t)rows * d); /* chunks of [K: d][rc], [V: d][rc], f32 */
    float *qall = malloc(sizeof(float) * (size_t)rows * d);
    float *att = malloc(sizeof(float) * (size_t)rows * d);
    kv_job kj;
    kj.m = m, kj.h = h, kj.kvf = kvf, kj.rows = rows, kj.chunk = chunk, kj.kv = kv, kj.full = or_record(kv, d, chunk);
    rows_job rj;
    rj.m = m, rj.h = h, rj.q = qall, rj.att = att, rj.logits = NULL, rj.out_n = 0;
    for (int l = 0; l < m->layers; l++) {
        float *scale = scales + (size_t)l * d;
        or_query_scale(m, l, rows, scale);
        kj.b = &m->layer[l], kj.out = out[l];
        par_for((rows + chunk - 1) / chunk, kv_chunk, &kj);
        if (l + 1 == m->layers) break;
        rj.l = l, rj.scale = scale;
        par_for(rows, query_one, &rj);
        or_attend(0, d, m->heads, (const uint8_t *)kvf, rows, chunk, qall, rows, 1, att);
        par_for(rows, tail_one, &rj);
    }
    free(kvf), free(qall), free(att);
}

/* ---- table.rs heads ------------------------------------------------------------------------------------------ */

/* table.rs:265-269: add one member's logits (in its relabelled class order) to the sums, in f64 */
EXPORT void or_add_member(double *sums, const float *logits, int n, int classes, int stride, const int32_t *member_classes) {
    for (int r = 0; r < n; r++)
        for (int c = 0; c < classes; c++) sums[(size_t)r * classes + c] += (double)logits[(size_t)r * stride + member_classes[c]];
}

/* table.rs:70-78 finish_proba */
EXPORT void or_finish_proba(double *sums, int n, int classes, int members, double temperature) {
    double inv = 1.0 / ((double)members * temperature);
    for (int r = 0; r < n; r++) {
        double *row = sums + (size_t)r * classes;
        double top = -1.7976931348623157e308;
        for (int c = 0; c < classes; c++) top = row[c] > top ? row[c] : top;
        double sum = 0;
        for (int c = 0; c < classes; c++) row[c] = exp((row[c] - top) * inv);
        for (int c = 0; c < classes; c++) sum += row[c];
        for (int c = 0; c < classes; c++) row[c] /= sum;
    }
}

/* f32 total order key (f32::total_cmp) */
static inline uint32_t total_key(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
static int cmp_total(const void *a, const void *b) {
    uint32_t x = total_key(*(const float *)a), y = total_key(*(const float *)b);
    return x < y ? -1 : x > y;
}

typedef struct {
    float *q, *levels;
    int n;
    float tl0, tl1, tr0, tr1;
} qdist;

/* table.rs:300-317 QuantileDist::new */
static void qdist_new(qdist *dd, float *q, float *levels, int n) {
    qsort(q, n, sizeof(float), cmp_total);
    for (int i = 0; i < n; i++) levels[i] = (float)(i + 1) / (float)(n + 1);
    int k = n / 4 < 20 ? n / 4 : 20;
    if (k < 1) k = 1;
    float ln_l[20], ln_r[20];
    for (int i = 0; i < k; i++) {
        float a = levels[i] > 1e-6f ? levels[i] : 1e-6f;
        ln_l[i] = logf(a);
        float b = 1.0f - levels[n - k + i];
        ln_r[i] = logf(b > 1e-6f ? b : 1e-6f);
    }
    float sl[2];
    for (int side = 0; side < 2; side++) {
        const float *xs = side == 0 ? ln_l : ln_r, *ys = side == 0 ? q : q + n - k;
        float sx = 0, sy = 0;
        for (int i = 0; i < k; i++) sx += xs[i];
        for (int i = 0; i < k; i++) sy += ys[i];
        float mx = sx / (float)k, my = sy / (float)k;
        float cov = 0, var = 0;
        for (int i = 0; i < k; i++) cov += (xs[i] - mx) * (ys[i] - my);
        cov /= (float)k;
        for (int i = 0; i < k; i++) var += (xs[i] - mx) * (xs[i] - mx);
        var /= (float)k;
        float s = fabsf(cov / (var > 1e-6f ? var : 1e-6f));
        sl[side] = clampf(s, 0.01f, 100.0f);
    }
    float bl = sl[0], br = sl[1];
    dd->q = q, dd->levels = levels, dd->n = n;
    dd->tl0 = bl;
    dd->tl1 = q[0] - bl * logf(levels[0] > 1e-6f ? levels[0] : 1e-6f);
    dd->tr0 = -br;
    float lr = levels[n - 1] < 1.0f - 1e-6f ? levels[n - 1] : 1.0f - 1e-6f;
    dd->tr1 = q[n - 1] + br * logf(1.0f - lr);
}

/* table.rs:319-345 */
static float qdist_mean(const qdist *dd) {
    float s = 0;
    for (int i = 0; i < dd->n; i++) s += dd->q[i];
    return s / (float)dd->n;
}
static float qdist_variance(const qdist *dd) {
    float m = qdist_mean(dd), s = 0;
    for (int i = 0; i < dd->n; i++) s += (dd->q[i] - m) * (dd->q[i] - m);
    return s / (float)(dd->n - 1);
}
static float qdist_icdf(const qdist *dd, float alpha) {
    int n = dd->n;
    if (alpha < dd->levels[0]) return dd->tl0 * logf(alpha > 1e-6f ? alpha : 1e-6f) + dd->tl1;
    if (alpha > dd->levels[n - 1]) {
        float b = 1.0f - alpha;
        return dd->tr0 * logf(b > 1e-6f ? b : 1e-6f) + dd->tr1;
    }
    if (alpha >= dd->levels[n - 1]) return dd->q[n - 1];
    int pp = 0; /* partition_point over levels[..n-1] of (l <= alpha) */
    while (pp < n - 1 && dd->levels[pp] <= alpha) pp++;
    int i = pp > 0 ? pp - 1 : 0;
    if (i > n - 2) i = n - 2;
    float den = dd->levels[i + 1] - dd->levels[i];
    float t = (alpha - dd->levels[i]) / (den > 1e-6f ? den : 1e-6f);
    t = clampf(t, 0.0f, 1.0f);
    return dd->q[i] + t * (dd->q[i + 1] - dd->q[i]);
}

typedef struct {
    const float *qout;
    int nq, stride, na;
    const double *alphas;
    double tmean, tscale, *mean, *variance, *median, *quantiles;
} reg_job;

static void reg_one(void *ctx, int r) {
    const reg_job *j = (const reg_job *)ctx;
    float *q = malloc(sizeof(float) * j->nq), *lv = malloc(sizeof(float) * j->nq);
    memcpy(q, j->qout + (size_t)r * j->stride, sizeof(float) * j->nq);
    qdist dd;
    qdist_new(&dd, q, lv, j->nq);
#define BACK(v) ((double)(v) * j->tscale + j->tmean)
    j->mean[r] += BACK(qdist_mean(&dd));
    j->variance[r] += BACK(qdist_variance(&dd));
    j->median[r] += BACK(qdist_icdf(&dd, 0.5f));
    for (int a = 0; a < j->na; a++) j->quantiles[(size_t)r * j->na + a] += BACK(qdist_icdf(&dd, (float)j->alphas[a]));
#undef BACK
    free(q), free(lv);
}

/* table.rs:457-496 (one member's share): quantile outputs [n][nq] to mean, variance, median and the quantiles at
 * `alphas`, back-transformed (v * scale + mean) and added to the f64 outputs; the caller divides by the member
 * count at the end (table.rs:491-494). */
EXPORT void or_regression_add(const float *qout, int n, int nq, int stride, const double *alphas, int na,
                              double target_mean, double target_scale, double *mean, double *variance,
                              double *median, double *quantiles) {
    reg_job j;
    j.qout = qout, j.nq = nq, j.stride = stride, j.na = na, j.alphas = alphas, j.tmean = target_mean;
    j.tscale = target_scale, j.mean = mean, j.variance = variance, j.median = median, j.quantiles = quantiles;
    par_for(n, reg_one, &j);
}

/* ---- the column and row stages of prediction (predict.rs:282-372, nn.rs:291-419) --------------------------- */

/* One pre-norm block of the column or row stage (model.rs:27-98 Block): in_w is [3e][e] (the query's rows first),
 * no scalable softmax (the column stage's second attention and the row blocks have none). */
typedef struct {
    const float *n1w, *n1b, *inw, *inb, *ow, *ob, *n2w, *n2b, *w1, *b1, *w2, *b2;
    int ff;
} or_cblock;

/* A column block's first attention (multihead_attn1: the inducing points over a column's training cells) with its
 * scalable softmax (base_mlp for the length term, query_mlp per head) and the inducing points; fit only. */
typedef struct {
    or_cblock b;
    const float *sb0w, *sb0b, *sb2w, *sb2b, *q0w, *q0b, *q2w, *q2b;
    int hid;
    const float *ind; /* [inds][e] */
} or_isab1;

typedef struct {
    int e, group, inds, cls, col_heads, row_heads, ncol, nrow;
    const float *in_w, *in_b;         /* col_embedder.in_linear: [e][group], [e] */
    const or_cblock *col;             /* the column blocks' second attention (multihead_attn2), ncol */
    const float *cls_tokens;          /* [cls][e] */
    const or_cblock *row;             /* nrow */
    const float *rope_freqs;          /* [row head width / 2] */
    const float *out_lnw, *out_lnb;   /* row_interactor.out_ln: [e] */
    const or_isab1 *col1;             /* fit: the column blocks' first attention, ncol (NULL for prediction) */
    const float *col_y;               /* fit: the label's embedding table (model.rs:163-177) */
    int max_classes;
} or_rows_model;

/* nn.rs:156-164 feed_forward: x += l2(gelu(l1(norm2 x))); t [e], h [ff] scratch */
static void feed_forward_c(const or_cblock *b, int e, float *x, float *t, float *h) {
    layer_norm(x, b->n2w, b->n2b, e, t);
    linear(b->w1, b->b1, t, e, b->ff, h);
    gelu_inplace(h, b->ff);
    linear(b->w2, b->b2, h, b->ff, e, t);
    for (int i = 0; i < e; i++) x[i] += t[i];
}

/* nn.rs:289-302 cached_block: x against n fixed keys/values kt, vt ([e][n]), queries scaled by `scale` (no
 * scalable softmax: nn.rs:136-141), then out-projection, residual and feed-forward. */
static void cached_block(const or_cblock *b, int e, int heads, const float *scale, const float *kt, const float *vt, int n,
                         float *x, float *t, float *q, float *h, float *sc, float *tmp, soft *st) {
    layer_norm(x, b->n1w, b->n1b, e, t);
    linear(b->inw, b->inb, t, e, e, q);
    for (int i = 0; i < e; i++) q[i] *= scale[i];
    soft_reset(st);
    soft_update_f32(st, q, kt, vt, n, sc, tmp);
    soft_finish(st);
    linear(b->ow, b->ob, st->acc, e, e, t);
    for (int i = 0; i < e; i++) x[i] += t[i];
    feed_forward_c(b, e, x, t, h);
}

/* nn.rs:422-429 group_values: the features one, two, four, ... places to the right of g, wrapping round */
static void group_values(const float *row, int feats, int g, int size, float *out) {
    for (int i = 0; i < size; i++) out[i] = row[(g + (1 << i)) % feats];
}

typedef struct {
    const or_rows_model *m;
    const float *x, *col_kv;
    int feats, digits;
    float *tok;
} embed_job;

static void embed_one(void *ctx, int r) {
    const embed_job *j = (const embed_job *)ctx;
    const or_rows_model *m = j->m;
    const int e = m->e, inds = m->inds, nb = m->ncol, tokens = m->cls + j->feats, hd = e / m->col_heads;
    int ffmax = 0;
    for (int b = 0; b < nb; b++) ffmax = m->col[b].ff > ffmax ? m->col[b].ff : ffmax;
    float *tok = j->tok + (size_t)r * tokens * e;
    memcpy(tok, m->cls_tokens, sizeof(float) * m->cls * e);
    float *scale = malloc(sizeof(float) * e), *t = malloc(sizeof(float) * e), *q = malloc(sizeof(float) * e);
    float *h = malloc(sizeof(float) * ffmax), *sc = malloc(sizeof(float) * inds), *tmp = malloc(sizeof(float) * hd);
    float *plain = malloc(sizeof(float) * e), *sum = malloc(sizeof(float) * e), *one = malloc(sizeof(float) * e);
    float vals[8];
    soft st;
    st.heads = m->col_heads, st.d = e;
    st.m = malloc(sizeof(float) * m->col_heads), st.s = malloc(sizeof(float) * m->col_heads), st.acc = malloc(sizeof(float) * e);
    for (int i = 0; i < e; i++) scale[i] = 1.0f / sqrtf((float)hd);
    const size_t per = (size_t)2 * e * inds, rec = (size_t)j->digits * nb * per;
    for (int g = 0; g < j->feats; g++) {
        float *cell = tok + (size_t)(m->cls + g) * e;
        group_values(j->x + (size_t)r * j->feats, j->feats, g, m->group, vals);
        int missing = 1;
        for (int i = 0; i < m->group; i++) missing &= vals[i] == -100.0f;
        if (missing)
            for (int i = 0; i < e; i++) cell[i] = -100.0f;
        else
            linear(m->in_w, m->in_b, vals, m->group, e, cell);
        const float *recs = j->col_kv + (size_t)g * rec;
        if (j->digits == 1) {
            for (int b = 0; b < nb; b++)
                cached_block(&m->col[b], e, m->col_heads, scale, recs + b * per, recs + b * per + (size_t)e * inds, inds, cell,
                             t, q, h, sc, tmp, &st);
        } else {
            /* once per label digit, then the average (predict.rs:326-346) */
            memcpy(plain, cell, sizeof(float) * e);
            memset(sum, 0, sizeof(float) * e);
            for (int dg = 0; dg < j->digits; dg++) {
                memcpy(one, plain, sizeof(float) * e);
                for (int b = 0; b < nb; b++) {
                    const float *at = recs + (size_t)(dg * nb + b) * per;
                    cached_block(&m->col[b], e, m->col_heads, scale, at, at + (size_t)e * inds, inds, one, t, q, h, sc, tmp, &st);
                }
                for (int i = 0; i < e; i++) sum[i] += one[i];
            }
            for (int i = 0; i < e; i++) cell[i] = sum[i] / (float)j->digits;
        }
    }
    free(scale), free(t), free(q), free(h), free(sc), free(tmp), free(plain), free(sum), free(one);
    free(st.m), free(st.s), free(st.acc);
}

/* predict.rs:282-353 embed: test rows x [n][feats] (normalised, missing cells -100) to their tokens
 * [n][cls + feats][e], class tokens first; col_kv as fit.rs:230 stores it: [feats][digits][blocks][2][e][inds]. */
EXPORT void or_embed(const or_rows_model *m, const float *x, int n, int feats, const float *col_kv, int digits, float *tok) {
    embed_job j;
    j.m = m, j.x = x, j.col_kv = col_kv, j.feats = feats, j.digits = digits, j.tok = tok;
    par_for(n, embed_one, &j);
}

typedef struct {
    const or_rows_model *m;
    float *tok, *rep;
    int tokens;
    const float *cosv, *sinv;
} represent_job;

/* nn.rs:357-419 row_forward for one row */
static void represent_one(void *ctx, int r) {
    const represent_job *jb = (const represent_job *)ctx;
    const or_rows_model *m = jb->m;
    const int d = m->e, heads = m->row_heads, hd = d / heads, half = hd / 2, tokens = jb->tokens;
    const float inv = 1.0f / sqrtf((float)hd);
    int ffmax = 0;
    for (int b = 0; b < m->nrow; b++) ffmax = m->row[b].ff > ffmax ? m->row[b].ff : ffmax;
    float *tok = jb->tok + (size_t)r * tokens * d, *out = jb->rep + (size_t)r * m->cls * d;
    float *tn = malloc(sizeof(float) * d), *qkv = malloc(sizeof(float) * 3 * d);
    float *q = malloc(sizeof(float) * tokens * d), *kt = malloc(sizeof(float) * tokens * d), *vt = malloc(sizeof(float) * tokens * d);
    float *nw = malloc(sizeof(float) * tokens * d), *sc = malloc(sizeof(float) * tokens), *att = malloc(sizeof(float) * d);
    float *tmp = malloc(sizeof(float) * hd), *h = malloc(sizeof(float) * ffmax);
    for (int bi = 0; bi < m->nrow; bi++) {
        const or_cblock *b = &m->row[bi];
        const int nq = bi == m->nrow - 1 ? m->cls : tokens;
        for (int t = 0; t < tokens; t++) {
            layer_norm(tok + (size_t)t * d, b->n1w, b->n1b, d, tn);
            if (t < nq)
                linear(b->inw, b->inb, tn, d, 3 * d, qkv);
            else
                linear(b->inw + (size_t)d * d, b->inb + d, tn, d, 2 * d, qkv + d);
            const float *cs = jb->cosv + (size_t)t * half, *sn = jb->sinv + (size_t)t * half;
            for (int hh = 0; hh < heads; hh++) {
                if (t < nq) {
                    const float *src = qkv + hh * hd;
                    float *dst = q + (size_t)t * d + hh * hd;
                    for (int i = 0; i < half; i++) {
                        const float a = src[i], c = src[i + half];
                        dst[i] = (a * cs[i] - c * sn[i]) * inv;
                        dst[i + half] = (c * cs[i] + a * sn[i]) * inv;
                    }
                }
                const float *src = qkv + d + hh * hd;
                for (int i = 0; i < half; i++) {
                    const float a = src[i], c = src[i + half];
                    kt[(size_t)(hh * hd + i) * tokens + t] = a * cs[i] - c * sn[i];
                    kt[(size_t)(hh * hd + i + half) * tokens + t] = c * cs[i] + a * sn[i];
                }
            }
            for (int jj = 0; jj < d; jj++) vt[(size_t)jj * tokens + t] = qkv[2 * d + jj];
        }
        for (int t = 0; t < nq; t++) {
            for (int hh = 0; hh < heads; hh++) {
                const float *ks = kt + (size_t)hh * hd * tokens, *vs = vt + (size_t)hh * hd * tokens;
                memset(sc, 0, sizeof(float) * tokens);
                weighted_sum(q + (size_t)t * d + hh * hd, ks, hd, tokens, sc);
                const float top = vmax(sc, tokens);
                const float s = 1.0f / exp_shift_sum(sc, tokens, top);
                matvec(vs, sc, tokens, hd, tmp);
                for (int i = 0; i < hd; i++) att[hh * hd + i] = tmp[i] * s;
            }
            float *x = nw + (size_t)t * d;
            linear(b->ow, b->ob, att, d, d, x);
            for (int i = 0; i < d; i++) x[i] += tok[(size_t)t * d + i];
            feed_forward_c(b, d, x, tn, h);
        }
        memcpy(tok, nw, sizeof(float) * (size_t)nq * d);
    }
    for (int c = 0; c < m->cls; c++) layer_norm(tok + (size_t)c * d, m->out_lnw, m->out_lnb, d, out + (size_t)c * d);
    free(tn), free(qkv), free(q), free(kt), free(vt), free(nw), free(sc), free(att), free(tmp), free(h);
}

/* predict.rs:356-372 represent: tokens [n][tokens][e] (consumed) to row representations [n][cls e]; the rotary
 * tables of nn.rs:304-321 (cos and sin of position times frequency, in f32). */
EXPORT void or_represent(const or_rows_model *m, float *tok, int n, int tokens, float *rep) {
    const int half = m->e / m->row_heads / 2;
    float *cosv = malloc(sizeof(float) * tokens * half), *sinv = malloc(sizeof(float) * tokens * half);
    for (int p = 0; p < tokens; p++)
        for (int i = 0; i < half; i++) {
            const float a = (float)p * m->rope_freqs[i];
            cosv[p * half + i] = cosf(a), sinv[p * half + i] = sinf(a);
        }
    represent_job j;
    j.m = m, j.tok = tok, j.rep = rep, j.tokens = tokens, j.cosv = cosv, j.sinv = sinv;
    par_for(n, represent_one, &j);
    free(cosv), free(sinv);
}


/* ---- fit.rs:298-420: the column stage of fitting ------------------------------------------------------------- */

/* nn.rs:97-107 query_scale for the column stage's first attention: the scalable softmax's length term for n rows,
 * times 1/sqrt(head width) */
static void query_scale_c(const or_isab1 *a, int e, int heads, int n, float *out) {
    const float inv = 1.0f / sqrtf((float)(e / heads));
    const float logn = logf((float)(n > 1 ? n : 1));
    float *h = malloc(sizeof(float) * a->hid);
    for (int i = 0; i < a->hid; i++) h[i] = a->sb0w[i] * logn + a->sb0b[i];
    gelu_inplace(h, a->hid);
    linear(a->sb2w, a->sb2b, h, a->hid, e, out);
    for (int i = 0; i < e; i++) out[i] *= inv;
    free(h);
}

/* nn.rs:130-152 query with the first attention's weights (its in_proj's query rows) */
static void query_c(const or_isab1 *a, int e, int heads, const float *scale, const float *x, float *q) {
    const int hd = e / heads;
    float *t = malloc(sizeof(float) * e), *h = malloc(sizeof(float) * a->hid), *mm = malloc(sizeof(float) * hd);
    layer_norm(x, a->b.n1w, a->b.n1b, e, t);
    linear(a->b.inw, a->b.inb, t, e, e, q);
    for (int hh = 0; hh < heads; hh++) {
        float *qh = q + hh * hd;
        linear(a->q0w, a->q0b, qh, hd, a->hid, h);
        gelu_inplace(h, a->hid);
        linear(a->q2w, a->q2b, h, a->hid, hd, mm);
        for (int i = 0; i < hd; i++) qh[i] *= scale[hh * hd + i] * (1.0f + or_tanh1(mm[i]));
    }
    free(t), free(h), free(mm);
}

/* model.rs:186-200 add_y: the embedding of target y added to a cell (a class's row of the table; for a regression
 * model, weight times y plus bias) */
static void add_y_c(const float *table, int max_classes, int w, float y, float *cell) {
    if (max_classes > 0) {
        const float *row = table + (size_t)y * w;
        for (int i = 0; i < w; i++) cell[i] += row[i];
    } else {
        for (int i = 0; i < w; i++) cell[i] += table[i] * y + table[w + i];
    }
}

typedef struct {
    const or_rows_model *m;
    const float *x, *y, *ind_q; /* ind_q [ncol][inds][e] */
    const int *bases;
    int n, feats, chunk, digits;
    float *col_kv, *tok;
} fitcol_job;

/* fit.rs:326-420 col_one: one feature group's training cells through the column blocks, its cache written */
static void fitcol_one(void *ctx, int g) {
    const fitcol_job *j = (const fitcol_job *)ctx;
    const or_rows_model *m = j->m;
    const int e = m->e, inds = m->inds, nb = m->ncol, n = j->n, heads = m->col_heads, hd = e / heads, D = j->digits;
    const int chunk = j->chunk < n ? j->chunk : n, tokens = m->cls + j->feats;
    int ffmax = 0;
    for (int b = 0; b < nb; b++) {
        ffmax = m->col[b].ff > ffmax ? m->col[b].ff : ffmax;
        ffmax = m->col1[b].b.ff > ffmax ? m->col1[b].b.ff : ffmax;
    }
    float *src = malloc(sizeof(float) * (size_t)n * e), *plain = NULL, *sum = NULL;
    if (D > 1) plain = malloc(sizeof(float) * (size_t)n * e), sum = calloc((size_t)n * e, sizeof(float));
    float *kt = malloc(sizeof(float) * (size_t)e * chunk), *vt = malloc(sizeof(float) * (size_t)e * chunk);
    float *kv = malloc(sizeof(float) * 2 * e), *t = malloc(sizeof(float) * e), *hidden = malloc(sizeof(float) * (size_t)inds * e);
    float *q = malloc(sizeof(float) * e), *h = malloc(sizeof(float) * ffmax), *tmp = malloc(sizeof(float) * hd);
    float *sc = malloc(sizeof(float) * (chunk > inds ? chunk : inds)), *scale2 = malloc(sizeof(float) * e);
    soft *softs = malloc(sizeof(soft) * inds);
    for (int i = 0; i < inds; i++) {
        softs[i].heads = heads, softs[i].d = e;
        softs[i].m = malloc(sizeof(float) * heads), softs[i].s = malloc(sizeof(float) * heads), softs[i].acc = malloc(sizeof(float) * e);
    }
    soft st;
    st.heads = heads, st.d = e;
    st.m = malloc(sizeof(float) * heads), st.s = malloc(sizeof(float) * heads), st.acc = malloc(sizeof(float) * e);
    for (int i = 0; i < e; i++) scale2[i] = 1.0f / sqrtf((float)hd);
    float vals[8];
    for (int r = 0; r < n; r++) {
        float *cell = src + (size_t)r * e;
        group_values(j->x + (size_t)r * j->feats, j->feats, g, m->group, vals);
        int missing = 1;
        for (int i = 0; i < m->group; i++) missing &= vals[i] == -100.0f;
        if (missing)
            for (int i = 0; i < e; i++) cell[i] = -100.0f;
        else
            linear(m->in_w, m->in_b, vals, m->group, e, cell);
    }
    if (D > 1) memcpy(plain, src, sizeof(float) * (size_t)n * e);
    const size_t per = (size_t)2 * e * inds;
    for (int dg = 0; dg < D; dg++) {
        if (dg > 0) memcpy(src, plain, sizeof(float) * (size_t)n * e);
        int divisor = 1;
        for (int b = dg + 1; b < D; b++) divisor *= j->bases[b];
        for (int r = 0; r < n; r++) {
            const float yv = D > 1 ? (float)(((int)j->y[r] / divisor) % j->bases[dg]) : j->y[r];
            add_y_c(m->col_y, m->max_classes, e, yv, src + (size_t)r * e);
        }
        float *rec = j->col_kv + (size_t)g * D * nb * per + (size_t)dg * nb * per;
        for (int bi = 0; bi < nb; bi++) {
            const or_isab1 *a1 = &m->col1[bi];
            /* the inducing points look at this column's training cells, a chunk of rows at a time */
            for (int i = 0; i < inds; i++) soft_reset(&softs[i]);
            for (int r0 = 0; r0 < n; r0 += chunk) {
                const int rc = chunk < n - r0 ? chunk : n - r0;
                for (int r = 0; r < rc; r++) {
                    layer_norm(src + (size_t)(r0 + r) * e, a1->b.n1w, a1->b.n1b, e, t);
                    linear(a1->b.inw + (size_t)e * e, a1->b.inb + e, t, e, 2 * e, kv);
                    for (int c = 0; c < e; c++) kt[(size_t)c * rc + r] = kv[c], vt[(size_t)c * rc + r] = kv[e + c];
                }
                for (int i = 0; i < inds; i++)
                    soft_update_f32(&softs[i], j->ind_q + ((size_t)bi * inds + i) * e, kt, vt, rc, sc, tmp);
            }
            for (int i = 0; i < inds; i++) {
                soft_finish(&softs[i]);
                float *hid = hidden + (size_t)i * e;
                linear(a1->b.ow, a1->b.ob, softs[i].acc, e, e, hid);
                for (int c = 0; c < e; c++) hid[c] += a1->ind[(size_t)i * e + c];
                feed_forward_c(&a1->b, e, hid, t, h);
            }
            /* their keys and values for the second attention: what prediction reuses */
            const or_cblock *a2 = &m->col[bi];
            float *rk = rec + (size_t)bi * per, *rv = rk + (size_t)e * inds;
            for (int i = 0; i < inds; i++) {
                layer_norm(hidden + (size_t)i * e, a2->n1w, a2->n1b, e, t);
                linear(a2->inw + (size_t)e * e, a2->inb + e, t, e, 2 * e, kv);
                for (int c = 0; c < e; c++) rk[(size_t)c * inds + i] = kv[c], rv[(size_t)c * inds + i] = kv[e + c];
            }
            for (int r = 0; r < n; r++) cached_block(a2, e, heads, scale2, rk, rv, inds, src + (size_t)r * e, t, q, h, sc, tmp, &st);
        }
        if (D > 1)
            for (size_t i = 0; i < (size_t)n * e; i++) sum[i] += src[i];
    }
    if (D > 1) {
        const float inv = 1.0f / (float)D;
        for (size_t i = 0; i < (size_t)n * e; i++) src[i] = sum[i] * inv;
    }
    for (int r = 0; r < n; r++) memcpy(j->tok + ((size_t)r * tokens + m->cls + g) * e, src + (size_t)r * e, sizeof(float) * e);
    for (int i = 0; i < inds; i++) free(softs[i].m), free(softs[i].s), free(softs[i].acc);
    free(softs), free(st.m), free(st.s), free(st.acc);
    free(src), free(plain), free(sum), free(kt), free(vt), free(kv), free(t), free(hidden), free(q), free(h), free(tmp), free(sc), free(scale2);
}

/* fit.rs:300-314: every column block's inducing-point queries for n training rows, out [blocks][inds][e] */
EXPORT void or_ind_queries(const or_rows_model *m, int n, float *out) {
    const int e = m->e, inds = m->inds;
    float *scale = malloc(sizeof(float) * e);
    for (int bi = 0; bi < m->ncol; bi++) {
        query_scale_c(&m->col1[bi], e, m->col_heads, n, scale);
        for (int i = 0; i < inds; i++)
            query_c(&m->col1[bi], e, m->col_heads, scale, m->col1[bi].ind + (size_t)i * e, out + ((size_t)bi * inds + i) * e);
    }
    free(scale);
}

/* fit.rs:333-345, 316-324 for one label digit: the training cells through the input layer with the label's embedding
 * added, out [n][feats][e] (what the `columns` hook of fit::Attend is given) */
EXPORT void or_fit_cells(const or_rows_model *m, const float *x, const float *y, int n, int feats, float *out) {
    const int e = m->e;
    float vals[8];
    for (int r = 0; r < n; r++)
        for (int g = 0; g < feats; g++) {
            float *cell = out + ((size_t)r * feats + g) * e;
            group_values(x + (size_t)r * feats, feats, g, m->group, vals);
            int missing = 1;
            for (int i = 0; i < m->group; i++) missing &= vals[i] == -100.0f;
            if (missing)
                for (int i = 0; i < e; i++) cell[i] = -100.0f;
            else
                linear(m->in_w, m->in_b, vals, m->group, e, cell);
            add_y_c(m->col_y, m->max_classes, e, y[r], cell);
        }
}

/* fit.rs:298-420 for a member's training rows: x [n][feats] (normalised), y [n] (classes, or the standardised target),
 * the rows `chunk` at a time through the inducing points' attention, `digits` label digits of mixed-radix `bases`.
 * Writes col_kv [feats][digits][blocks][2][e][inds] and the training tokens [n][cls + feats][e] (the class tokens,
 * then the cells after the column stage), the row stage's input. */
EXPORT void or_fit_columns(const or_rows_model *m, const float *x, const float *y, int n, int feats, int chunk,
                           int digits, const int *bases, float *col_kv, float *tok) {
    const int e = m->e, inds = m->inds, nb = m->ncol;
    float *ind_q = malloc(sizeof(float) * (size_t)nb * inds * e), *scale = malloc(sizeof(float) * e);
    /* fit.rs:300-314: the inducing points' queries are the same for every column */
    for (int bi = 0; bi < nb; bi++) {
        query_scale_c(&m->col1[bi], e, m->col_heads, n, scale);
        for (int i = 0; i < inds; i++)
            query_c(&m->col1[bi], e, m->col_heads, scale, m->col1[bi].ind + (size_t)i * e, ind_q + ((size_t)bi * inds + i) * e);
    }
    for (int r = 0; r < n; r++) memcpy(tok + (size_t)r * (m->cls + feats) * e, m->cls_tokens, sizeof(float) * m->cls * e);
    fitcol_job j;
    j.m = m, j.x = x, j.y = y, j.ind_q = ind_q, j.bases = bases, j.n = n, j.feats = feats, j.chunk = chunk < 8 ? 8 : chunk;
    j.digits = digits, j.col_kv = col_kv, j.tok = tok;
    par_for(feats, fitcol_one, &j);
    free(ind_q), free(scale);
}
