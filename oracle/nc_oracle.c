/* nc_oracle.c -- CPU restatement of nanocompile's fused Qwen2 step (TEST INFRASTRUCTURE ONLY).
 *
 * Every function below restates one kind of fused kernel that nanocompile's
 * fusion.py emits, in the operation order of the C its codegen_c.py writes
 * (compiled there with -O3 -ffp-contract=off: a multiply and an add stay two
 * roundings; fmaf appears only where the loop IR has an Fma node).  This file
 * is compiled with -ffp-contract=off too, so its float32 results are the
 * reference's bit for bit.  Citations are to files of the nanocompile project.
 *
 * It is the parity checker for the CUDA path and the CPU baseline of bench.py;
 * the product never links or calls it.
 */
#include "nc_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define QBLOCK 32   /* quantize.py:43 DEFAULT_BLOCK */

/* ---- transcendental functions ------------------------------------------------ */

float orc_expf_libm(float x) { return expf(x); }
float orc_cosf_libm(float x) { return cosf(x); }
float orc_sinf_libm(float x) { return sinf(x); }

/* A table-driven exp in double precision: x*32/ln2 = k + r, exp(x) = 2^(k/32) *
 * p(r) with p a cubic, then one rounding to float.  This is the method of ARM's
 * optimized-routines expf that glibc (2.28+) ships; the 2^(i/32) table is
 * computed from its definition, and the reduction's remainder is a fused
 * multiply-subtract as in glibc's FMA build.  Checked against glibc's expf on
 * every float in (-103.9, 88.7) by the tests; the CUDA kernels use the same
 * steps in double precision. */
static const uint64_t EXP_TAB[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

float orc_expf_restated(float x) {
    uint32_t ux;
    memcpy(&ux, &x, 4);
    uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) {                     /* |x| >= 88, or inf / nan */
        if (ux == 0xff800000u) return 0.0f;    /* -inf */
        if (abstop >= 0x7f8) return x + x;     /* +inf, nan */
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double inv_ln2_32 = 0x1.71547652b82fep+0 * 32;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
    double xd = (double)x;
    double z = inv_ln2_32 * xd;
    double kd = z + shift;
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= shift;
    double r = fma(inv_ln2_32, xd, -kd);
    uint64_t t = EXP_TAB[ki % 32] + (ki << 47);
    double s;
    memcpy(&s, &t, 8);
    double p = fma(c0, r, c1);
    double y = fma(c2, r, 1.0);
    y = fma(p, r * r, y);
    return (float)(y * s);
}

void orc_map(int32_t which, const float *x, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) {
        switch (which) {
            case 0: out[i] = expf(x[i]); break;
            case 1: out[i] = orc_expf_restated(x[i]); break;
            case 2: out[i] = cosf(x[i]); break;
            default: out[i] = sinf(x[i]); break;
        }
    }
}

/* ---- small helpers ---------------------------------------------------------------- */

/* Row-parallel loops run on plain pthreads, a static block of rows per thread.  Every
 * output is still computed by one thread in the reference's order, so the thread count
 * never changes a bit. */
static int g_threads = 1;

static void set_threads(const orc_config *c) {
    if (c && c->threads > 0) g_threads = c->threads;
}

typedef void (*row_fn)(void *ctx, int64_t begin, int64_t end);
typedef struct { row_fn fn; void *ctx; int64_t begin, end; } par_job;

static void *par_main(void *p) {
    par_job *j = (par_job *)p;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

static void parallel_rows(int64_t n, row_fn fn, void *ctx) {
    int t = g_threads;
    if (t > 64) t = 64;
    if (t <= 1 || n < 256) { fn(ctx, 0, n); return; }
    pthread_t tid[64];
    par_job jobs[64];
    int64_t chunk = (n + t - 1) / t;
    for (int i = 0; i < t; ++i) {
        jobs[i].fn = fn; jobs[i].ctx = ctx;
        jobs[i].begin = i * chunk < n ? i * chunk : n;
        jobs[i].end = (i + 1) * chunk < n ? (i + 1) * chunk : n;
    }
    for (int i = 1; i < t; ++i) pthread_create(&tid[i], NULL, par_main, &jobs[i]);
    par_main(&jobs[0]);
    for (int i = 1; i < t; ++i) pthread_join(tid[i], NULL);
}

/* codegen_c.py:85-89 nc_dp4: four signed weight bytes offset to unsigned, times four
 * signed activation bytes, summed exactly in int32. */
static inline int32_t dp4(const int8_t *w, const int8_t *x) {
    int32_t sum = 0;
    for (int j = 0; j < 4; ++j) sum += ((int32_t)w[j] + 128) * (int32_t)x[j];
    return sum;
}

/* lower.py:298-317 _combine: the 32 accumulators in AVX2's order. */
static inline float combine32(const float *acc) {
    float h[8];
    for (int kh = 0; kh < 8; ++kh) h[kh] = (acc[kh] + acc[8 + kh]) + (acc[16 + kh] + acc[24 + kh]);
    return ((h[0] + h[4]) + (h[1] + h[5])) + ((h[2] + h[6]) + (h[3] + h[7]));
}

/* lower.py:363-397 int8_vnni_dots for one (token, output row): 128-byte strides into
 * accumulators 8c+l, leftover 32-byte groups into accumulators 0..7. */
static float vnni_dot(const int8_t *w, const int8_t *x, const float *xs, int64_t k, int32_t *lanes) {
    float acc[32];
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
    int64_t chunks = k / 128, stride = chunks * 128, groups = (k % 128) / 32;
    for (int64_t k0 = 0; k0 < chunks; ++k0)
        for (int c = 0; c < 4; ++c) {
            int64_t g = k0 * 128 + c * 32;
            float s = xs[g / QBLOCK];
            for (int l = 0; l < 8; ++l) {
                int32_t v = dp4(w + g + 4 * l, x + g + 4 * l);
                if (lanes) lanes[(g + 4 * l) / 4] = v;
                acc[c * 8 + l] = fmaf((float)v, s, acc[c * 8 + l]);
            }
        }
    for (int64_t k1 = 0; k1 < groups; ++k1) {
        int64_t g = stride + k1 * 32;
        float s = xs[g / QBLOCK];
        for (int l = 0; l < 8; ++l) {
            int32_t v = dp4(w + g + 4 * l, x + g + 4 * l);
            if (lanes) lanes[(g + 4 * l) / 4] = v;
            acc[l] = fmaf((float)v, s, acc[l]);
        }
    }
    return combine32(acc);
}

/* lower.py:320-356 int8_dots for one (token, output row), int8 weights widened to float times
 * float activations: accumulator j (0..31) takes element j of every 32-element block in order,
 * acc = fmaf(float(w), x, acc); the 8-element groups past the last whole block go into
 * accumulators 0..7, group after group; _combine; then each element past the last group is added
 * as sum = sum + float(w) * x (a multiply and an add, two roundings). */
static float i8f_dot(const int8_t *w, const float *x, int64_t k) {
    float acc[32] = {0};
    const int64_t wide = k / 32 * 32, groups = (k % 32) / 8, tail = wide + groups * 8;
    for (int64_t k0 = 0; k0 < k / 32; ++k0)
        for (int j = 0; j < 32; ++j) acc[j] = fmaf((float)w[k0 * 32 + j], x[k0 * 32 + j], acc[j]);
    for (int64_t k1 = 0; k1 < groups; ++k1)
        for (int j = 0; j < 8; ++j) acc[j] = fmaf((float)w[wide + k1 * 8 + j], x[wide + k1 * 8 + j], acc[j]);
    float sum = combine32(acc);
    for (int64_t r = tail; r < k; ++r) sum = sum + (float)w[r] * x[r];
    return sum;
}

/* lower.py:255-274 _matmul_kernel: acc = acc + a*b in index order, no FMA. */
static inline float f32_dot(const float *x, const float *w, int64_t k) {
    float acc = 0.0f;
    for (int64_t i = 0; i < k; ++i) acc = acc + x[i] * w[i];
    return acc;
}

/* ---- the fused groups ---------------------------------------------------------------- */

/* quantize.py:102-124 as fusion emits it (calls 2-7): block absmax with NaN propagation,
 * scale = mag <= 0 ? 1 : mag / 127, xq = (int8)clamp(roundf(x / scale)), int32 block sums,
 * offset = 128 * (in-order sum over blocks of float(sum_b) * scale_b). */
void orc_quantize_blocks(const float *x, int64_t rows, int64_t k, int8_t *xq, float *xs,
                         float *offset, int32_t *block_sums) {
    int64_t blocks = k / QBLOCK;
    for (int64_t m = 0; m < rows; ++m) {
        const float *xr = x + m * k;
        float acc_off = 0.0f;
        for (int64_t b = 0; b < blocks; ++b) {
            float mag = -INFINITY;
            for (int r = 0; r < QBLOCK; ++r) {
                float v = xr[b * QBLOCK + r];
                float a = (0.0f <= v) ? v : -v;
                mag = (mag < a || a != a) ? a : mag;
            }
            float scale = (mag <= 0.0f) ? 1.0f : mag / 127.0f;
            int32_t bsum = 0;
            for (int r = 0; r < QBLOCK; ++r) {
                float t = roundf(xr[b * QBLOCK + r] / scale);
                t = (t <= 127.0f) ? t : 127.0f;
                t = (-127.0f <= t) ? t : -127.0f;
                int8_t q = (int8_t)t;
                xq[m * k + b * QBLOCK + r] = q;
                bsum += (int32_t)q;
            }
            xs[m * blocks + b] = scale;
            if (block_sums) block_sums[m * blocks + b] = bsum;
            acc_off = acc_off + (float)bsum * scale;
        }
        offset[m] = acc_off * 128.0f;
    }
}

typedef struct {
    const int8_t *xq, *q;
    const float *xs, *offset, *scales;
    int64_t m, n, k;
    float *out;
    int32_t *lanes;
} vnni_job;

static void vnni_rows(void *p, int64_t begin, int64_t end) {
    const vnni_job *a = (const vnni_job *)p;
    int64_t blocks = a->k / QBLOCK;
    for (int64_t j = begin; j < end; ++j) {
        float sum = vnni_dot(a->q + j * a->k, a->xq + a->m * a->k, a->xs + a->m * blocks, a->k,
                             a->lanes ? a->lanes + (a->m * a->n + j) * (a->k / 4) : NULL);
        a->out[a->m * a->n + j] = (sum - a->offset[a->m]) * a->scales[j];
    }
}

void orc_matmul_i8_vnni(const int8_t *xq, const float *xs, const float *offset, const int8_t *q,
                        const float *scales, int64_t rows, int64_t n, int64_t k, float *out,
                        int32_t *lanes) {
    for (int64_t m = 0; m < rows; ++m) {
        vnni_job job = {xq, q, xs, offset, scales, m, n, k, out, lanes};
        parallel_rows(n, vnni_rows, &job);
    }
}

typedef struct {
    const float *x;
    const int8_t *q;
    const float *scales;
    int64_t m, n, k;
    float *out;
} i8f_job;

static void i8f_rows(void *p, int64_t begin, int64_t end) {
    const i8f_job *a = (const i8f_job *)p;
    const float *x = a->x + a->m * a->k;
    for (int64_t j = begin; j < end; ++j) a->out[a->m * a->n + j] = i8f_dot(a->q + j * a->k, x, a->k) * a->scales[j];
}

/* lower.py:398-412 / fusion.py:677-711 matmul_i8: out[m, n] = int8_dots(q[n], x[m]) * scales[n]. */
void orc_matmul_i8(const float *x, const int8_t *q, const float *scales, int64_t rows, int64_t n, int64_t k,
                   float *out) {
    for (int64_t m = 0; m < rows; ++m) {
        i8f_job job = {x, q, scales, m, n, k, out};
        parallel_rows(n, i8f_rows, &job);
    }
}

/* nn.py:34-38 rms_norm as one row kernel (fusion.py:631-650): in-order sum of squares, then
 * per element t = x * (1 / sqrtf(acc / n + eps)) * w.  With `residual`, the row is
 * x + residual (the final norm with the last block's residual add fused in, call 40). */
void orc_rms_norm(const float *x, const float *residual, const float *w, int64_t rows, int64_t n,
                  float eps, float *out) {
    const float fn = (float)n;
    for (int64_t m = 0; m < rows; ++m) {
        const float *xr = x + m * n;
        const float *rr = residual ? residual + m * n : NULL;
        float acc = 0.0f;
        for (int64_t r = 0; r < n; ++r) {
            float v = rr ? xr[r] + rr[r] : xr[r];
            acc = acc + v * v;
        }
        float inv = 1.0f / sqrtf(acc / fn + eps);
        for (int64_t j = 0; j < n; ++j) {
            float v = rr ? xr[j] + rr[j] : xr[j];
            out[m * n + j] = (v * inv) * w[j];
        }
    }
}

typedef struct {
    const float *x, *w;
    int64_t k;
    float *out;
} f32_job;

static void f32_rows(void *p, int64_t begin, int64_t end) {
    const f32_job *a = (const f32_job *)p;
    for (int64_t j = begin; j < end; ++j) a->out[j] = f32_dot(a->x, a->w + j * a->k, a->k);
}

void orc_lm_head(const float *x, const float *embed, int64_t vocab, int64_t hidden, float *logits) {
    f32_job job = {x, embed, hidden, logits};
    parallel_rows(vocab, f32_rows, &job);
}

/* models/qwen2.py:364 np.argmax: the first maximum wins (NaN counts as the maximum). */
int64_t orc_argmax(const float *v, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i) {
        if (v[best] != v[best]) break;
        if (v[i] > v[best] || v[i] != v[i]) best = i;
    }
    return best;
}

/* nn.py:57-66 softmax as one row kernel with two reductions (call 15): t = s * scale + mask,
 * NaN-propagating max, in-order sum of expf(t - max), then expf(t - max) / sum. */
static void softmax_row(const float *scores, int64_t len, int64_t visible, float scale, float *p) {
    float mx = -INFINITY;
    for (int64_t r = 0; r < len; ++r) {
        float t = scores[r] * scale + ((r <= visible) ? 0.0f : -INFINITY);
        mx = (mx < t || t != t) ? t : mx;
    }
    float sum = 0.0f;
    for (int64_t r = 0; r < len; ++r) {
        float t = scores[r] * scale + ((r <= visible) ? 0.0f : -INFINITY);
        sum = sum + expf(t - mx);
    }
    for (int64_t r = 0; r < len; ++r) {
        float t = scores[r] * scale + ((r <= visible) ? 0.0f : -INFINITY);
        p[r] = expf(t - mx) / sum;
    }
}

void orc_attention_decode(const float *q, const float *keys, const float *values, int64_t heads,
                          int64_t kv_heads, int64_t len, int64_t d, int64_t cap, float scale,
                          float *out, float *probs) {
    int64_t group = heads / kv_heads;
    float *buf = (float *)malloc(sizeof(float) * (size_t)len * 2);
    for (int64_t h = 0; h < heads; ++h) {
        const float *kh = keys + (h / group) * cap * d;
        const float *vh = values + (h / group) * cap * d;
        float *sc = buf, *p = buf + len;
        for (int64_t j = 0; j < len; ++j) sc[j] = f32_dot(q + h * d, kh + j * d, d);
        softmax_row(sc, len, len - 1, scale, p);
        if (probs) memcpy(probs + h * len, p, sizeof(float) * (size_t)len);
        for (int64_t e = 0; e < d; ++e) {
            float acc = 0.0f;
            for (int64_t j = 0; j < len; ++j) acc = acc + p[j] * vh[j * d + e];
            out[h * d + e] = acc;
        }
    }
    free(buf);
}

/* One projection of `rows` activations: float32 (acc = acc + x*w) or int8-vnni.  The
 * int8 form takes the already-quantized activations. */
typedef struct {
    const float *x;           /* float32 mode */
    const int8_t *xq;         /* int8 mode */
    const float *xs, *offset;
} acts;

static void project(const orc_config *c, const acts *a, const float *w32, const int8_t *w8,
                    const float *scales, int64_t rows, int64_t n, int64_t k, float *out) {
    if (c->quant == 1) {
        orc_matmul_i8_vnni(a->xq, a->xs, a->offset, w8, scales, rows, n, k, out, NULL);
        return;
    }
    if (c->quant == 2) {
        orc_matmul_i8(a->x, w8, scales, rows, n, k, out);
        return;
    }
    for (int64_t m = 0; m < rows; ++m) {
        f32_job job = {a->x + m * k, w32, k, out + m * n};
        parallel_rows(n, f32_rows, &job);
    }
}

typedef struct {
    int8_t *xq;
    float *xs, *offset;
} qbuf;

static acts make_acts(const orc_config *c, const float *x, int64_t rows, int64_t k, qbuf *q) {
    acts a = {x, NULL, NULL, NULL};
    if (c->quant == 1) {
        orc_quantize_blocks(x, rows, k, q->xq, q->xs, q->offset, NULL);
        a.xq = q->xq;
        a.xs = q->xs;
        a.offset = q->offset;
    }
    return a;
}

/* nn.py:97-106 apply_rope fused with the projection bias (calls 11 and 13): for head h,
 * t1 = y + b, out = t1 * cos + (i < half ? -(y' + b') : (y' + b')) * sin. */
static void bias_rope(const float *y, const float *bias, int64_t rows, int64_t nheads, int64_t d,
                      const float *cosv, const float *sinv, float *out /* [nheads, rows, d] */) {
    int64_t half = d / 2, width = nheads * d;
    for (int64_t h = 0; h < nheads; ++h)
        for (int64_t s = 0; s < rows; ++s)
            for (int64_t i = 0; i < d; ++i) {
                float t1 = y[s * width + h * d + i] + bias[h * d + i];
                float t2 = t1 * cosv[s * d + i];
                float rot = (i < half) ? -(y[s * width + h * d + i + half] + bias[h * d + i + half])
                                       : y[s * width + h * d + i - half] + bias[h * d + i - half];
                out[(h * rows + s) * d + i] = t2 + rot * sinv[s * d + i];
            }
}

void orc_swiglu(const float *g, const float *u, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) {
        float g0 = g[i];
        int nonneg = 0.0f <= g0;
        float e = expf(nonneg ? -g0 : g0);
        float sig = (nonneg ? 1.0f : e) / (e + 1.0f);
        out[i] = (g0 * sig) * u[i];
    }
}

int32_t orc_qwen2_step(const orc_config *c, const float *embed, const float *final_norm,
                       const orc_layer *layers, const float *inv_freq,
                       const int64_t *ids, int64_t seq,
                       const float *past_keys, const float *past_values, int64_t past, int64_t past_cap,
                       int32_t last_only, float *logits, float *keys, float *values,
                       int64_t *bad_index) {
    set_threads(c);
    const int64_t H = c->hidden, I = c->inter, d = c->head_dim, nh = c->heads, nkv = c->kv_heads;
    const int64_t group = nh / nkv, half = d / 2, total = past + seq, L = c->layers;

    /* fusion.py:713-731 gather, failing on the first id out of range (status 1). */
    for (int64_t s = 0; s < seq; ++s)
        if (ids[s] < 0 || ids[s] >= c->vocab) {
            if (bad_index) *bad_index = ids[s];
            return 1;
        }

    float *x = (float *)malloc(sizeof(float) * seq * H);
    float *normed = (float *)malloc(sizeof(float) * seq * H);
    float *y = (float *)malloc(sizeof(float) * seq * (I > H ? I : H));
    float *y2 = (float *)malloc(sizeof(float) * seq * I);
    float *qr = (float *)malloc(sizeof(float) * nh * seq * d);
    float *kr = (float *)malloc(sizeof(float) * nkv * seq * d);
    float *vv = (float *)malloc(sizeof(float) * seq * nkv * d);
    float *ctx = (float *)malloc(sizeof(float) * seq * H);
    float *sc = (float *)malloc(sizeof(float) * total);
    float *pr = (float *)malloc(sizeof(float) * total);
    float *cosv = (float *)malloc(sizeof(float) * seq * d);
    float *sinv = (float *)malloc(sizeof(float) * seq * d);
    int64_t kmax = I > H ? I : H;
    qbuf qb = {(int8_t *)malloc((size_t)(seq * kmax)), (float *)malloc(sizeof(float) * seq * (kmax / QBLOCK + 1)),
               (float *)malloc(sizeof(float) * seq)};

    for (int64_t s = 0; s < seq; ++s) memcpy(x + s * H, embed + ids[s] * H, sizeof(float) * H);

    /* nn.py:78-94 rope_tables (calls 9-10): angle = float(past + s) * inv_freq[i mod d/2]. */
    for (int64_t s = 0; s < seq; ++s)
        for (int64_t i = 0; i < d; ++i) {
            float angle = (float)(s + past) * inv_freq[i % half];
            cosv[s * d + i] = cosf(angle);
            sinv[s * d + i] = sinf(angle);
        }

    for (int64_t l = 0; l < L; ++l) {
        const orc_layer *w = &layers[l];
        /* models/qwen2.py:113-155 _attention */
        orc_rms_norm(x, NULL, w->in_norm, seq, H, c->eps, normed);
        acts a = make_acts(c, normed, seq, H, &qb);
        project(c, &a, w->wq, w->qq, w->sq, seq, nh * d, H, y);
        bias_rope(y, w->bq, seq, nh, d, cosv, sinv, qr);
        project(c, &a, w->wk, w->qk, w->sk, seq, nkv * d, H, y);
        bias_rope(y, w->bk, seq, nkv, d, cosv, sinv, kr);
        project(c, &a, w->wv, w->qv, w->sv, seq, nkv * d, H, vv);
        for (int64_t i = 0; i < seq * nkv * d; ++i) vv[i] = vv[i] + w->bv[i % (nkv * d)];

        const float *pk = past_keys + l * nkv * past_cap * d;
        const float *pv = past_values + l * nkv * past_cap * d;
        for (int64_t h = 0; h < nh; ++h) {
            int64_t g = h / group;
            for (int64_t s = 0; s < seq; ++s) {
                const float *qh = qr + (h * seq + s) * d;
                for (int64_t j = 0; j < total; ++j) {
                    const float *kj = j < past ? pk + (g * past_cap + j) * d : kr + (g * seq + (j - past)) * d;
                    sc[j] = f32_dot(qh, kj, d);
                }
                softmax_row(sc, total, s + past, c->attn_scale, pr);
                for (int64_t e = 0; e < d; ++e) {
                    float acc = 0.0f;
                    for (int64_t j = 0; j < total; ++j) {
                        float vj = j < past ? pv[(g * past_cap + j) * d + e] : vv[(j - past) * nkv * d + g * d + e];
                        acc = acc + pr[j] * vj;
                    }
                    ctx[s * H + h * d + e] = acc;
                }
            }
        }
        for (int64_t g = 0; g < nkv; ++g)
            for (int64_t s = 0; s < seq; ++s)
                for (int64_t e = 0; e < d; ++e) {
                    keys[((l * nkv + g) * seq + s) * d + e] = kr[(g * seq + s) * d + e];
                    values[((l * nkv + g) * seq + s) * d + e] = vv[s * nkv * d + g * d + e];
                }

        a = make_acts(c, ctx, seq, H, &qb);
        project(c, &a, w->wo, w->qo, w->so, seq, H, nh * d, y);
        for (int64_t i = 0; i < seq * H; ++i) x[i] = x[i] + y[i];   /* residual epilogue */

        /* models/qwen2.py:158-164 _feed_forward; nn.py:41-55 silu */
        orc_rms_norm(x, NULL, w->post_norm, seq, H, c->eps, normed);
        a = make_acts(c, normed, seq, H, &qb);
        project(c, &a, w->wg, w->qg, w->sg, seq, I, H, y);
        project(c, &a, w->wu, w->qu, w->su, seq, I, H, y2);
        orc_swiglu(y, y2, seq * I, y);
        a = make_acts(c, y, seq, I, &qb);
        project(c, &a, w->wd, w->qd, w->sd, seq, H, I, y2);
        for (int64_t i = 0; i < seq * H; ++i) x[i] = x[i] + y2[i];
    }

    int64_t first = last_only ? seq - 1 : 0;
    orc_rms_norm(x + first * H, NULL, final_norm, seq - first, H, c->eps, normed);
    for (int64_t s = 0; s < seq - first; ++s) orc_lm_head(normed + s * H, embed, c->vocab, H, logits + s * c->vocab);

    free(x); free(normed); free(y); free(y2); free(qr); free(kr); free(vv); free(ctx);
    free(sc); free(pr); free(cosv); free(sinv); free(qb.xq); free(qb.xs); free(qb.offset);
    return 0;
}
