/*
 * w4j_oracle.c — CPU restatement of whisper4j's Whisper text-decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA path is compared
 * against; it is never linked into, loaded by, or called from the product
 * library (libwhisper4j_cuda.so) or its Python wrapper.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm use it.
 *
 * It restates, in plain C with strict IEEE f32 arithmetic (built with
 * -ffp-contract=off, no fast-math), the scalar Java 25 path of
 * sparrowlogic/whisper4j (the path taken on Linux, where Apple Accelerate is
 * absent and the Vector API module is not loaded):
 *
 *   forward            nn/WhisperDecoder.java:66-104   (embedding, blocks, ln, logits)
 *   block              nn/ResidualAttentionBlock.java:42-60
 *   attention + cache  nn/MultiHeadAttention.java:38-164
 *   fused M=1 head     tensor/SimdOps.java:182-226
 *   linear             nn/Linear.java:16-26 -> tensor/Tensor.java:403-422, :383-398,
 *                      :460-489 (row-accumulate, k ascending, bias added after)
 *   logits             tensor/Tensor.java:316-340 (dot, k ascending) with
 *                      tensor/SimdOps.java:155-166
 *   layer norm         tensor/Tensor.java:592-619
 *   GELU (f16 LUT)     tensor/Tensor.java:493-538
 *   softmax / mask     tensor/Tensor.java:541-569, :622-640
 *   greedy decode      nn/WhisperDecoder.java:161-204
 *   beam decode        nn/WhisperDecoder.java:214-394, :397-431
 *   logit processors   nn/WhisperDecoder.java:442-626
 *   Q8_0 / f16 dequant model/GgmlLoader.java:224-238, :292-300 (done by the caller,
 *                      which passes f32 tensors here)
 *
 * Every sum runs in the same order as the Java loop it restates, so the oracle
 * is deterministic and independent of thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

#include "w4j_oracle.h"

/* ------------------------------------------------------------------------ */
/* error text                                                                */
/* ------------------------------------------------------------------------ */

static _Thread_local char g_err[512];
static _Thread_local double g_loop_seconds; /* wall time of the token loop after the first step */

#include <time.h>
static double now_seconds(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

double orc_last_loop_seconds(void) { return g_loop_seconds; }

/* Threads of the oracle's own loops (tests only; 1 = the reference's single-threaded decoder).
 * Work is split over independent output elements (rows, column blocks, heads, vocabulary ids),
 * so every sum keeps the order of the loop it restates and results do not depend on it. */
static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n > 256 ? 256 : n; }

/* fn(ctx, i) for i in [0, n), split into g_threads contiguous ranges */
typedef void (*par_fn)(void *ctx, int i);
typedef struct {
    par_fn fn;
    void *ctx;
    int i0, i1, slot;
} par_range;
static __thread int g_worker = 0; /* index of the par_for range this thread runs (scratch buffers) */
static void *par_worker(void *p) {
    par_range *r = (par_range *)p;
    const int saved = g_worker;
    g_worker = r->slot;
    for (int i = r->i0; i < r->i1; i++) r->fn(r->ctx, i);
    g_worker = saved;
    return NULL;
}
static void par_for(int n, par_fn fn, void *ctx) {
    const int T = g_threads < n ? g_threads : n;
    if (T <= 1) {
        for (int i = 0; i < n; i++) fn(ctx, i);
        return;
    }
    pthread_t th[256];
    par_range rg[256];
    int ok[256];
    for (int t = 0; t < T; t++) {
        rg[t].fn = fn;
        rg[t].ctx = ctx;
        rg[t].i0 = (int)((long long)n * t / T);
        rg[t].i1 = (int)((long long)n * (t + 1) / T);
        rg[t].slot = t;
        ok[t] = t > 0 && pthread_create(&th[t], NULL, par_worker, &rg[t]) == 0;
    }
    par_worker(&rg[0]);
    for (int t = 1; t < T; t++) {
        if (ok[t]) pthread_join(th[t], NULL);
        else par_worker(&rg[t]); /* a thread that could not start: its range runs here */
    }
}

static int fail(const char *msg, const char *detail) {
    snprintf(g_err, sizeof g_err, "%s%s%s", msg, detail ? ": " : "", detail ? detail : "");
    return -1;
}

const char *orc_last_error(void) { return g_err; }

/* ------------------------------------------------------------------------ */
/* model                                                                     */
/* ------------------------------------------------------------------------ */

typedef struct {
    /* Linear weights are stored pre-transposed (in, out), as Linear.java:16-20 does. */
    float *attn_ln_w, *attn_ln_b;
    float *q_wt, *q_b, *k_wt, *k_b, *v_wt, *v_b, *o_wt, *o_b;
    float *x_ln_w, *x_ln_b;
    float *xq_wt, *xq_b, *xk_wt, *xk_b, *xv_wt, *xv_b, *xo_wt, *xo_b;
    float *mlp_ln_w, *mlp_ln_b;
    float *m0_wt, *m0_b, *m2_wt, *m2_b;
} orc_layer;

struct orc_model {
    orc_dims d;
    float *tok_emb; /* (V, d) native layout, used untransposed by matmulTransB */
    float *pos_emb; /* (C, d) */
    float *ln_w, *ln_b;
    orc_layer *layers;
    float gelu_table[65536];
};

/* f32 -> f16 bits, round to nearest even (Float.floatToFloat16 semantics). */
static uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf or nan */
        if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((absx >> 13) & 0x3ffu));
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (absx < 0x38800000u) {                                     /* subnormal or zero in f16 */
        if (absx < 0x33000000u) return (uint16_t)sign;            /* < 2^-25 -> 0 (2^-25 ties to even 0) */
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14 + (112 - e) - 0 ... produces 10-bit subnormal mantissa */
        /* value = m * 2^(e-150); f16 subnormal unit = 2^-24 -> q = m * 2^(e-126) */
        uint32_t q = m >> (shift);
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 112; /* rebias 127 -> 15 */
    uint32_t m = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t out;
    if (e == 0) {
        if (m == 0) {
            out = sign;
        } else { /* subnormal: normalise */
            e = 113;
            while ((m & 0x400u) == 0) { m <<= 1; e--; }
            m &= 0x3ffu;
            out = sign | (e << 23) | (m << 13);
        }
    } else if (e == 31) {
        out = sign | 0x7f800000u | (m << 13);
    } else {
        out = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) { return f32_to_f16_bits(f); }

/* Tensor.java:493-501 */
static void build_gelu_table(float *table) {
    float s = (float)sqrt(2.0 / M_PI);
    for (int i = 0; i < 65536; i++) {
        float x = orc_f16_to_f32((uint16_t)i);
        table[i] = 0.5f * x * (1.0f + (float)tanh((double)(s * (x + 0.044715f * x * x * x))));
    }
}

const float *orc_gelu_table(const orc_model *m) { return m->gelu_table; }

orc_model *orc_model_new(const orc_dims *d) {
    if (!d || d->n_text_state <= 0 || d->n_text_head <= 0 || d->n_text_state % d->n_text_head != 0 ||
        d->n_text_layer <= 0 || d->n_vocab <= 0 || d->n_text_ctx <= 0) {
        fail("orc_model_new", "invalid dimensions");
        return NULL;
    }
    orc_model *m = (orc_model *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->d = *d;
    m->layers = (orc_layer *)calloc((size_t)d->n_text_layer, sizeof(orc_layer));
    build_gelu_table(m->gelu_table);
    return m;
}

static void free_layer(orc_layer *l) {
    float **p = (float **)l;
    for (size_t i = 0; i < sizeof(orc_layer) / sizeof(float *); i++) free(p[i]);
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    for (int i = 0; i < m->d.n_text_layer; i++) free_layer(&m->layers[i]);
    free(m->layers);
    free(m->tok_emb);
    free(m->pos_emb);
    free(m->ln_w);
    free(m->ln_b);
    free(m);
}

static float *dup_f32(const float *src, long n) {
    float *p = (float *)malloc((size_t)n * sizeof(float));
    if (p) memcpy(p, src, (size_t)n * sizeof(float));
    return p;
}

/* Linear.java:18 — weight (out, in) -> weightT (in, out). */
static float *dup_transposed(const float *w, int out, int in) {
    float *t = (float *)malloc((size_t)out * in * sizeof(float));
    if (!t) return NULL;
    for (int o = 0; o < out; o++)
        for (int i = 0; i < in; i++) t[(size_t)i * out + o] = w[(size_t)o * in + i];
    return t;
}

int orc_set_tensor(orc_model *m, const char *name, const float *data, long n) {
    const int d = m->d.n_text_state, V = m->d.n_vocab, C = m->d.n_text_ctx;
    if (strncmp(name, "decoder.", 8) != 0) return 1; /* encoder and others: not on this path */
    const char *s = name + 8;
#define EXPECT(cnt)                                                             \
    do {                                                                        \
        if (n != (long)(cnt)) return fail("orc_set_tensor: wrong element count", name); \
    } while (0)
    if (!strcmp(s, "token_embedding.weight")) { EXPECT((long)V * d); free(m->tok_emb); m->tok_emb = dup_f32(data, n); return 0; }
    if (!strcmp(s, "positional_embedding")) { EXPECT((long)C * d); free(m->pos_emb); m->pos_emb = dup_f32(data, n); return 0; }
    if (!strcmp(s, "ln.weight")) { EXPECT(d); free(m->ln_w); m->ln_w = dup_f32(data, n); return 0; }
    if (!strcmp(s, "ln.bias")) { EXPECT(d); free(m->ln_b); m->ln_b = dup_f32(data, n); return 0; }
    int li = -1, off = 0;
    if (sscanf(s, "blocks.%d.%n", &li, &off) != 1 || li < 0 || li >= m->d.n_text_layer)
        return fail("orc_set_tensor: unknown tensor", name);
    orc_layer *L = &m->layers[li];
    const char *t = s + off;
    struct { const char *nm; float **dst; int rows, cols; } tab[] = {
        {"attn_ln.weight", &L->attn_ln_w, 0, d}, {"attn_ln.bias", &L->attn_ln_b, 0, d},
        {"attn.query.weight", &L->q_wt, d, d}, {"attn.query.bias", &L->q_b, 0, d},
        {"attn.key.weight", &L->k_wt, d, d}, {"attn.key.bias", &L->k_b, 0, d},
        {"attn.value.weight", &L->v_wt, d, d}, {"attn.value.bias", &L->v_b, 0, d},
        {"attn.out.weight", &L->o_wt, d, d}, {"attn.out.bias", &L->o_b, 0, d},
        {"cross_attn_ln.weight", &L->x_ln_w, 0, d}, {"cross_attn_ln.bias", &L->x_ln_b, 0, d},
        {"cross_attn.query.weight", &L->xq_wt, d, d}, {"cross_attn.query.bias", &L->xq_b, 0, d},
        {"cross_attn.key.weight", &L->xk_wt, d, d}, {"cross_attn.key.bias", &L->xk_b, 0, d},
        {"cross_attn.value.weight", &L->xv_wt, d, d}, {"cross_attn.value.bias", &L->xv_b, 0, d},
        {"cross_attn.out.weight", &L->xo_wt, d, d}, {"cross_attn.out.bias", &L->xo_b, 0, d},
        {"mlp_ln.weight", &L->mlp_ln_w, 0, d}, {"mlp_ln.bias", &L->mlp_ln_b, 0, d},
        {"mlp.0.weight", &L->m0_wt, 4 * d, d}, {"mlp.0.bias", &L->m0_b, 0, 4 * d},
        {"mlp.2.weight", &L->m2_wt, d, 4 * d}, {"mlp.2.bias", &L->m2_b, 0, d},
    };
    for (size_t i = 0; i < sizeof tab / sizeof tab[0]; i++) {
        if (strcmp(t, tab[i].nm) != 0) continue;
        free(*tab[i].dst);
        if (tab[i].rows == 0) {
            EXPECT(tab[i].cols);
            *tab[i].dst = dup_f32(data, n);
        } else {
            EXPECT((long)tab[i].rows * tab[i].cols);
            *tab[i].dst = dup_transposed(data, tab[i].rows, tab[i].cols);
        }
        return 0;
    }
    return fail("orc_set_tensor: unknown tensor", name);
#undef EXPECT
}

int orc_model_check(const orc_model *m) {
    if (!m->tok_emb) return fail("weight not found", "decoder.token_embedding.weight");
    if (!m->pos_emb) return fail("weight not found", "decoder.positional_embedding");
    if (!m->ln_w || !m->ln_b) return fail("weight not found", "decoder.ln");
    for (int i = 0; i < m->d.n_text_layer; i++) {
        const orc_layer *L = &m->layers[i];
        /* key biases are optional (WhisperEncoder.java:101); everything else is required */
        const float *req[] = {L->attn_ln_w, L->attn_ln_b, L->q_wt, L->q_b, L->k_wt, L->v_wt, L->v_b, L->o_wt, L->o_b,
                              L->x_ln_w, L->x_ln_b, L->xq_wt, L->xq_b, L->xk_wt, L->xv_wt, L->xv_b, L->xo_wt, L->xo_b,
                              L->mlp_ln_w, L->mlp_ln_b, L->m0_wt, L->m0_b, L->m2_wt, L->m2_b};
        for (size_t j = 0; j < sizeof req / sizeof req[0]; j++)
            if (!req[j]) {
                char b[64];
                snprintf(b, sizeof b, "decoder.blocks.%d (tensor %zu)", i, j);
                return fail("weight not found", b);
            }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* tensor primitives (Tensor.java / SimdOps.java scalar paths)               */
/* ------------------------------------------------------------------------ */

/* SimdOps.java:155-166 */
float orc_dot(const float *a, const float *b, int n) {
    float sum = 0;
    for (int i = 0; i < n; i++) sum += a[i] * b[i];
    return sum;
}

/* y(M,N) = x(M,K) . wt(K,N) [+ bias]; Tensor.java:383-398 (M=1) and :460-489 (M>1):
 * both accumulate out[i][j] over k ascending from 0.  Bias added after
 * (Linear.java:25 -> Tensor.java:251-263). */
static void linear_cols(const float *xi, int K, const float *wt, const float *bias, int N, float *yi, int j0, int j1) {
    for (int j = j0; j < j1; j++) yi[j] = 0.0f;
    for (int k = 0; k < K; k++) {
        const float xk = xi[k];
        const float *wk = wt + (size_t)k * N;
        for (int j = j0; j < j1; j++) yi[j] = yi[j] + xk * wk[j];
    }
    if (bias)
        for (int j = j0; j < j1; j++) yi[j] = yi[j] + bias[j];
}

typedef struct {
    const float *x, *wt, *bias;
    int K, N, row;
    float *y;
} linear_job;
static void linear_row_job(void *p, int i) {
    const linear_job *j = (const linear_job *)p;
    linear_cols(j->x + (size_t)i * j->K, j->K, j->wt, j->bias, j->N, j->y + (size_t)i * j->N, 0, j->N);
}
static void linear_block_job(void *p, int b) {
    const linear_job *j = (const linear_job *)p;
    const int j0 = b * 256, j1 = j0 + 256 < j->N ? j0 + 256 : j->N;
    linear_cols(j->x + (size_t)j->row * j->K, j->K, j->wt, j->bias, j->N, j->y + (size_t)j->row * j->N, j0, j1);
}

static void linear(const float *x, int M, int K, const float *wt, const float *bias, int N, float *y) {
    linear_job job = {x, wt, bias, K, N, 0, y};
    if (g_threads > 1 && M >= 2 * g_threads) {
        par_for(M, linear_row_job, &job);
        return;
    }
    for (int i = 0; i < M; i++) {
        if (g_threads > 1 && N >= 512) {
            job.row = i;
            par_for((N + 255) / 256, linear_block_job, &job);
        } else {
            linear_cols(x + (size_t)i * K, K, wt, bias, N, y + (size_t)i * N, 0, N);
        }
    }
}

/* Tensor.java:592-619 */
static void layer_norm(const float *x, int M, int n, const float *g, const float *b, float eps, float *y) {
    for (int i = 0; i < M; i++) {
        const float *row = x + (size_t)i * n;
        float mean = 0;
        for (int j = 0; j < n; j++) mean += row[j];
        mean /= n;
        float variance = 0;
        for (int j = 0; j < n; j++) {
            float dd = row[j] - mean;
            variance += dd * dd;
        }
        float inv_std = 1.0f / (float)sqrt((double)(variance / n + eps));
        float *out = y + (size_t)i * n;
        for (int j = 0; j < n; j++) out[j] = (row[j] - mean) * inv_std * g[j] + b[j];
    }
}

/* Tensor.java:524-538 */
static void gelu_inplace(const float *table, float *x, long n) {
    for (long i = 0; i < n; i++) x[i] = table[f32_to_f16_bits(x[i])];
}

/* SimdOps.java:182-226 — one head of single-query attention; also equals the
 * multi-query path (Tensor.java:316-374 dot*alpha, :622-640 mask, :541-569
 * softmax, :460-489 matmul) row by row, with keys [masked_from, masked_to)
 * given -inf. */
static void attention_head(const float *q, const float *k, const float *v, int kv_len, int row_stride,
                           int masked_from, int masked_to, float scale, float *scores, float *out) {
    float max_score = -INFINITY;
    for (int j = 0; j < kv_len; j++) {
        float s = orc_dot(q, k + (size_t)j * row_stride, 64) * scale;
        if (j >= masked_from && j < masked_to) s = s + -INFINITY;
        scores[j] = s;
        if (s > max_score) max_score = s;
    }
    float sum = 0;
    for (int j = 0; j < kv_len; j++) {
        scores[j] = (float)exp((double)(scores[j] - max_score));
        sum += scores[j];
    }
    float inv_sum = 1.0f / sum;
    for (int j = 0; j < kv_len; j++) scores[j] *= inv_sum;
    for (int dd = 0; dd < 64; dd++) out[dd] = 0.0f;
    for (int j = 0; j < kv_len; j++) {
        const float sj = scores[j];
        const float *vr = v + (size_t)j * row_stride;
        for (int dd = 0; dd < 64; dd++) out[dd] = out[dd] + sj * vr[dd];
    }
}

/* one (row, head) of an attention loop; mask_c >= 0: the multi-token causal mask with n_ctx mask_c */
typedef struct {
    const float *q, *K, *V;
    float *out;
    int d, H, kv_len, mask_c;
    float scale;
    float *scores;
    int scores_len;
} attn_job;
static void attn_self_job(void *p, int th) {
    const attn_job *j = (const attn_job *)p;
    const int t = th / j->H, hh = th % j->H;
    int masked_from = j->kv_len, masked_to = j->kv_len;
    if (j->mask_c >= 0 && t < j->mask_c) {
        masked_from = t + 1;
        masked_to = j->kv_len < j->mask_c ? j->kv_len : j->mask_c;
    }
    float *sc = j->scores + (size_t)j->scores_len * (size_t)g_worker; /* this range's score buffer */
    attention_head(j->q + (size_t)t * j->d + hh * 64, j->K + hh * 64, j->V + hh * 64, j->kv_len, j->d, masked_from,
                   masked_to, j->scale, sc, j->out + (size_t)t * j->d + hh * 64);
}

typedef struct {
    const float *x, *E;
    int d, V;
    float *out;
} logits_job;
static void logits_block_job(void *p, int b) {
    const logits_job *j = (const logits_job *)p;
    const int j1 = (b + 1) * 1024 < j->V ? (b + 1) * 1024 : j->V;
    for (int v = b * 1024; v < j1; v++) j->out[v] = orc_dot(j->x, j->E + (size_t)v * j->d, j->d) * 1.0f;
}

/* KATs for the reference's tensor unit tests (TensorTest.java). */
void orc_matmul(const float *a, const float *b, int M, int K, int N, float *out) {
    linear(a, M, K, b, NULL, N, out);
}
void orc_matmul_transb(const float *a, const float *b, int M, int K, int N, float alpha, float *out) {
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) out[(size_t)i * N + j] = orc_dot(a + (size_t)i * K, b + (size_t)j * K, K) * alpha;
}
void orc_softmax_rows(float *x, int rows, int n) {
    for (int i = 0; i < rows; i++) {
        float *row = x + (size_t)i * n;
        float max = row[0];
        for (int j = 1; j < n; j++)
            if (row[j] > max) max = row[j];
        float sum = 0;
        for (int j = 0; j < n; j++) {
            row[j] = (float)exp((double)(row[j] - max));
            sum += row[j];
        }
        float inv = 1.0f / sum;
        for (int j = 0; j < n; j++) row[j] *= inv;
    }
}
void orc_layer_norm(const float *x, int rows, int n, const float *g, const float *b, float eps, float *y) {
    layer_norm(x, rows, n, g, b, eps, y);
}
void orc_gelu(const orc_model *m, float *x, long n) { gelu_inplace(m->gelu_table, x, n); }

/* ------------------------------------------------------------------------ */
/* KV cache (MultiHeadAttention.java:140-164, kvCache map in WhisperDecoder)  */
/* ------------------------------------------------------------------------ */

struct orc_cache {
    int L, d, A;
    int len, cap;
    float **sk, **sv; /* per layer: (cap, d) rows = new K / V projections, heads interleaved */
    int has_cross;
    float **xk, **xv; /* per layer: (A, d) */
    int cross_shared; /* cross arrays borrowed from another cache (beam sharing) */
};

orc_cache *orc_cache_new(const orc_model *m, int n_audio_ctx) {
    orc_cache *c = (orc_cache *)calloc(1, sizeof *c);
    c->L = m->d.n_text_layer;
    c->d = m->d.n_text_state;
    c->A = n_audio_ctx;
    c->sk = (float **)calloc((size_t)c->L, sizeof(float *));
    c->sv = (float **)calloc((size_t)c->L, sizeof(float *));
    c->xk = (float **)calloc((size_t)c->L, sizeof(float *));
    c->xv = (float **)calloc((size_t)c->L, sizeof(float *));
    return c;
}

void orc_cache_free(orc_cache *c) {
    if (!c) return;
    for (int l = 0; l < c->L; l++) {
        free(c->sk[l]);
        free(c->sv[l]);
        if (!c->cross_shared) {
            free(c->xk[l]);
            free(c->xv[l]);
        }
    }
    free(c->sk); free(c->sv); free(c->xk); free(c->xv);
    free(c);
}

int orc_cache_len(const orc_cache *c) { return c->len; }

static void cache_reserve(orc_cache *c, int need) {
    if (need <= c->cap) return;
    int cap = c->cap ? c->cap : 16;
    while (cap < need) cap *= 2;
    for (int l = 0; l < c->L; l++) {
        c->sk[l] = (float *)realloc(c->sk[l], (size_t)cap * c->d * sizeof(float));
        c->sv[l] = (float *)realloc(c->sv[l], (size_t)cap * c->d * sizeof(float));
    }
    c->cap = cap;
}

/* Copy of another beam's self cache (the reference re-points map entries; the
 * copy is numerically identical because appendHeadsCache never mutates). */
static void cache_copy_self(orc_cache *dst, const orc_cache *src) {
    cache_reserve(dst, src->len > 0 ? src->len : 1);
    for (int l = 0; l < dst->L; l++) {
        memcpy(dst->sk[l], src->sk[l], (size_t)src->len * dst->d * sizeof(float));
        memcpy(dst->sv[l], src->sv[l], (size_t)src->len * dst->d * sizeof(float));
    }
    dst->len = src->len;
}

static void cache_share_cross(orc_cache *dst, const orc_cache *src) {
    if (!dst->cross_shared)
        for (int l = 0; l < dst->L; l++) {
            free(dst->xk[l]);
            free(dst->xv[l]);
        }
    for (int l = 0; l < dst->L; l++) {
        dst->xk[l] = src->xk[l];
        dst->xv[l] = src->xv[l];
    }
    dst->has_cross = src->has_cross;
    dst->cross_shared = 1;
}

/* ------------------------------------------------------------------------ */
/* forward (WhisperDecoder.java:66-104)                                      */
/* ------------------------------------------------------------------------ */

int orc_forward(const orc_model *m, const int *tokens, int n, const float *xa, int n_audio_ctx, orc_cache *cache,
                float *logits) {
    const int d = m->d.n_text_state, H = m->d.n_text_head, V = m->d.n_vocab, C = m->d.n_text_ctx;
    const int L = m->d.n_text_layer;
    if (n <= 0) return fail("orc_forward", "empty token list");
    for (int t = 0; t < n; t++)
        if (tokens[t] < 0 || tokens[t] >= V) return fail("orc_forward", "token id out of range");
    if (cache && cache->A != n_audio_ctx) return fail("orc_forward", "cache built for another n_audio_ctx");
    const int head_dim = d / H;
    if (head_dim != 64) return fail("orc_forward", "head dim must be 64");
    const float scale = (float)(1.0 / sqrt((double)head_dim));

    int offset = 0;
    if (cache) {
        offset = cache->len;
        if (offset > C - n) offset = C - n;
    }
    if (offset < 0 || offset + n > C) return fail("orc_forward", "sequence longer than n_text_ctx");

    const int past = cache ? cache->len : 0;
    const int kv_len = past + n;
    float *x = (float *)malloc((size_t)n * d * sizeof(float));
    float *ln = (float *)malloc((size_t)n * d * sizeof(float));
    float *q = (float *)malloc((size_t)n * d * sizeof(float));
    float *merged = (float *)malloc((size_t)n * d * sizeof(float));
    float *tmp = (float *)malloc((size_t)n * d * sizeof(float));
    float *h = (float *)malloc((size_t)n * 4 * d * sizeof(float));
    float *knew = (float *)malloc((size_t)n * d * sizeof(float));
    float *vnew = (float *)malloc((size_t)n * d * sizeof(float));
    int scores_len = kv_len > n_audio_ctx ? kv_len : n_audio_ctx;
    float *scores = (float *)malloc((size_t)scores_len * g_threads * sizeof(float));
    float *selfk = NULL, *selfv = NULL; /* no-cache path: own K/V */
    float *xk_tmp = NULL, *xv_tmp = NULL;
    if (cache) cache_reserve(cache, kv_len);

    for (int t = 0; t < n; t++) {
        const float *te = m->tok_emb + (size_t)tokens[t] * d;
        const float *pe = m->pos_emb + (size_t)(offset + t) * d;
        for (int j = 0; j < d; j++) x[(size_t)t * d + j] = te[j] + pe[j];
    }

    for (int l = 0; l < L; l++) {
        const orc_layer *Ly = &m->layers[l];
        /* ---- self attention (MultiHeadAttention.java:42-96 with xa == null) ---- */
        layer_norm(x, n, d, Ly->attn_ln_w, Ly->attn_ln_b, 1e-5f, ln);
        linear(ln, n, d, Ly->q_wt, Ly->q_b, d, q);
        linear(ln, n, d, Ly->k_wt, Ly->k_b, d, knew);
        linear(ln, n, d, Ly->v_wt, Ly->v_b, d, vnew);
        const float *K, *Vv;
        if (cache) {
            memcpy(cache->sk[l] + (size_t)past * d, knew, (size_t)n * d * sizeof(float));
            memcpy(cache->sv[l] + (size_t)past * d, vnew, (size_t)n * d * sizeof(float));
            K = cache->sk[l];
            Vv = cache->sv[l];
        } else {
            selfk = knew;
            selfv = vnew;
            K = selfk;
            Vv = selfv;
        }
        {
            /* mask (WhisperDecoder.java:43-49, Tensor.java:622-640) applies only when
             * qLen > 1, relative to this call's first row, and only to the first
             * min(kvLen, C) key columns. */
            attn_job job = {q, K, Vv, merged, d, H, kv_len, n > 1 ? C : -1, scale, scores, scores_len};
            par_for(n * H, attn_self_job, &job);
        }
        linear(merged, n, d, Ly->o_wt, Ly->o_b, d, tmp);
        for (long i = 0; i < (long)n * d; i++) x[i] = tmp[i] + x[i]; /* attnOut.addInPlace(x) */

        /* ---- cross attention (MultiHeadAttention.java:55-57, :65-75) ---- */
        layer_norm(x, n, d, Ly->x_ln_w, Ly->x_ln_b, 1e-5f, ln);
        linear(ln, n, d, Ly->xq_wt, Ly->xq_b, d, q);
        const float *XK, *XV;
        if (cache && cache->has_cross) {
            XK = cache->xk[l];
            XV = cache->xv[l];
        } else {
            float *kk = (float *)malloc((size_t)n_audio_ctx * d * sizeof(float));
            float *vv = (float *)malloc((size_t)n_audio_ctx * d * sizeof(float));
            linear(xa, n_audio_ctx, d, Ly->xk_wt, Ly->xk_b, d, kk);
            linear(xa, n_audio_ctx, d, Ly->xv_wt, Ly->xv_b, d, vv);
            if (cache) {
                free(cache->xk[l]);
                free(cache->xv[l]);
                cache->xk[l] = kk;
                cache->xv[l] = vv;
            } else {
                free(xk_tmp);
                free(xv_tmp);
                xk_tmp = kk;
                xv_tmp = vv;
            }
            XK = kk;
            XV = vv;
        }
        {
            attn_job job = {q, XK, XV, merged, d, H, n_audio_ctx, -1, scale, scores, scores_len};
            par_for(n * H, attn_self_job, &job);
        }
        linear(merged, n, d, Ly->xo_wt, Ly->xo_b, d, tmp);
        for (long i = 0; i < (long)n * d; i++) x[i] = x[i] + tmp[i];

        /* ---- MLP ---- */
        layer_norm(x, n, d, Ly->mlp_ln_w, Ly->mlp_ln_b, 1e-5f, ln);
        linear(ln, n, d, Ly->m0_wt, Ly->m0_b, 4 * d, h);
        gelu_inplace(m->gelu_table, h, (long)n * 4 * d);
        linear(h, n, 4 * d, Ly->m2_wt, Ly->m2_b, d, tmp);
        for (long i = 0; i < (long)n * d; i++) x[i] = x[i] + tmp[i];
    }
    if (cache) {
        cache->len = kv_len;
        cache->has_cross = 1;
    }

    layer_norm(x, n, d, m->ln_w, m->ln_b, 1e-5f, ln);
    for (int t = 0; t < n; t++) {
        logits_job job = {ln + (size_t)t * d, m->tok_emb, d, V, logits + (size_t)t * V};
        par_for((V + 1023) / 1024, logits_block_job, &job);
    }

    free(x); free(ln); free(q); free(merged); free(tmp); free(h); free(knew); free(vnew); free(scores);
    free(xk_tmp); free(xv_tmp);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* logit processors (WhisperDecoder.java:442-626)                            */
/* ------------------------------------------------------------------------ */

static float softmax_at(const float *logits, int n, int index) { /* :600-612 */
    float max = -INFINITY;
    for (int i = 0; i < n; i++)
        if (logits[i] > max) max = logits[i];
    double sum = 0;
    for (int i = 0; i < n; i++) sum += exp((double)(logits[i] - max));
    return (float)(exp((double)(logits[index] - max)) / sum);
}

static double log_softmax_at(const float *logits, int n, int index) { /* :614-626 */
    float max = -INFINITY;
    for (int i = 0; i < n; i++)
        if (logits[i] > max) max = logits[i];
    double log_sum = 0;
    for (int i = 0; i < n; i++) log_sum += exp((double)(logits[i] - max));
    return (double)(logits[index] - max) - log(log_sum);
}

static void compute_log_softmax(const float *logits, int n, float *out) { /* :397-412 */
    float max = -INFINITY;
    for (int i = 0; i < n; i++)
        if (logits[i] > max) max = logits[i];
    double log_sum = 0;
    for (int i = 0; i < n; i++) log_sum += exp((double)(logits[i] - max));
    float log_sum_f = (float)((double)max + log(log_sum));
    for (int i = 0; i < n; i++) out[i] = logits[i] - log_sum_f;
}

static void topk_indices(const float *values, int k, int n, int *indices) { /* :415-431 */
    float top[64];
    for (int i = 0; i < k; i++) {
        top[i] = -INFINITY;
        indices[i] = 0;
    }
    for (int i = 0; i < n; i++) {
        if (values[i] > top[k - 1]) {
            int pos = k - 1;
            while (pos > 0 && values[i] > top[pos - 1]) pos--;
            memmove(&top[pos + 1], &top[pos], (size_t)(k - 1 - pos) * sizeof(float));
            memmove(&indices[pos + 1], &indices[pos], (size_t)(k - 1 - pos) * sizeof(int));
            top[pos] = values[i];
            indices[pos] = i;
        }
    }
}

static void suppress_blank(float *logits, int n, int eot) { /* :450-455 */
    logits[eot] = -INFINITY;
    if (220 < n) logits[220] = -INFINITY;
}

static void apply_suppress(float *logits, const int *tokens, int n_tokens, int n) { /* :457-466 */
    if (!tokens) return;
    for (int i = 0; i < n_tokens; i++)
        if (tokens[i] >= 0 && tokens[i] < n) logits[tokens[i]] = -INFINITY;
}

static void ngram_block(float *logits, const int *gen, int count, int nn, int n) { /* :543-564 */
    if (count < nn - 1) return;
    for (int i = 0; i <= count - nn; i++) {
        int match = 1;
        for (int j = 0; j < nn - 1; j++)
            if (gen[i + j] != gen[count - (nn - 1) + j]) {
                match = 0;
                break;
            }
        if (match) {
            int blocked = gen[i + nn - 1];
            if (blocked >= 0 && blocked < n) logits[blocked] = -INFINITY;
        }
    }
}

void orc_apply_repetition_penalty(float *logits, const int *gen, int count, int n) { /* :472-476 */
    ngram_block(logits, gen, count, 3, n);
    ngram_block(logits, gen, count, 4, n);
}

void orc_apply_timestamp_rules(float *logits, const int *gen, int count, int ts_begin, int eot, int n,
                               int is_first) { /* :484-541 */
    if (ts_begin > 0 && ts_begin - 1 >= 0 && ts_begin - 1 < n) logits[ts_begin - 1] = -INFINITY;
    if (is_first) {
        for (int i = 0; i < ts_begin; i++) logits[i] = -INFINITY;
        int last_allowed = ts_begin + 50;
        for (int i = last_allowed + 1; i < n; i++) logits[i] = -INFINITY;
        return;
    }
    if (count == 0) return;
    int last_ts = gen[count - 1] >= ts_begin;
    int pen_ts = count < 2 || gen[count - 2] >= ts_begin;
    if (last_ts) {
        if (pen_ts) {
            for (int i = ts_begin; i < n; i++) logits[i] = -INFINITY;
        } else {
            for (int i = 0; i < eot; i++) logits[i] = -INFINITY;
        }
    }
    int lts = -1;
    for (int i = count - 1; i >= 0; i--)
        if (gen[i] >= ts_begin) {
            lts = gen[i];
            break;
        }
    if (lts >= 0) {
        int block_up_to = last_ts && !pen_ts ? lts + 1 : lts;
        for (int i = ts_begin; i < block_up_to && i < n; i++) logits[i] = -INFINITY;
    }
}

static int argmax(const float *a, int n) { /* :566-574 */
    int best = 0;
    for (int i = 1; i < n; i++)
        if (a[i] > a[best]) best = i;
    return best;
}

/* splitmix64: a seeded stand-in for Math.random() (the reference's draw is not
 * reproducible, so sampled tokens are compared statistically, not by value). */
static double next_uniform(uint64_t *s) {
    uint64_t z = (*s += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    z ^= z >> 31;
    return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

static int sample(float *logits, int n, float temperature, uint64_t *rng) { /* :576-598 */
    float max = -INFINITY;
    for (int i = 0; i < n; i++)
        if (logits[i] > max) max = logits[i];
    double sum = 0;
    for (int i = 0; i < n; i++) {
        double p = exp((double)((logits[i] - max) / temperature));
        logits[i] = (float)p;
        sum += p;
    }
    double r = next_uniform(rng) * sum;
    double cum = 0;
    for (int i = 0; i < n; i++) {
        cum += logits[i];
        if (cum >= r) return i;
    }
    return n - 1;
}

/* ------------------------------------------------------------------------ */
/* greedy / temperature decode (WhisperDecoder.java:161-204)                 */
/* ------------------------------------------------------------------------ */

int orc_decode(const orc_model *m, const float *xa, int n_audio_ctx, const int *prompt, int n_prompt, int eot,
               int max_tokens, const int *suppress, int n_suppress, int no_speech, float temperature, int ts_begin,
               uint64_t seed, int *out_tokens, int *out_len, double *out_sum_logprob, float *out_avg_logprob,
               float *out_no_speech_prob, int max_steps) {
    const int V = m->d.n_vocab;
    if (eot < 0 || eot >= V) return fail("orc_decode", "eot token out of range");
    if (orc_model_check(m)) return -1;
    orc_cache *cache = orc_cache_new(m, n_audio_ctx);
    float *logits = (float *)malloc((size_t)(n_prompt > 1 ? n_prompt : 1) * V * sizeof(float));
    float *last = (float *)malloc((size_t)V * sizeof(float));
    int *generated = (int *)malloc((size_t)(max_tokens > 0 ? max_tokens : 1) * sizeof(int));
    const int *cur = prompt;
    int n_cur = n_prompt, gen_count = 0, rc = 0, tok_buf = 0;
    double sum_lp = 0;
    float nsp = 0;
    uint64_t rng = seed;
    int steps = max_tokens;
    if (max_steps > 0 && max_steps < steps) steps = max_steps;
    double t_loop = 0;
    g_loop_seconds = 0;
    for (int step = 0; step < steps; step++) {
        if (step == 1) t_loop = now_seconds();
        if (orc_forward(m, cur, n_cur, xa, n_audio_ctx, cache, logits)) { rc = -1; break; }
        memcpy(last, logits + (size_t)(n_cur - 1) * V, (size_t)V * sizeof(float));
        if (step == 0) {
            nsp = (no_speech < 0 || no_speech >= V) ? 0.0f : softmax_at(logits, V, no_speech);
            suppress_blank(last, V, eot);
        }
        apply_suppress(last, suppress, n_suppress, V);
        orc_apply_repetition_penalty(last, generated, gen_count, V);
        if (ts_begin > 0) orc_apply_timestamp_rules(last, generated, gen_count, ts_begin, eot, V, step == 0);
        int best = temperature == 0.0f ? argmax(last, V) : sample(last, V, temperature, &rng);
        sum_lp += log_softmax_at(last, V, best);
        if (best == eot) break;
        generated[gen_count++] = best;
        tok_buf = best;
        cur = &tok_buf;
        n_cur = 1;
    }
    if (t_loop > 0) g_loop_seconds = now_seconds() - t_loop;
    if (rc == 0) {
        memcpy(out_tokens, generated, (size_t)gen_count * sizeof(int));
        *out_len = gen_count;
        *out_sum_logprob = sum_lp;
        *out_avg_logprob = gen_count > 0 ? (float)(sum_lp / gen_count) : 0.0f;
        *out_no_speech_prob = nsp;
    }
    free(logits); free(last); free(generated);
    orc_cache_free(cache);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* beam search (WhisperDecoder.java:214-394)                                 */
/* ------------------------------------------------------------------------ */

typedef struct { double score; int beam, token; } cand_t;

/* Double.compare(b, a) descending; List.sort is stable (insertion sort keeps order). */
static int dcompare(double a, double b) {
    if (a < b) return -1;
    if (a > b) return 1;
    int an = isnan(a), bn = isnan(b);
    if (an || bn) return an - bn;
    int as = signbit(a) != 0, bs = signbit(b) != 0; /* -0.0 < 0.0 */
    return bs - as;
}

/* Optional trace of the beam search for parity tests: every ranked candidate of every step as
 * (step, parent beam, token, score, outcome), outcome = new beam index (kept), -2 (finished) or
 * -1 (dropped or not reached).  Step 0 records the initial top-beam expansion (parent -1). */
static __thread double *g_trace = NULL;
static __thread long g_trace_cap = 0, g_trace_n = 0;

void orc_set_beam_trace(double *buf, long cap_entries) {
    g_trace = buf;
    g_trace_cap = buf ? cap_entries : 0;
    g_trace_n = 0;
}

long orc_beam_trace_count(void) { return g_trace_n; }

static void trace_put(int step, int parent, int token, double score, int outcome) {
    if (!g_trace || g_trace_n >= g_trace_cap) return;
    double *e = g_trace + g_trace_n * 5;
    e[0] = step;
    e[1] = parent;
    e[2] = token;
    e[3] = score;
    e[4] = outcome;
    g_trace_n++;
}

int orc_decode_beam(const orc_model *m, const float *xa, int n_audio_ctx, const int *prompt, int n_prompt, int eot,
                    int max_tokens, const int *suppress, int n_suppress, int no_speech, int ts_begin, int beam,
                    int *out_tokens, int *out_len, double *out_sum_logprob, float *out_avg_logprob,
                    float *out_no_speech_prob, int max_steps) {
    const int V = m->d.n_vocab;
    if (eot < 0 || eot >= V) return fail("orc_decode_beam", "eot token out of range");
    if (beam < 1 || beam > 32) return fail("orc_decode_beam", "beam size out of range");
    if (max_tokens < 1) return fail("orc_decode_beam", "max_tokens must be >= 1");
    if (orc_model_check(m)) return -1;
    int rc = 0;
    orc_cache **caches = (orc_cache **)calloc((size_t)beam, sizeof *caches);
    orc_cache **ncaches = (orc_cache **)calloc((size_t)beam, sizeof *ncaches);
    orc_cache *owner = orc_cache_new(m, n_audio_ctx);
    for (int b = 0; b < beam; b++) {
        caches[b] = orc_cache_new(m, n_audio_ctx);
        ncaches[b] = orc_cache_new(m, n_audio_ctx);
    }
    int *btok = (int *)calloc((size_t)beam * max_tokens, sizeof(int));
    int *nbtok = (int *)calloc((size_t)beam * max_tokens, sizeof(int));
    int *blen = (int *)calloc((size_t)beam, sizeof(int)), *nblen = (int *)calloc((size_t)beam, sizeof(int));
    double *blp = (double *)calloc((size_t)beam, sizeof(double)), *nblp = (double *)calloc((size_t)beam, sizeof(double));
    int *src = (int *)calloc((size_t)beam, sizeof(int));
    int fin_cap = beam * 2 + 2, fin_n = 0;
    int **fin_tok = (int **)calloc((size_t)fin_cap, sizeof(int *));
    int *fin_len = (int *)calloc((size_t)fin_cap, sizeof(int));
    double *fin_lp = (double *)calloc((size_t)fin_cap, sizeof(double));
    float *logits = (float *)malloc((size_t)(n_prompt > 1 ? n_prompt : 1) * V * sizeof(float));
    float *last = (float *)malloc((size_t)V * sizeof(float));
    float *lp = (float *)malloc((size_t)V * sizeof(float));
    int *top = (int *)malloc((size_t)(beam + 1) * sizeof(int));
    cand_t *cands = (cand_t *)malloc((size_t)beam * (beam + 1) * sizeof(cand_t));
    float nsp = 0;

    /* step 0 (:236-266) */
    if (orc_forward(m, prompt, n_prompt, xa, n_audio_ctx, caches[0], logits)) { rc = -1; goto done; }
    nsp = (no_speech < 0 || no_speech >= V) ? 0.0f : softmax_at(logits, V, no_speech);
    memcpy(last, logits + (size_t)(n_prompt - 1) * V, (size_t)V * sizeof(float));
    suppress_blank(last, V, eot);
    apply_suppress(last, suppress, n_suppress, V);
    compute_log_softmax(last, V, lp);
    topk_indices(lp, beam, V, top);
    /* The cross K/V projected by beam 0 are shared by every beam (:240-246); an
     * owner cache that is never swapped holds them. */
    for (int l = 0; l < owner->L; l++) {
        owner->xk[l] = caches[0]->xk[l];
        owner->xv[l] = caches[0]->xv[l];
    }
    owner->has_cross = 1;
    caches[0]->cross_shared = 1;
    for (int b = 0; b < beam; b++) {
        btok[(size_t)b * max_tokens] = top[b];
        blen[b] = 1;
        blp[b] = (double)lp[top[b]];
        trace_put(0, -1, top[b], blp[b], b);
        if (b > 0) {
            cache_share_cross(caches[b], owner);
            cache_copy_self(caches[b], caches[0]);
        }
    }

    int steps = max_tokens;
    if (max_steps > 0 && max_steps < steps) steps = max_steps;
    g_loop_seconds = 0;
    const double t_loop = now_seconds();
    for (int step = 1; step < steps; step++) { /* :269-367 */
        int nc = 0;
        for (int b = 0; b < beam; b++) {
            int *bt = btok + (size_t)b * max_tokens;
            if (bt[blen[b] - 1] == eot) continue;
            int last_tok = bt[blen[b] - 1];
            if (orc_forward(m, &last_tok, 1, xa, n_audio_ctx, caches[b], logits)) { rc = -1; goto done; }
            memcpy(last, logits, (size_t)V * sizeof(float));
            apply_suppress(last, suppress, n_suppress, V);
            orc_apply_repetition_penalty(last, bt, blen[b], V);
            if (ts_begin > 0) orc_apply_timestamp_rules(last, bt, blen[b], ts_begin, eot, V, 0);
            compute_log_softmax(last, V, lp);
            topk_indices(lp, beam + 1, V, top);
            for (int k = 0; k < beam + 1; k++) {
                cands[nc].score = blp[b] + (double)lp[top[k]];
                cands[nc].beam = b;
                cands[nc].token = top[k];
                nc++;
            }
        }
        if (nc == 0) break;
        for (int i = 1; i < nc; i++) { /* stable sort, score descending */
            cand_t c = cands[i];
            int j = i - 1;
            while (j >= 0 && dcompare(c.score, cands[j].score) > 0) {
                cands[j + 1] = cands[j];
                j--;
            }
            cands[j + 1] = c;
        }
        int saved = 0, walked = 0;
        for (int i = 0; i < nc; i++) {
            int sb = cands[i].beam, token = cands[i].token;
            walked = i + 1;
            if (token == eot) {
                trace_put(step, sb, token, cands[i].score, -2);
                if (fin_n == fin_cap) break; /* unreachable: loop breaks at beam finished */
                fin_tok[fin_n] = (int *)malloc((size_t)blen[sb] * sizeof(int) + 1);
                memcpy(fin_tok[fin_n], btok + (size_t)sb * max_tokens, (size_t)blen[sb] * sizeof(int));
                fin_len[fin_n] = blen[sb];
                fin_lp[fin_n] = cands[i].score;
                fin_n++;
                if (fin_n >= beam) break;
                continue;
            }
            trace_put(step, sb, token, cands[i].score, saved < beam ? saved : -1);
            if (saved >= beam) continue;
            memcpy(nbtok + (size_t)saved * max_tokens, btok + (size_t)sb * max_tokens, (size_t)blen[sb] * sizeof(int));
            nbtok[(size_t)saved * max_tokens + blen[sb]] = token;
            nblen[saved] = blen[sb] + 1;
            nblp[saved] = cands[i].score;
            src[saved] = sb;
            saved++;
        }
        for (int i = walked; i < nc; i++) trace_put(step, cands[i].beam, cands[i].token, cands[i].score, -1);
        if (saved == 0 || fin_n >= beam) break;
        /* :343-361 rearrange caches */
        for (int b = 0; b < saved; b++) {
            cache_share_cross(ncaches[b], owner);
            cache_copy_self(ncaches[b], caches[src[b]]);
        }
        for (int b = saved; b < beam; b++) {
            cache_share_cross(ncaches[b], owner);
            cache_copy_self(ncaches[b], ncaches[0]);
            memcpy(nbtok + (size_t)b * max_tokens, nbtok, (size_t)nblen[0] * sizeof(int));
            nblen[b] = nblen[0];
            nblp[b] = nblp[0];
        }
        { orc_cache **t = caches; caches = ncaches; ncaches = t; }
        { int *t = btok; btok = nbtok; nbtok = t; }
        { int *t = blen; blen = nblen; nblen = t; }
        { double *t = blp; blp = nblp; nblp = t; }
    }

    g_loop_seconds = now_seconds() - t_loop;
    if (fin_n < beam) { /* :370-377 */
        for (int b = 0; b < beam && fin_n < beam; b++) {
            fin_tok[fin_n] = (int *)malloc((size_t)blen[b] * sizeof(int) + 1);
            memcpy(fin_tok[fin_n], btok + (size_t)b * max_tokens, (size_t)blen[b] * sizeof(int));
            fin_len[fin_n] = blen[b];
            fin_lp[fin_n] = blp[b];
            fin_n++;
        }
    }
    {
        int best = 0;
        double best_score = -INFINITY;
        for (int i = 0; i < fin_n; i++) { /* :380-388 */
            double score = fin_lp[i] / (double)(fin_len[i] > 1 ? fin_len[i] : 1);
            if (score > best_score) {
                best_score = score;
                best = i;
            }
        }
        memcpy(out_tokens, fin_tok[best], (size_t)fin_len[best] * sizeof(int));
        *out_len = fin_len[best];
        *out_sum_logprob = fin_lp[best];
        *out_avg_logprob = fin_len[best] > 0 ? (float)(fin_lp[best] / fin_len[best]) : 0.0f;
        *out_no_speech_prob = nsp;
    }
done:
    orc_cache_free(owner);
    for (int b = 0; b < beam; b++) {
        orc_cache_free(caches[b]);
        orc_cache_free(ncaches[b]);
    }
    free(caches); free(ncaches);
    free(btok); free(nbtok); free(blen); free(nblen); free(blp); free(nblp); free(src);
    for (int i = 0; i < fin_n; i++) free(fin_tok[i]);
    free(fin_tok); free(fin_len); free(fin_lp);
    free(logits); free(last); free(lp); free(top); free(cands);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* audio encoder (WhisperEncoder.java:42-76; Conv1d.java:38-80)             */
/* ------------------------------------------------------------------------ */

typedef struct {
    float *attn_ln_w, *attn_ln_b;
    float *q_wt, *q_b, *k_wt, *v_wt, *v_b, *o_wt, *o_b; /* transposed (in, out); the key has no bias */
    float *mlp_ln_w, *mlp_ln_b;
    float *m0_wt, *m0_b, *m2_wt, *m2_b;
} orc_enc_layer;

struct orc_encoder {
    orc_enc_dims d;
    float *conv1_wt, *conv1_b; /* conv weights as (in * k, out): Conv1d's (out, in * k) weightMatrix transposed */
    float *conv2_wt, *conv2_b;
    float *pos;                /* (n_audio_ctx, d) */
    float *ln_w, *ln_b;        /* ln_post */
    orc_enc_layer *layers;
    float gelu_table[65536];
};

orc_encoder *orc_encoder_new(const orc_enc_dims *d) {
    if (!d || d->n_mels <= 0 || d->n_audio_ctx <= 0 || d->n_audio_state <= 0 || d->n_audio_head <= 0 ||
        d->n_audio_state % d->n_audio_head != 0 || d->n_audio_state / d->n_audio_head != 64 || d->n_audio_layer <= 0) {
        fail("orc_encoder_new", "invalid dimensions");
        return NULL;
    }
    orc_encoder *e = (orc_encoder *)calloc(1, sizeof *e);
    if (!e) return NULL;
    e->d = *d;
    e->layers = (orc_enc_layer *)calloc((size_t)d->n_audio_layer, sizeof(orc_enc_layer));
    build_gelu_table(e->gelu_table);
    return e;
}

void orc_encoder_free(orc_encoder *e) {
    if (!e) return;
    for (int i = 0; i < e->d.n_audio_layer; i++) {
        float **p = (float **)&e->layers[i];
        for (size_t j = 0; j < sizeof(orc_enc_layer) / sizeof(float *); j++) free(p[j]);
    }
    free(e->layers);
    free(e->conv1_wt); free(e->conv1_b); free(e->conv2_wt); free(e->conv2_b);
    free(e->pos); free(e->ln_w); free(e->ln_b);
    free(e);
}

int orc_encoder_set_tensor(orc_encoder *e, const char *name, const float *data, long n) {
    const int d = e->d.n_audio_state, nm = e->d.n_mels;
    if (strncmp(name, "encoder.", 8) != 0) return 1;
    const char *s = name + 8;
#define EXPECT(cnt)                                                                      \
    do {                                                                                 \
        if (n != (long)(cnt)) return fail("orc_encoder_set_tensor: wrong element count", name); \
    } while (0)
    struct { const char *nm; float **dst; int rows, cols; } top[] = {
        {"conv1.weight", &e->conv1_wt, d, nm * 3}, {"conv1.bias", &e->conv1_b, 0, d},
        {"conv2.weight", &e->conv2_wt, d, d * 3}, {"conv2.bias", &e->conv2_b, 0, d},
        {"positional_embedding", &e->pos, 0, e->d.n_audio_ctx * d},
        {"ln_post.weight", &e->ln_w, 0, d}, {"ln_post.bias", &e->ln_b, 0, d},
    };
    float **dst = NULL;
    int rows = 0, cols = 0;
    for (size_t i = 0; i < sizeof top / sizeof top[0] && !dst; i++)
        if (!strcmp(s, top[i].nm)) dst = top[i].dst, rows = top[i].rows, cols = top[i].cols;
    if (!dst) {
        int li = -1, off = 0;
        if (sscanf(s, "blocks.%d.%n", &li, &off) != 1 || li < 0 || li >= e->d.n_audio_layer)
            return fail("orc_encoder_set_tensor: unknown tensor", name);
        orc_enc_layer *L = &e->layers[li];
        struct { const char *nm; float **dst; int rows, cols; } tab[] = {
            {"attn_ln.weight", &L->attn_ln_w, 0, d}, {"attn_ln.bias", &L->attn_ln_b, 0, d},
            {"attn.query.weight", &L->q_wt, d, d}, {"attn.query.bias", &L->q_b, 0, d},
            {"attn.key.weight", &L->k_wt, d, d},
            {"attn.value.weight", &L->v_wt, d, d}, {"attn.value.bias", &L->v_b, 0, d},
            {"attn.out.weight", &L->o_wt, d, d}, {"attn.out.bias", &L->o_b, 0, d},
            {"mlp_ln.weight", &L->mlp_ln_w, 0, d}, {"mlp_ln.bias", &L->mlp_ln_b, 0, d},
            {"mlp.0.weight", &L->m0_wt, 4 * d, d}, {"mlp.0.bias", &L->m0_b, 0, 4 * d},
            {"mlp.2.weight", &L->m2_wt, d, 4 * d}, {"mlp.2.bias", &L->m2_b, 0, d},
        };
        for (size_t i = 0; i < sizeof tab / sizeof tab[0] && !dst; i++)
            if (!strcmp(s + off, tab[i].nm)) dst = tab[i].dst, rows = tab[i].rows, cols = tab[i].cols;
        if (!dst) return fail("orc_encoder_set_tensor: unknown tensor", name);
    }
    free(*dst);
    if (rows == 0) {
        EXPECT(cols);
        *dst = dup_f32(data, n);
    } else {
        EXPECT((long)rows * cols);
        *dst = dup_transposed(data, rows, cols);
    }
    return *dst ? 0 : fail("orc_encoder_set_tensor: out of memory", name);
#undef EXPECT
}

int orc_encoder_check(const orc_encoder *e) {
    if (!e->conv1_wt || !e->conv1_b || !e->conv2_wt || !e->conv2_b) return fail("weight not found", "encoder.conv");
    if (!e->pos) return fail("weight not found", "encoder.positional_embedding");
    if (!e->ln_w || !e->ln_b) return fail("weight not found", "encoder.ln_post");
    for (int i = 0; i < e->d.n_audio_layer; i++) {
        const orc_enc_layer *L = &e->layers[i];
        if (!L->attn_ln_w || !L->attn_ln_b || !L->q_wt || !L->q_b || !L->k_wt || !L->v_wt || !L->v_b || !L->o_wt ||
            !L->o_b || !L->mlp_ln_w || !L->mlp_ln_b || !L->m0_wt || !L->m0_b || !L->m2_wt || !L->m2_b)
            return fail("weight not found", "encoder.blocks");
    }
    return 0;
}

/* Conv1d.forward (:38-47): im2col (:49-64) as rows colT[t][ic * k + kk] = in(ic, t * stride - pad + kk)
 * (zero outside), then the (out, in * k) weight matrix times col, summed over ic * k + kk ascending
 * (Tensor.java:460-489), then the bias (:66-80).  in(ic, i) = src[ic * in_ld + i] for a channel-major
 * source (the mel input), src[i * in_ld + ic] for a time-major one (conv1's output).  y: (out_len, out). */
static void conv1d_k3(const float *src, int in_ch, int in_len, int in_ld, int time_major, int stride, int out_ch,
                      const float *wt, const float *bias, float *y) {
    const int pad = 1, k = 3, out_len = (in_len + 2 * pad - k) / stride + 1, R = in_ch * k;
    float *col = (float *)malloc((size_t)out_len * R * sizeof(float));
    for (int t = 0; t < out_len; t++)
        for (int ic = 0; ic < in_ch; ic++)
            for (int kk = 0; kk < k; kk++) {
                const int i = t * stride - pad + kk;
                float v = 0.0f;
                if (i >= 0 && i < in_len) v = time_major ? src[(size_t)i * in_ld + ic] : src[(size_t)ic * in_ld + i];
                col[(size_t)t * R + ic * k + kk] = v;
            }
    linear(col, out_len, R, wt, bias, out_ch, y);
    free(col);
}

int orc_encoder_forward(const orc_encoder *e, const float *mel, float *out) {
    if (!e || !mel || !out) return fail("orc_encoder_forward", "null argument");
    if (orc_encoder_check(e)) return -1;
    const int d = e->d.n_audio_state, T = e->d.n_audio_ctx, H = e->d.n_audio_head, nm = e->d.n_mels;
    const int T1 = 2 * T; /* mel frames; conv2 (stride 2) halves them */
    float *y1 = (float *)malloc((size_t)T1 * d * sizeof(float));
    float *x = (float *)malloc((size_t)T * d * sizeof(float));
    float *h = (float *)malloc((size_t)T * d * sizeof(float));
    float *q = (float *)malloc((size_t)T * d * sizeof(float));
    float *kk = (float *)malloc((size_t)T * d * sizeof(float));
    float *v = (float *)malloc((size_t)T * d * sizeof(float));
    float *att = (float *)malloc((size_t)T * d * sizeof(float));
    float *m = (float *)malloc((size_t)T * 4 * d * sizeof(float));
    const int nthr = g_threads > 1 ? g_threads : 1;
    float *scores = (float *)malloc((size_t)T * nthr * sizeof(float));
    int rc = 0;
    if (!y1 || !x || !h || !q || !kk || !v || !att || !m || !scores) {
        rc = fail("orc_encoder_forward", "out of memory");
        goto done;
    }
    /* conv1 + GELU, conv2 + GELU (WhisperEncoder.java:47-54), transpose, + positional embedding (:56-58) */
    conv1d_k3(mel, nm, T1, T1, 0, 1, d, e->conv1_wt, e->conv1_b, y1);
    gelu_inplace(e->gelu_table, y1, (long)T1 * d);
    conv1d_k3(y1, d, T1, d, 1, 2, d, e->conv2_wt, e->conv2_b, x);
    gelu_inplace(e->gelu_table, x, (long)T * d);
    for (long i = 0; i < (long)T * d; i++) x[i] = x[i] + e->pos[i];
    /* blocks (:60-70): ResidualAttentionBlock.forwardWithAttn without cross-attention, mask or cache */
    for (int l = 0; l < e->d.n_audio_layer; l++) {
        const orc_enc_layer *L = &e->layers[l];
        layer_norm(x, T, d, L->attn_ln_w, L->attn_ln_b, 1e-5f, h);
        linear(h, T, d, L->q_wt, L->q_b, d, q);
        linear(h, T, d, L->k_wt, NULL, d, kk);
        linear(h, T, d, L->v_wt, L->v_b, d, v);
        attn_job aj = {q, kk, v, att, d, H, T, -1, (float)(1.0 / sqrt(64.0)), scores, T};
        if (g_threads > 1) par_for(T * H, attn_self_job, &aj);
        else for (int th = 0; th < T * H; th++) attn_self_job(&aj, th);
        linear(att, T, d, L->o_wt, L->o_b, d, h);
        for (long i = 0; i < (long)T * d; i++) x[i] = h[i] + x[i];  /* attnOut[0].addInPlace(x) */
        layer_norm(x, T, d, L->mlp_ln_w, L->mlp_ln_b, 1e-5f, h);
        linear(h, T, d, L->m0_wt, L->m0_b, 4 * d, m);
        gelu_inplace(e->gelu_table, m, (long)T * 4 * d);
        linear(m, T, 4 * d, L->m2_wt, L->m2_b, d, q);
        for (long i = 0; i < (long)T * d; i++) x[i] = x[i] + q[i];  /* result.addInPlace(mlpOut) */
    }
    layer_norm(x, T, d, e->ln_w, e->ln_b, 1e-5f, out); /* ln_post (:72) */
done:
    free(y1); free(x); free(h); free(q); free(kk); free(v); free(att); free(m); free(scores);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* log-mel front end (FeatureExtractor.java:68-160 extract + padOrTrim,     */
/* :248-320 Bluestein / radix-2 FFT, :322-328 Hann window)                  */
/* ------------------------------------------------------------------------ */

/* :282-320 radix-2 FFT, twiddles by recurrence in float (as the Java loop does) */
static void fft_radix2(float *re, float *im, int n) {
    for (int i = 1, j = 0; i < n; i++) {
        int bit = n >> 1;
        while (j & bit) {
            j ^= bit;
            bit >>= 1;
        }
        j ^= bit;
        if (i < j) {
            float t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
    for (int len = 2; len <= n; len <<= 1) {
        const double angle = -2.0 * M_PI / len;
        const float wre = (float)cos(angle), wim = (float)sin(angle);
        for (int i = 0; i < n; i += len) {
            float cre = 1.0f, cim = 0.0f;
            for (int j = 0; j < len / 2; j++) {
                const int a = i + j, b = i + j + len / 2;
                const float ure = re[a], uim = im[a];
                const float vre = re[b] * cre - im[b] * cim;
                const float vim = re[b] * cim + im[b] * cre;
                re[a] = ure + vre;
                im[a] = uim + vim;
                re[b] = ure - vre;
                im[b] = uim - vim;
                const float ncre = cre * wre - cim * wim;
                cim = cre * wim + cim * wre;
                cre = ncre;
            }
        }
    }
}

/* :200-280 Bluestein for a non-power-of-two n (Whisper's n_fft = 400) */
static void fft_bluestein(float *re, float *im, int n) {
    int m = 1;
    while (m < 2 * n - 1) m <<= 1;
    float *cre = (float *)calloc((size_t)n, sizeof(float)), *cim = (float *)calloc((size_t)n, sizeof(float));
    float *are = (float *)calloc((size_t)m, sizeof(float)), *aim = (float *)calloc((size_t)m, sizeof(float));
    float *bre = (float *)calloc((size_t)m, sizeof(float)), *bim = (float *)calloc((size_t)m, sizeof(float));
    for (int k = 0; k < n; k++) {
        const double angle = -M_PI * (double)(((long long)k * k) % (2LL * n)) / n;
        cre[k] = (float)cos(angle);
        cim[k] = (float)sin(angle);
    }
    for (int k = 0; k < n; k++) {
        are[k] = re[k] * cre[k] + im[k] * cim[k];
        aim[k] = im[k] * cre[k] - re[k] * cim[k];
    }
    bre[0] = cre[0];
    bim[0] = cim[0];
    for (int k = 1; k < n; k++) {
        bre[k] = bre[m - k] = cre[k];
        bim[k] = bim[m - k] = cim[k];
    }
    fft_radix2(are, aim, m);
    fft_radix2(bre, bim, m);
    for (int k = 0; k < m; k++) {
        const float tr = are[k] * bre[k] - aim[k] * bim[k];
        const float ti = are[k] * bim[k] + aim[k] * bre[k];
        are[k] = tr;
        aim[k] = ti;
    }
    for (int k = 0; k < m; k++) aim[k] = -aim[k];
    fft_radix2(are, aim, m);
    const float inv_m = 1.0f / m;
    for (int k = 0; k < m; k++) {
        are[k] *= inv_m;
        aim[k] *= -inv_m;
    }
    for (int k = 0; k < n; k++) {
        re[k] = are[k] * cre[k] + aim[k] * cim[k];
        im[k] = aim[k] * cre[k] - are[k] * cim[k];
    }
    free(cre); free(cim); free(are); free(aim); free(bre); free(bim);
}

int orc_log_mel(const float *audio, int n_samples, const float *filters, int n_mels, int n_bins, int hop,
                int out_frames, float *out) {
    const int n_fft = (n_bins - 1) * 2, pad = n_fft / 2;
    if ((!audio && n_samples > 0) || !filters || !out || n_samples < 0 || n_mels <= 0 || n_bins < 2 || hop <= 0 ||
        out_frames <= 0)
        return fail("orc_log_mel", "bad argument");
    const int len = n_samples < n_fft ? n_fft : n_samples; /* :75-79 short inputs padded to n_fft */
    const int plen = len + 2 * pad;
    float *padded = (float *)calloc((size_t)plen, sizeof(float));
    if (n_samples > 0) memcpy(padded + pad, audio, (size_t)n_samples * sizeof(float));
    float *window = (float *)malloc((size_t)n_fft * sizeof(float));
    for (int i = 0; i < n_fft; i++) window[i] = 0.5f * (1.0f - (float)cos(2.0 * M_PI * i / n_fft));
    const int frames = 1 + (plen - n_fft) / hop;
    float *mag = (float *)malloc((size_t)n_bins * frames * sizeof(float));
    float *re = (float *)malloc((size_t)n_fft * sizeof(float)), *im = (float *)malloc((size_t)n_fft * sizeof(float));
    for (int t = 0; t < frames; t++) {
        for (int i = 0; i < n_fft; i++) {
            re[i] = padded[(size_t)t * hop + i] * window[i];
            im[i] = 0.0f;
        }
        if ((n_fft & (n_fft - 1)) == 0) fft_radix2(re, im, n_fft);
        else fft_bluestein(re, im, n_fft);
        for (int f = 0; f < n_bins; f++) mag[(size_t)f * frames + t] = re[f] * re[f] + im[f] * im[f];
    }
    float *spec = (float *)malloc((size_t)n_mels * frames * sizeof(float));
    float gmax = -INFINITY;
    for (int mm = 0; mm < n_mels; mm++)
        for (int t = 0; t < frames; t++) {
            float sum = 0.0f;
            for (int f = 0; f < n_bins; f++) sum += filters[(size_t)mm * n_bins + f] * mag[(size_t)f * frames + t];
            const float v = (float)log10(fmax((double)sum, 1e-10));
            spec[(size_t)mm * frames + t] = v;
            if (v > gmax) gmax = v;
        }
    const float floor_v = gmax - 8.0f;
    float vmin = INFINITY;
    for (long i = 0; i < (long)n_mels * frames; i++) {
        spec[i] = ((spec[i] > floor_v ? spec[i] : floor_v) + 4.0f) / 4.0f;
        if (spec[i] < vmin) vmin = spec[i];
    }
    /* padOrTrim (:130-160): the first out_frames frames, or padded with the spectrogram's minimum */
    for (int mm = 0; mm < n_mels; mm++)
        for (int t = 0; t < out_frames; t++)
            out[(size_t)mm * out_frames + t] = t < frames ? spec[(size_t)mm * frames + t] : vmin;
    free(padded); free(window); free(mag); free(re); free(im); free(spec);
    return 0;
}
