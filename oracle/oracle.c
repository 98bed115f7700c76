/*
 * CPU oracle for the mlxd decoder step -- TEST INFRASTRUCTURE ONLY.
 * See oracle.h. Each function names the reference lines it restates.
 * Built with -ffp-contract=off so every float operation rounds where the
 * source says it does.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------ bf16 */

static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline float rbf(float f) { return bf2f(f2bf(f)); }

static inline float sdt_get(const void *p, int sdtype, size_t i) {
    return sdtype == ORC_F32 ? ((const float *)p)[i] : bf2f(((const uint16_t *)p)[i]);
}

/* --------------------------------------------------------- own exp (Cody-Waite)
 * exp(x) = 2^n * exp(r), n = rint(x*log2(e)), r = x - n*ln2 with ln2 split in a
 * high part with trailing zero bits and a low part (Cody & Waite, 1980);
 * exp(r) by its degree-7 Taylor polynomial in Horner form with fmaf. Valid
 * on [-104, 88.7]; 0 below, +inf above. The CUDA sampler evaluates the same
 * expression, so both sides produce identical bits. */
float orc_expf(float x) {
    if (!(x > -104.0f)) return 0.0f;          /* also -inf and NaN */
    if (x > 88.72f) return INFINITY;
    float n = rintf(x * 1.44269504f);
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.428606765330187e-06f, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    int a = ni / 2, b = ni - a;
    uint32_t ua = (uint32_t)(a + 127) << 23, ub = (uint32_t)(b + 127) << 23;
    float sa, sb;
    memcpy(&sa, &ua, 4);
    memcpy(&sb, &ub, 4);
    return (p * sa) * sb;
}

/* ------------------------------------------------------------ thread pool */

static int g_threads = 0;
void orc_set_threads(int n) { g_threads = n; }
int orc_get_threads(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef void (*range_fn)(void *ctx, int lo, int hi);
typedef struct { range_fn fn; void *ctx; int lo, hi; } prange;
static void *prange_run(void *a) {
    prange *p = (prange *)a;
    p->fn(p->ctx, p->lo, p->hi);
    return NULL;
}
/* split [0, n) into contiguous ranges over the pool */
static void parallel_for(int n, int min_chunk, range_fn fn, void *ctx) {
    int nt = orc_get_threads();
    if (nt > n / (min_chunk > 0 ? min_chunk : 1)) nt = n / (min_chunk > 0 ? min_chunk : 1);
    if (nt <= 1) {
        fn(ctx, 0, n);
        return;
    }
    if (nt > 256) nt = 256;
    pthread_t th[256];
    prange pr[256];
    int step = (n + nt - 1) / nt;
    int launched = 0;
    for (int t = 0; t < nt; t++) {
        int lo = t * step, hi = lo + step < n ? lo + step : n;
        if (lo >= hi) break;
        pr[t] = (prange){fn, ctx, lo, hi};
        if (t == 0) continue;
        if (pthread_create(&th[t], NULL, prange_run, &pr[t]) != 0) {
            fn(ctx, lo, hi);
            pr[t].fn = NULL;
        }
        launched = t + 1;
    }
    fn(ctx, pr[0].lo, pr[0].hi);
    for (int t = 1; t < launched; t++)
        if (pr[t].fn) pthread_join(th[t], NULL);
}

/* ---------------------------------------------------------------- tensors */

typedef struct {
    char name[128];
    int dtype, ndim;
    int64_t shape[4];
    void *data;
    size_t bytes;
} tensor;

typedef struct {
    int quant;           /* 1: 4-bit affine triplet, 0: dense bf16 */
    int rows, cols;      /* out, in */
    int sdtype;
    const uint32_t *w;
    const void *s, *b;
    const uint16_t *dense;
} linear_t;

typedef struct {
    linear_t q, k, v, o, gate, up, down;
    const uint16_t *ln1, *ln2, *qn, *kn;
} layer_t;

struct orc_model {
    orc_config c;
    tensor *t;
    int nt, capt;
    layer_t *L;
    linear_t embed, lm;
    const uint16_t *norm;
    float *freqs;        /* llama3 custom freqs [D/2] or NULL */
};

struct orc_kv {
    int layers, hkv, d, cap;
    int *off;
    uint16_t **k, **v;   /* [hkv][cap][d] */
};

static size_t dtype_size(int dt) { return dt == ORC_BF16 ? 2 : 4; }

orc_model *orc_model_new(const orc_config *cfg) {
    orc_model *m = calloc(1, sizeof(*m));
    if (!m) return NULL;
    m->c = *cfg;
    return m;
}

int orc_model_set_tensor(orc_model *m, const char *name, int dtype,
                         const int64_t *shape, int ndim, const void *data) {
    if (!m || !name || ndim < 1 || ndim > 4) return -1;
    if (m->nt == m->capt) {
        int nc = m->capt ? m->capt * 2 : 64;
        tensor *nt = realloc(m->t, (size_t)nc * sizeof(tensor));
        if (!nt) return -1;
        m->t = nt;
        m->capt = nc;
    }
    tensor *t = &m->t[m->nt];
    memset(t, 0, sizeof(*t));
    snprintf(t->name, sizeof(t->name), "%s", name);
    t->dtype = dtype;
    t->ndim = ndim;
    size_t n = 1;
    for (int i = 0; i < ndim; i++) {
        t->shape[i] = shape[i];
        n *= (size_t)shape[i];
    }
    t->bytes = n * dtype_size(dtype);
    t->data = malloc(t->bytes ? t->bytes : 1);
    if (!t->data) return -1;
    memcpy(t->data, data, t->bytes);
    m->nt++;
    return 0;
}

static const tensor *find(const orc_model *m, const char *name) {
    for (int i = 0; i < m->nt; i++)
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}

/* weights_get_triplet (weights.c:1053-1088): {base}.weight plus optional
   scales/biases; a partial triplet is an error. */
static int get_linear(const orc_model *m, const char *base, linear_t *out,
                      char *err, int errlen) {
    char n[200];
    snprintf(n, sizeof n, "%s.weight", base);
    const tensor *w = find(m, n);
    snprintf(n, sizeof n, "%s.scales", base);
    const tensor *s = find(m, n);
    snprintf(n, sizeof n, "%s.biases", base);
    const tensor *b = find(m, n);
    memset(out, 0, sizeof(*out));
    if (!w) {
        snprintf(err, errlen, "missing %s.weight", base);
        return -1;
    }
    if ((s == NULL) != (b == NULL)) {
        snprintf(err, errlen, "partial quantized triplet %s", base);
        return -1;
    }
    if (s) {
        if (w->dtype != ORC_U32 || w->ndim != 2) {
            snprintf(err, errlen, "%s.weight: quantized weight must be U32 2-D", base);
            return -1;
        }
        out->quant = 1;
        out->rows = (int)w->shape[0];
        out->cols = (int)w->shape[1] * 8;
        out->w = w->data;
        out->s = s->data;
        out->b = b->data;
        out->sdtype = s->dtype;
        int g = m->c.qgroup;
        if (s->shape[0] != out->rows || s->shape[1] * g != out->cols) {
            snprintf(err, errlen, "%s: scales shape mismatch", base);
            return -1;
        }
    } else {
        if (w->dtype != ORC_BF16 || w->ndim != 2) {
            snprintf(err, errlen, "%s.weight: dense weight must be BF16 2-D", base);
            return -1;
        }
        out->rows = (int)w->shape[0];
        out->cols = (int)w->shape[1];
        out->dense = w->data;
    }
    return 0;
}

static const uint16_t *get_vec(const orc_model *m, const char *name, int n,
                               char *err, int errlen) {
    const tensor *t = find(m, name);
    if (!t || t->dtype != ORC_BF16 || (int)t->shape[0] != n) {
        snprintf(err, errlen, "missing or bad %s", name);
        return NULL;
    }
    return t->data;
}

/* fwd_rope_llama3_freqs (forward.c:323-358): fp64 host math, f32 result */
int orc_rope_llama3_freqs(float theta, float factor, float lo, float hi,
                          int orig_max, int head_dim, float *out) {
    if (head_dim < 2 || (head_dim & 1) || factor <= 0 || orig_max <= 0 ||
        lo <= 0 || hi <= lo)
        return -1;
    double base = theta, f = factor, lf = lo, hf = hi, old = orig_max;
    double low_wl = old / lf, high_wl = old / hf;
    for (int i = 0; i < head_dim / 2; i++) {
        double fr = pow(base, 2.0 * i / (double)head_dim);
        double wl = 2.0 * M_PI * fr;
        if (wl > low_wl) {
            fr = fr * f;
        } else if (wl > high_wl) {
            double sm = (old / wl - lf) / (hf - lf);
            fr = fr / ((1.0 - sm) / f + sm);
        }
        out[i] = (float)fr;
    }
    return 0;
}

int orc_model_finalize(orc_model *m, char *err, int errlen) {
    const orc_config *c = &m->c;
    char nb[200];
    char dummy[8];
    if (!err) { err = dummy; errlen = sizeof dummy; }
    m->L = calloc((size_t)c->layers, sizeof(layer_t));
    if (!m->L) return -1;
    if (get_linear(m, "model.embed_tokens", &m->embed, err, errlen)) return -1;
    if (c->tie) m->lm = m->embed;
    else if (get_linear(m, "lm_head", &m->lm, err, errlen)) return -1;
    if (!(m->norm = get_vec(m, "model.norm.weight", c->hidden, err, errlen))) return -1;
    for (int l = 0; l < c->layers; l++) {
        layer_t *L = &m->L[l];
        const char *sfx[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                              "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj",
                              "mlp.down_proj"};
        linear_t *dst[7] = {&L->q, &L->k, &L->v, &L->o, &L->gate, &L->up, &L->down};
        for (int i = 0; i < 7; i++) {
            snprintf(nb, sizeof nb, "model.layers.%d.%s", l, sfx[i]);
            if (get_linear(m, nb, dst[i], err, errlen)) return -1;
        }
        snprintf(nb, sizeof nb, "model.layers.%d.input_layernorm.weight", l);
        if (!(L->ln1 = get_vec(m, nb, c->hidden, err, errlen))) return -1;
        snprintf(nb, sizeof nb, "model.layers.%d.post_attention_layernorm.weight", l);
        if (!(L->ln2 = get_vec(m, nb, c->hidden, err, errlen))) return -1;
        if (c->qk_norm) {
            snprintf(nb, sizeof nb, "model.layers.%d.self_attn.q_norm.weight", l);
            if (!(L->qn = get_vec(m, nb, c->head_dim, err, errlen))) return -1;
            snprintf(nb, sizeof nb, "model.layers.%d.self_attn.k_norm.weight", l);
            if (!(L->kn = get_vec(m, nb, c->head_dim, err, errlen))) return -1;
        }
        int qrows = c->n_heads * c->head_dim * (c->attn_gate ? 2 : 1);
        if (L->q.rows != qrows || L->q.cols != c->hidden ||
            L->k.rows != c->n_kv_heads * c->head_dim ||
            L->v.rows != c->n_kv_heads * c->head_dim ||
            L->o.cols != c->n_heads * c->head_dim || L->o.rows != c->hidden ||
            L->gate.rows != c->inter || L->up.rows != c->inter ||
            L->down.cols != c->inter || L->down.rows != c->hidden) {
            snprintf(err, errlen, "layer %d: projection shape mismatch", l);
            return -1;
        }
    }
    if (c->rope_llama3) {
        m->freqs = malloc(sizeof(float) * (size_t)(c->head_dim / 2));
        if (orc_rope_llama3_freqs(c->rope_theta, c->rope_factor, c->rope_lo, c->rope_hi,
                                  c->rope_orig_max, c->head_dim, m->freqs)) {
            snprintf(err, errlen, "bad llama3 rope parameters");
            return -1;
        }
    }
    return 0;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    for (int i = 0; i < m->nt; i++) free(m->t[i].data);
    free(m->t);
    free(m->L);
    free(m->freqs);
    free(m);
}

orc_kv *orc_kv_new(const orc_model *m, int capacity) {
    orc_kv *kv = calloc(1, sizeof(*kv));
    if (!kv) return NULL;
    kv->layers = m->c.layers;
    kv->hkv = m->c.n_kv_heads;
    kv->d = m->c.head_dim;
    kv->cap = capacity;
    kv->off = calloc((size_t)kv->layers, sizeof(int));
    kv->k = calloc((size_t)kv->layers, sizeof(uint16_t *));
    kv->v = calloc((size_t)kv->layers, sizeof(uint16_t *));
    for (int l = 0; l < kv->layers; l++) {
        size_t n = (size_t)kv->hkv * (size_t)capacity * (size_t)kv->d;
        kv->k[l] = calloc(n, 2);
        kv->v[l] = calloc(n, 2);
        if (!kv->k[l] || !kv->v[l]) { orc_kv_free(kv); return NULL; }
    }
    return kv;
}

void orc_kv_free(orc_kv *kv) {
    if (!kv) return;
    for (int l = 0; l < kv->layers; l++) {
        if (kv->k) free(kv->k[l]);
        if (kv->v) free(kv->v[l]);
    }
    free(kv->k);
    free(kv->v);
    free(kv->off);
    free(kv);
}

/* kvcache_layer_offset (kvcache.c:25-28) */
int orc_kv_offset(const orc_kv *kv, int layer) {
    if (!kv || layer < 0 || layer >= kv->layers) return -1;
    return kv->off[layer];
}

int orc_kv_read(const orc_kv *kv, int layer, int is_value, uint16_t *out) {
    if (!kv || layer < 0 || layer >= kv->layers) return -1;
    int off = kv->off[layer];
    const uint16_t *src = is_value ? kv->v[layer] : kv->k[layer];
    for (int h = 0; h < kv->hkv; h++)
        memcpy(out + (size_t)h * off * kv->d, src + (size_t)h * kv->cap * kv->d,
               (size_t)off * kv->d * 2);
    return 0;
}

/* ---------------------------------------------------------------- linear */

void orc_dequantize_row(const uint32_t *w, const void *s, const void *b,
                        int sdtype, int cols, int group, float *out) {
    for (int j = 0; j < cols; j++) {
        uint32_t q = (w[j >> 3] >> ((j & 7) * 4)) & 0xFu;
        float sc = sdt_get(s, sdtype, (size_t)(j / group));
        float bi = sdt_get(b, sdtype, (size_t)(j / group));
        out[j] = fmaf(sc, (float)q, bi);
    }
}

/* f64 -> bf16 with one correct rounding (to nearest, ties to even): the
   value is first cut to f32 by rounding toward zero with the lowest bit set
   when anything was cut (round to odd, 24 >= 8 + 2 bits), then rounded to
   bf16; this equals the direct rounding of the f64 value. */
static uint16_t d2bf(double d) {
    if (isnan(d)) return 0x7fc0;
    float f = (float)d;
    if (fabs((double)f) > fabs(d)) f = nextafterf(f, 0.0f);
    if ((double)f != d) {
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= 1u;
        memcpy(&f, &u, 4);
    }
    return f2bf(f);
}

/* The projection arithmetic shared with the CUDA kernels (decode GEMV,
   prefill GEMM, tensor-parallel shards): mlx's quantized_matmul
   (forward.c:17-32, cast to bf16 :46-54) computes per output row
       sum over groups g of  s_g * sum_k(x_k q_k) + b_g * sum_k(x_k)
   (qmv) in f32 with an order of its own, which is not observable. Here the
   order is taken out of the result:
   - each group's 64 (or 32) inputs are written in fixed point on the grid of
     their largest magnitude: E_g = exponent of max|x_k| over the group
     (clamped at -100), X_k = round-to-nearest-even(x_k * 2^(20 - E_g)),
     |X_k| < 2^21; a bf16 input within 13 binades of its group's largest is
     exact, a smaller one is rounded at 2^(E_g - 21) (below the rounding of
     an f32 sum of the products);
   - P_g = sum_k q_k X_k and T_g = sum_k X_k are exact integers;
   - the row's value sum_g (s_g P_g + b_g T_g) 2^(E_g - 20) is summed in f64,
     where every product is exact (bf16 scales) and the sum is exact while it
     spans at most 53 bits (otherwise correct to 2^-53, so the order of the
     sum shows only in outputs within 2^-52 of a bf16 rounding boundary);
   - the row value is rounded once to bf16 (d2bf).
   The grid depends on the group only, so a shard of whole groups (the
   row-parallel projections of tensor parallelism) gives the same integers,
   and prefill (S > 1) and decode (S = 1) give the same bits. A group
   holding a non-finite input gives NaN. Dense bf16 weights: the f64 sum of
   the exact products x_k w_k, rounded once. */
static void fixed_point_groups(const float *xf, int n, int G, int32_t *X, double *pf, int64_t *T,
                               uint8_t *bad) {
    int ng = n / G;
    for (int g = 0; g < ng; g++) {
        const float *xg = xf + (size_t)g * G;
        uint32_t eb = 0;
        for (int k = 0; k < G; k++) {
            uint32_t u;
            memcpy(&u, &xg[k], 4);
            uint32_t e = (u >> 23) & 0xffu;
            if (e > eb) eb = e;
        }
        bad[g] = eb == 0xffu;
        int E = (int)eb - 127;
        if (E < -100) E = -100;
        float sc = ldexpf(1.0f, 20 - E);
        int64_t t = 0;
        for (int k = 0; k < G; k++) {
            int32_t v = bad[g] ? 0 : (int32_t)nearbyintf(xg[k] * sc);
            X[(size_t)g * G + k] = v;
            t += v;
        }
        T[g] = t;
        pf[g] = ldexp(1.0, E - 20);
    }
}

typedef struct {
    const uint16_t *x;
    int S, in, out;
    const linear_t *W;
    int group, exact;
    uint16_t *y;
    /* per token: fixed-point inputs [S][in], group factors/sums [S][ng] */
    const int32_t *X;
    const double *pf;
    const int64_t *T;
    const uint8_t *bad;
} lin_ctx;

/* exact: the arithmetic above. !exact: mlx's qmm tile semantics (weights
   dequantized and rounded to bf16, f32 dot in element order), kept for the
   quantized-matmul known-answer test only. */
static void lin_rows(void *vc, int r0, int r1) {
    lin_ctx *c = vc;
    const linear_t *W = c->W;
    int in = c->in, G = c->group;
    int ng = W->quant ? in / G : 0;
    float *wrow = malloc(sizeof(float) * (size_t)in);
    float *xf = malloc(sizeof(float) * (size_t)in * (size_t)c->S);
    int32_t *q = malloc(sizeof(int32_t) * (size_t)in);
    for (int s = 0; s < c->S; s++)
        for (int j = 0; j < in; j++) xf[(size_t)s * in + j] = bf2f(c->x[(size_t)s * in + j]);
    for (int r = r0; r < r1; r++) {
        if (W->quant && c->exact) {
            const uint32_t *wr = W->w + (size_t)r * (in / 8);
            for (int j = 0; j < in; j++) q[j] = (int32_t)((wr[j >> 3] >> ((j & 7) * 4)) & 0xFu);
            for (int s = 0; s < c->S; s++) {
                const int32_t *X = c->X + (size_t)s * in;
                const double *pf = c->pf + (size_t)s * ng;
                const int64_t *T = c->T + (size_t)s * ng;
                const uint8_t *bad = c->bad + (size_t)s * ng;
                double acc = 0.0;
                int nan = 0;
                for (int g = 0; g < ng; g++) {
                    int32_t P = 0;
                    for (int k = 0; k < G; k++) P += q[g * G + k] * X[g * G + k];
                    double sc = (double)sdt_get(W->s, W->sdtype, (size_t)r * ng + g);
                    double bi = (double)sdt_get(W->b, W->sdtype, (size_t)r * ng + g);
                    acc += sc * ((double)P * pf[g]);
                    acc += bi * ((double)T[g] * pf[g]);
                    nan |= bad[g];
                }
                c->y[(size_t)s * c->out + r] = nan ? 0x7fc0 : d2bf(acc);
            }
            continue;
        }
        if (W->quant) {
            const uint32_t *wr = W->w + (size_t)r * (in / 8);
            orc_dequantize_row(wr, (const char *)W->s + (size_t)r * ng * dtype_size(W->sdtype),
                               (const char *)W->b + (size_t)r * ng * dtype_size(W->sdtype),
                               W->sdtype, in, G, wrow);
            for (int j = 0; j < in; j++) wrow[j] = rbf(wrow[j]);
            for (int s = 0; s < c->S; s++) {
                float acc = 0.f;
                for (int j = 0; j < in; j++) acc = fmaf(xf[(size_t)s * in + j], wrow[j], acc);
                c->y[(size_t)s * c->out + r] = f2bf(acc);
            }
            continue;
        }
        for (int s = 0; s < c->S; s++) {
            double acc = 0.0;
            for (int j = 0; j < in; j++)
                acc += (double)xf[(size_t)s * in + j] * (double)bf2f(W->dense[(size_t)r * in + j]);
            c->y[(size_t)s * c->out + r] = d2bf(acc);
        }
    }
    free(wrow);
    free(xf);
    free(q);
}

static void run_linear(const linear_t *W, const uint16_t *x, int S, int group, int exact,
                       uint16_t *y) {
    lin_ctx c = {x, S, W->cols, W->rows, W, group, exact, y, NULL, NULL, NULL, NULL};
    int32_t *X = NULL;
    double *pf = NULL;
    int64_t *T = NULL;
    uint8_t *bad = NULL;
    if (W->quant && exact) {
        int in = W->cols, ng = in / group;
        X = malloc(sizeof(int32_t) * (size_t)S * in);
        pf = malloc(sizeof(double) * (size_t)S * ng);
        T = malloc(sizeof(int64_t) * (size_t)S * ng);
        bad = malloc((size_t)S * ng);
        float *xf = malloc(sizeof(float) * (size_t)in);
        for (int s = 0; s < S; s++) {
            for (int j = 0; j < in; j++) xf[j] = bf2f(x[(size_t)s * in + j]);
            fixed_point_groups(xf, in, group, X + (size_t)s * in, pf + (size_t)s * ng,
                               T + (size_t)s * ng, bad + (size_t)s * ng);
        }
        free(xf);
        c.X = X;
        c.pf = pf;
        c.T = T;
        c.bad = bad;
    }
    parallel_for(W->rows, 16, lin_rows, &c);
    free(X);
    free(pf);
    free(T);
    free(bad);
}

static void linear(const linear_t *W, const uint16_t *x, int S, int group, uint16_t *y) {
    run_linear(W, x, S, group, 1, y);
}

void orc_qlinear(const uint16_t *x, int S, int in, int out, const uint32_t *w,
                 const void *scales, const void *biases, int sdtype, int group,
                 int exact_dequant, uint16_t *y) {
    linear_t W = {1, out, in, sdtype, w, scales, biases, NULL};
    run_linear(&W, x, S, group, exact_dequant, y);
}

void orc_dense_linear(const uint16_t *x, int S, int in, int out,
                      const uint16_t *w, uint16_t *y) {
    linear_t W = {0, out, in, 0, NULL, NULL, NULL, w};
    run_linear(&W, x, S, 0, 1, y);
}

/* ------------------------------------------------------------- norm, rope */

/* mlx_fast_rms_norm (forward.c:208): f32 sum of squares, precise rsqrt,
   normalised value rounded to bf16, then times the weight in bf16. */
/* Sum of squares with a fixed association (mlx's own is not observable):
   T = 256 (n >= 1024), 128 (n >= 256) or 32 strided partial sums, partial
   tau taking elements tau, tau+T, ... with fused multiply-adds; each group
   of 32 partials combined by the butterfly v_l += v_(l^o), o = 16,8,4,2,1;
   the group totals added in order. The CUDA kernels use this association. */
static float sumsq_assoc(const uint16_t *x, int n) {
    int T = n >= 1024 ? 256 : (n >= 256 ? 128 : 32);
    float part[256];
    for (int t = 0; t < T; t++) {
        float a = 0.f;
        for (int i = t; i < n; i += T) {
            float v = bf2f(x[i]);
            a = fmaf(v, v, a);
        }
        part[t] = a;
    }
    float tot = 0.f;
    for (int w = 0; w < T / 32; w++) {
        float v[32], nv[32];
        for (int l = 0; l < 32; l++) v[l] = part[w * 32 + l];
        for (int o = 16; o > 0; o >>= 1) {
            for (int l = 0; l < 32; l++) nv[l] = v[l] + v[l ^ o];
            for (int l = 0; l < 32; l++) v[l] = nv[l];
        }
        tot += v[0];
    }
    return tot;
}

void orc_rmsnorm(const uint16_t *x, int rows, int n, const uint16_t *w,
                 float eps, uint16_t *y) {
    for (int r = 0; r < rows; r++) {
        const uint16_t *xr = x + (size_t)r * n;
        float acc = sumsq_assoc(xr, n);
        float inv = 1.0f / sqrtf(acc / (float)n + eps);
        for (int i = 0; i < n; i++)
            y[(size_t)r * n + i] = f2bf(bf2f(w[i]) * rbf(bf2f(xr[i]) * inv));
    }
}

/* mlx_fast_rope traditional=false (forward.c:433, :453): rotate-half on the
   first `dims` features; angle = pos * inv_freq, inv_freq =
   2^(-(i/half)*log2(theta)) or 1/freqs[i]; output rounded to bf16. */
void orc_rope(uint16_t *x, int D, int dims, int pos, float theta,
              const float *freqs) {
    (void)D;
    int half = dims / 2;
    float lb = log2f(theta);
    float L = (float)pos;
    for (int i = 0; i < half; i++) {
        float inv = freqs ? 1.0f / freqs[i] : exp2f(-((float)i / (float)half) * lb);
        float th = L * inv;
        float cs = cosf(th), sn = sinf(th);
        float x1 = bf2f(x[i]), x2 = bf2f(x[i + half]);
        float a = x1 * cs - x2 * sn;
        float b = x1 * sn + x2 * cs;
        x[i] = f2bf(a);
        x[i + half] = f2bf(b);
    }
}

/* --------------------------------------------------------------- attention */

typedef struct {
    const orc_model *m;
    orc_kv *kv;
    int layer, S, kv_len, view0;
    const uint16_t *q;      /* [S][Hq][D] roped */
    uint16_t *out;          /* [S][Hq][D] */
    int composed;
    int local;
} att_ctx;

/* mlx_fast_scaled_dot_product_attention (forward.c:713-731). Fused kernels
   (mlx sdpa_vector / steel attention, head_dim 64/96/128/256) keep scores,
   softmax and the output accumulator in f32. Other head dims take mlx's
   composed fallback: q scaled in bf16, bf16 scores, precise softmax rounded
   to bf16, bf16 matmul with v. Masking: causal bottom-right aligned; local
   layers add the window rule 0 <= (kv_len-S+i) - j < window
   (fwd_sliding_window_mask, forward.c:241-292); decode on a local layer
   attends to the last `window` rows (kvcache.c:147-148). */
/* Key range [j0, j1) of query row i (S queries, kv_len keys): causal,
   bottom-right aligned; with a window, prefill rows allow
   0 <= (kv_len - S + i) - j < window (fwd_sliding_window_mask,
   forward.c:241-292) and a decode row sees the last `window` keys (the
   kvcache_update view trim, kvcache.c:147-148). */
static void attn_range(int S, int kv_len, int i, int window, int *j0, int *j1) {
    int qpos = kv_len - S + i;
    *j1 = qpos + 1;
    *j0 = 0;
    if (window > 0) {
        if (S == 1) *j0 = kv_len > window ? kv_len - window : 0;
        else if (qpos - window + 1 > 0) *j0 = qpos - window + 1;
    }
}

int orc_window_mask(int q_len, int kv_len, int window, uint8_t *out) {
    if (q_len <= 0 || kv_len <= 0 || window < 0 || q_len > kv_len) return -1;
    for (int i = 0; i < q_len; i++) {
        int j0, j1;
        attn_range(q_len, kv_len, i, window, &j0, &j1);
        for (int j = 0; j < kv_len; j++) out[(size_t)i * kv_len + j] = j >= j0 && j < j1;
    }
    return 0;
}

/* Attention arithmetic shared with the CUDA kernels (decode and prefill).
   Fused head dims (mlx sdpa_vector / steel attention keep scores, softmax
   and the accumulator in f32; their order is not observable, so one is
   fixed here):
     q_d' = f32(scale * q_d), scale = 1/sqrtf(D);
     z_j  = fmaf chain over d = 0..D-1 of q_d' * k_jd (one rounding per step);
     keys are cut into blocks of 64 absolute positions [64b, 64b + 64); a
     block with attended keys has m_b = max z_j over them, p_j = own
     exp(z_j - m_b), l_b = in-order f32 sum of p_j and o_bd = fmaf chain of
     p_j v_jd in key order;
     the blocks merge in key order into f64 (M, L, O_d): the first sets
     M = m_b, L = l_b, O_d = o_bd; a block with m_b > M scales the sums by
     s = own exp(M - m_b) (f32) first: L = fma(L, s, l_b), O_d = fma(O_d, s,
     o_bd), M = m_b; any other adds with e = own exp(m_b - M): L = fma(l_b,
     e, L), O_d = fma(o_bd, e, O_d);
     out_d = bf16(O_d / L), the f64 quotient rounded once.
   Every block is complete before the merge sees it, so a decode step can
   split the blocks over CTAs and merge their results in one place, and a
   prefill tile needs one pass over the keys.
   The blocks are absolute positions, so a decode step and a prefill row at
   the same position give the same bits. Other head dims take mlx's composed
   fallback: q scaled in bf16, bf16 scores (fmaf chain rounded once), precise
   softmax (in-order f32 sum) rounded to bf16, bf16 output of an fmaf chain
   over the keys. */
static void att_heads(void *vc, int h0, int h1) {
    att_ctx *c = vc;
    const orc_config *cf = &c->m->c;
    int D = cf->head_dim, Hq = cf->n_heads, rep = Hq / cf->n_kv_heads;
    float scale = 1.0f / sqrtf((float)D);
    int T = c->kv_len;
    float *sc = malloc(sizeof(float) * (size_t)T);
    float *qf = malloc(sizeof(float) * (size_t)D);
    float *o = malloc(sizeof(float) * (size_t)D);
    double *O = malloc(sizeof(double) * (size_t)D);
    for (int h = h0; h < h1; h++) {
        int kh = h / rep;
        const uint16_t *K = c->kv->k[c->layer] + (size_t)kh * c->kv->cap * D;
        const uint16_t *V = c->kv->v[c->layer] + (size_t)kh * c->kv->cap * D;
        for (int i = 0; i < c->S; i++) {
            const uint16_t *q = c->q + ((size_t)i * Hq + h) * D;
            int j0, j1;
            attn_range(c->S, T, i, c->local ? cf->window : 0, &j0, &j1);
            if (c->composed) {
                float sbf = rbf(scale);
                for (int d = 0; d < D; d++) qf[d] = rbf(sbf * bf2f(q[d]));
            } else {
                for (int d = 0; d < D; d++) qf[d] = scale * bf2f(q[d]);
            }
            float mx = -INFINITY;
            for (int j = j0; j < j1; j++) {
                float a = 0.f;
                for (int d = 0; d < D; d++) a = fmaf(qf[d], bf2f(K[(size_t)j * D + d]), a);
                if (c->composed) a = rbf(a);
                sc[j] = a;
                if (a > mx) mx = a;
            }
            uint16_t *dst = c->out + ((size_t)i * Hq + h) * D;
            if (c->composed) {
                float l = 0.f;
                for (int j = j0; j < j1; j++) {
                    sc[j] = orc_expf(sc[j] - mx);
                    l += sc[j];
                }
                for (int d = 0; d < D; d++) o[d] = 0.f;
                for (int j = j0; j < j1; j++) {
                    float p = rbf(sc[j] / l);
                    for (int d = 0; d < D; d++) o[d] = fmaf(p, bf2f(V[(size_t)j * D + d]), o[d]);
                }
                for (int d = 0; d < D; d++) dst[d] = f2bf(o[d]);
                continue;
            }
            /* blocks of 64 absolute positions in key order, each with its
               own maximum, merged into f64 running sums */
            double L = 0.0;
            float M = -INFINITY;
            for (int d = 0; d < D; d++) O[d] = 0.0;
            for (int b0 = j0; b0 < j1;) {
                int b1 = (b0 / 64 + 1) * 64;
                if (b1 > j1) b1 = j1;
                float mb = -INFINITY;
                for (int j = b0; j < b1; j++) mb = sc[j] > mb ? sc[j] : mb;
                float l = 0.f;
                for (int d = 0; d < D; d++) o[d] = 0.f;
                for (int j = b0; j < b1; j++) {
                    float p = orc_expf(sc[j] - mb);
                    l += p;
                    for (int d = 0; d < D; d++) o[d] = fmaf(p, bf2f(V[(size_t)j * D + d]), o[d]);
                }
                if (M == -INFINITY) {
                    M = mb;
                    L = (double)l;
                    for (int d = 0; d < D; d++) O[d] = (double)o[d];
                } else if (mb > M) {
                    double s = (double)orc_expf(M - mb);
                    M = mb;
                    L = fma(L, s, (double)l);
                    for (int d = 0; d < D; d++) O[d] = fma(O[d], s, (double)o[d]);
                } else {
                    double e = (double)orc_expf(mb - M);
                    L = fma((double)l, e, L);
                    for (int d = 0; d < D; d++) O[d] = fma((double)o[d], e, O[d]);
                }
                b0 = b1;
            }
            for (int d = 0; d < D; d++) dst[d] = d2bf(O[d] / L);
        }
    }
    free(sc);
    free(qf);
    free(o);
    free(O);
}

static int fused_head_dim(int D) { return D == 64 || D == 96 || D == 128 || D == 256; }

/* ---------------------------------------------------------------- forward */

/* mlx Sigmoid on a bf16 array (mlx metal unary op): y = 1/(1+exp(|x|)),
   result y for x < 0 and 1-y otherwise, every intermediate a bf16 value
   (bfloat16 arithmetic rounds after each operation). This staging, and not
   a single f32 sigmoid rounded once, is what reproduces the reference's
   pinned greedy sequence (tests/test_engine_gpu.c:21-23). */
static float sigmoid_bf16(float g) {
    float e = rbf(orc_expf(fabsf(g)));
    float y = rbf(1.0f / rbf(1.0f + e));
    return g < 0.0f ? y : rbf(1.0f - y);
}

/* fwd_decoder_layer (forward.c:1288-1380) with fwd_attention (:495-795) and
   fwd_swiglu (:900-958); pre-norm block, bf16 at every mlx op boundary. */
static int layer_forward(orc_model *m, orc_kv *kv, int l, uint16_t *h, int S) {
    const orc_config *c = &m->c;
    layer_t *L = &m->L[l];
    int H = c->hidden, D = c->head_dim, Hq = c->n_heads, Hk = c->n_kv_heads;
    int G = c->qgroup;
    int qw = Hq * D * (c->attn_gate ? 2 : 1);
    int off = kv->off[l];
    if (off + S > kv->cap) return -1;
    uint16_t *x = malloc(2 * (size_t)S * H);
    uint16_t *qraw = malloc(2 * (size_t)S * qw);
    uint16_t *q = malloc(2 * (size_t)S * Hq * D);
    uint16_t *gate = c->attn_gate ? malloc(2 * (size_t)S * Hq * D) : NULL;
    uint16_t *k = malloc(2 * (size_t)S * Hk * D);
    uint16_t *v = malloc(2 * (size_t)S * Hk * D);
    uint16_t *att = malloc(2 * (size_t)S * Hq * D);
    uint16_t *ao = malloc(2 * (size_t)S * H);
    uint16_t *g = malloc(2 * (size_t)S * c->inter);
    uint16_t *u = malloc(2 * (size_t)S * c->inter);
    uint16_t *mo = malloc(2 * (size_t)S * H);

    orc_rmsnorm(h, S, H, L->ln1, c->eps, x);
    linear(&L->q, x, S, G, qraw);
    linear(&L->k, x, S, G, k);
    linear(&L->v, x, S, G, v);
    for (int s = 0; s < S; s++)
        for (int hh = 0; hh < Hq; hh++) {
            const uint16_t *src = qraw + (size_t)s * qw + (size_t)hh * D * (c->attn_gate ? 2 : 1);
            memcpy(q + ((size_t)s * Hq + hh) * D, src, 2 * (size_t)D);
            if (gate) memcpy(gate + ((size_t)s * Hq + hh) * D, src + D, 2 * (size_t)D);
        }
    if (c->qk_norm) {
        orc_rmsnorm(q, S * Hq, D, L->qn, c->eps, q);
        orc_rmsnorm(k, S * Hk, D, L->kn, c->eps, k);
    }
    for (int s = 0; s < S; s++) {
        for (int hh = 0; hh < Hq; hh++)
            orc_rope(q + ((size_t)s * Hq + hh) * D, D, c->rope_dims, off + s, c->rope_theta, m->freqs);
        for (int hh = 0; hh < Hk; hh++)
            orc_rope(k + ((size_t)s * Hk + hh) * D, D, c->rope_dims, off + s, c->rope_theta, m->freqs);
    }
    /* kvcache_update (kvcache.c:98-180): append at offset */
    for (int s = 0; s < S; s++)
        for (int hh = 0; hh < Hk; hh++) {
            memcpy(kv->k[l] + ((size_t)hh * kv->cap + off + s) * D, k + ((size_t)s * Hk + hh) * D, 2 * (size_t)D);
            memcpy(kv->v[l] + ((size_t)hh * kv->cap + off + s) * D, v + ((size_t)s * Hk + hh) * D, 2 * (size_t)D);
        }
    kv->off[l] = off + S;
    int T = off + S;
    int local = c->window > 0;
    int view0 = (local && S == 1 && T > c->window) ? T - c->window : 0;
    att_ctx ac = {m, kv, l, S, T, view0, q, att, !fused_head_dim(D), local};
    parallel_for(Hq, 1, att_heads, &ac);
    if (gate) {
        /* attn * sigmoid(gate), each op rounded (forward.c:741-754) */
        size_t n = (size_t)S * Hq * D;
        for (size_t i = 0; i < n; i++) {
            float sg = sigmoid_bf16(bf2f(gate[i]));
            att[i] = f2bf(bf2f(att[i]) * sg);
        }
    }
    linear(&L->o, att, S, G, ao);
    for (size_t i = 0; i < (size_t)S * H; i++) h[i] = f2bf(bf2f(h[i]) + bf2f(ao[i]));
    orc_rmsnorm(h, S, H, L->ln2, c->eps, x);
    linear(&L->gate, x, S, G, g);
    linear(&L->up, x, S, G, u);
    for (size_t i = 0; i < (size_t)S * c->inter; i++) {
        float gv = bf2f(g[i]);
        float sg = sigmoid_bf16(gv);
        float si = rbf(gv * sg);
        g[i] = f2bf(si * bf2f(u[i]));
    }
    linear(&L->down, g, S, G, mo);
    for (size_t i = 0; i < (size_t)S * H; i++) h[i] = f2bf(bf2f(h[i]) + bf2f(mo[i]));
    free(x); free(qraw); free(q); free(gate); free(k); free(v); free(att);
    free(ao); free(g); free(u); free(mo);
    return 0;
}

/* fwd_embed (forward.c:65-147): take rows, dequantise, bf16 */
static void embed(const orc_model *m, const int32_t *ids, int S, uint16_t *h) {
    const orc_config *c = &m->c;
    int H = c->hidden;
    float *row = malloc(sizeof(float) * (size_t)H);
    for (int s = 0; s < S; s++) {
        int id = ids[s];
        if (m->embed.quant) {
            int ng = H / c->qgroup;
            size_t es = dtype_size(m->embed.sdtype);
            orc_dequantize_row(m->embed.w + (size_t)id * (H / 8),
                               (const char *)m->embed.s + (size_t)id * ng * es,
                               (const char *)m->embed.b + (size_t)id * ng * es,
                               m->embed.sdtype, H, c->qgroup, row);
            for (int j = 0; j < H; j++) h[(size_t)s * H + j] = f2bf(row[j]);
        } else {
            memcpy(h + (size_t)s * H, m->embed.dense + (size_t)id * H, 2 * (size_t)H);
        }
    }
    free(row);
}

static int forward_impl(orc_model *m, orc_kv *kv, const int32_t *ids, int S,
                        int want_logits, float *logits_out, uint16_t *hidden_out) {
    const orc_config *c = &m->c;
    int H = c->hidden;
    if (S <= 0) return -1;
    for (int s = 0; s < S; s++)
        if (ids[s] < 0 || ids[s] >= c->vocab) return -1;
    uint16_t *h = malloc(2 * (size_t)S * H);
    embed(m, ids, S, h);
    for (int l = 0; l < c->layers; l++)
        if (layer_forward(m, kv, l, h, S)) { free(h); return -1; }
    if (hidden_out) memcpy(hidden_out, h, 2 * (size_t)S * H);
    if (want_logits && logits_out) {
        uint16_t *xn = malloc(2 * (size_t)H);
        orc_rmsnorm(h + (size_t)(S - 1) * H, 1, H, m->norm, c->eps, xn);
        uint16_t *lg = malloc(2 * (size_t)c->vocab);
        linear(&m->lm, xn, 1, c->qgroup, lg);
        for (int i = 0; i < c->vocab; i++) logits_out[i] = bf2f(lg[i]);
        free(lg);
        free(xn);
    }
    free(h);
    return 0;
}

int orc_forward(orc_model *m, orc_kv *kv, const int32_t *ids, int S,
                int want_logits, float *logits_out) {
    return forward_impl(m, kv, ids, S, want_logits, logits_out, NULL);
}

int orc_forward_hidden(orc_model *m, orc_kv *kv, const int32_t *ids, int S,
                       uint16_t *hidden_out) {
    return forward_impl(m, kv, ids, S, 0, NULL, hidden_out);
}

/* ---------------------------------------------------------- quantisation */

/* mlx affine_quantize (mlx ops.cpp): per group, scale = (max-min)/15 with the
   sign chosen so the larger-magnitude edge maps exactly to an integer level,
   bias = that edge; q = clip(round((w - bias)/scale), 0, 15); element j of a
   row lives in word j/8 at nibble (j%8)*4, LSB first. */
void orc_affine_quantize(const float *w, int rows, int cols, int group,
                         uint32_t *wq, float *scales, float *biases) {
    const float n_bins = 15.0f, eps = 1e-7f;
    int ng = cols / group;
    for (int r = 0; r < rows; r++) {
        for (int g = 0; g < ng; g++) {
            const float *x = w + (size_t)r * cols + (size_t)g * group;
            float mx = x[0], mn = x[0];
            for (int j = 1; j < group; j++) {
                if (x[j] > mx) mx = x[j];
                if (x[j] < mn) mn = x[j];
            }
            int mask = fabsf(mn) > fabsf(mx);
            float sc = (mx - mn) / n_bins;
            if (sc < eps) sc = eps;
            if (!mask) sc = -sc;
            float edge = mask ? mn : mx;
            float q0 = rintf(edge / sc);
            if (q0 != 0.0f) sc = edge / q0;
            float bi = q0 == 0.0f ? 0.0f : edge;
            scales[(size_t)r * ng + g] = sc;
            biases[(size_t)r * ng + g] = bi;
            for (int j = 0; j < group; j++) {
                float qv = rintf((x[j] - bi) / sc);
                if (qv < 0) qv = 0;
                if (qv > n_bins) qv = n_bins;
                int col = g * group + j;
                uint32_t *word = &wq[(size_t)r * (cols / 8) + col / 8];
                if ((col & 7) == 0) *word = 0;
                *word |= ((uint32_t)qv & 0xFu) << ((col & 7) * 4);
            }
        }
    }
}

/* ---------------------------------------------------------------- sampler */

static int cmp_desc_f(const void *a, const void *b) {
    float x = *(const float *)a, y = *(const float *)b;
    return (x < y) - (x > y);
}

/* sampler_apply_top_k (sampler.c:97-122): keep x >= k-th largest (ties kept) */
void orc_top_k(float *x, int V, int k) {
    if (k <= 0 || k >= V) return;
    float *t = malloc(sizeof(float) * (size_t)V);
    memcpy(t, x, sizeof(float) * (size_t)V);
    qsort(t, (size_t)V, sizeof(float), cmp_desc_f);
    float cut = t[k - 1];
    for (int i = 0; i < V; i++)
        if (!(x[i] >= cut)) x[i] = -INFINITY;
    free(t);
}

/* Cumulative sums over the ascending order use one fixed association so the
   CUDA sampler reproduces them bit for bit: the n sorted positions are cut
   into NB = 1024 blocks of ceil(n/1024); a running f32 sum goes through the
   blocks in order and, inside a block, through its elements in order; the
   prefix entering a block is the running sum of the previous blocks' f32
   block totals, each block total being the in-order f32 sum of that block
   started from zero. For n <= 1024 this is the plain sequential sum. */
#define ORC_NB 1024
static void blocked_cumsum(const float *p, int n, float *cum, float *total) {
    int bs = (n + ORC_NB - 1) / ORC_NB;
    if (bs < 1) bs = 1;
    float prefix = 0.f;
    for (int b0 = 0; b0 < n; b0 += bs) {
        int b1 = b0 + bs < n ? b0 + bs : n;
        float run = prefix, bt = 0.f;
        for (int i = b0; i < b1; i++) {
            run += p[i];
            bt += p[i];
            if (cum) cum[i] = run;
        }
        prefix += bt;
    }
    if (total) *total = prefix;
}

typedef struct { float v; int i; } vi_t;
static int cmp_asc_vi(const void *a, const void *b) {
    const vi_t *x = a, *y = b;
    if (x->v < y->v) return -1;
    if (x->v > y->v) return 1;
    return (x->i > y->i) - (x->i < y->i);
}

/* ascending sort of (value, index); -inf first. Ties by ascending index. */
static vi_t *sorted_asc(const float *x, int V) {
    vi_t *s = malloc(sizeof(vi_t) * (size_t)V);
    for (int i = 0; i < V; i++) s[i] = (vi_t){x[i], i};
    qsort(s, (size_t)V, sizeof(vi_t), cmp_asc_vi);
    return s;
}

static float max_of(const float *x, int V) {
    float m = -INFINITY;
    for (int i = 0; i < V; i++)
        if (x[i] > m) m = x[i];
    return m;
}

/* sampler_apply_top_p (sampler.c:124-196): ascending sort, precise softmax,
   inclusive cumsum, cutoff = smallest sorted logit whose cumsum > 1-p,
   clamped to the max; keep x >= cutoff. p <= 0 keeps only the max. */
void orc_top_p(float *x, int V, float p) {
    if (p >= 1.0f) return;
    float mx = max_of(x, V);
    if (p <= 0.0f) {
        for (int i = 0; i < V; i++)
            if (!(x[i] >= mx)) x[i] = -INFINITY;
        return;
    }
    vi_t *s = sorted_asc(x, V);
    float *e = malloc(sizeof(float) * (size_t)V);
    float *cum = malloc(sizeof(float) * (size_t)V);
    for (int i = 0; i < V; i++) e[i] = orc_expf(s[i].v - mx);
    float z;
    blocked_cumsum(e, V, NULL, &z);
    for (int i = 0; i < V; i++) e[i] = e[i] / z;
    blocked_cumsum(e, V, cum, NULL);
    float thr = 1.0f - p;
    float cut = INFINITY;
    for (int i = 0; i < V; i++)
        if (cum[i] > thr) { cut = s[i].v; break; }
    if (cut > mx) cut = mx;
    for (int i = 0; i < V; i++)
        if (!(x[i] >= cut)) x[i] = -INFINITY;
    free(s);
    free(e);
    free(cum);
}

/* sampler_apply_min_p (sampler.c:198-232): keep x >= max + log(min_p) */
void orc_min_p(float *x, int V, float mp) {
    if (mp <= 0.0f) return;
    float thr = max_of(x, V) + logf(mp);
    for (int i = 0; i < V; i++)
        if (!(x[i] >= thr)) x[i] = -INFINITY;
}

/* SplitMix64 (Steele, Lea & Flood 2014) */
static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* uniform in [0,1) with 24 bits for draw `step` of stream `seed` */
static float draw_uniform(int seed, uint64_t step) {
    uint64_t k = splitmix64(((uint64_t)(uint32_t)seed << 32) ^ 0x6d6c7864ull);
    uint64_t r = splitmix64(k + step * 0x9E3779B97F4A7C15ull);
    return (float)(r >> 40) * (1.0f / 16777216.0f);
}

/* sampler_sample_lazy (sampler.c:269-380). Repetition penalty first
   (build-defined; the reference has none: mlx-lm's rule, x>0 ? x/p : x*p
   over the distinct ids among the last R context tokens, on the raw logits,
   applied before greedy and sampled draws alike as mlx-lm's logits
   processors are). Greedy below T=0.01: first maximum; logprob from the
   (penalised) raw logits. Otherwise logits/T in f32, top_k, top_p, min_p,
   then a categorical draw by
   inverse CDF over the ascending order (blocked sums, SplitMix64 uniform).
   mlx's categorical RNG stream is not reproducible here; the candidate set
   is. Logprob = x[tok] - logsumexp(x) on the (penalised) raw logits. */
int orc_sample(const float *logits, int V, const orc_sampling *sp,
               const int32_t *ctx, int n_ctx, uint64_t step,
               int32_t *tok_out, float *logprob_out, uint8_t *keep_out) {
    float *x = malloc(sizeof(float) * (size_t)V);
    memcpy(x, logits, sizeof(float) * (size_t)V);
    int greedy = sp->temperature < 0.01f;
    if (sp->repetition_penalty > 0.f && sp->repetition_penalty != 1.0f && ctx && n_ctx > 0) {
        int R = sp->repetition_context > 0 ? sp->repetition_context : n_ctx;
        int start = n_ctx > R ? n_ctx - R : 0;
        uint8_t *seen = calloc((size_t)V, 1);
        for (int i = start; i < n_ctx; i++) {
            int id = ctx[i];
            if (id < 0 || id >= V || seen[id]) continue;
            seen[id] = 1;
            x[id] = x[id] > 0.f ? x[id] / sp->repetition_penalty : x[id] * sp->repetition_penalty;
        }
        free(seen);
    }
    /* raw logprobs */
    float mx = max_of(x, V);
    double se = 0;
    for (int i = 0; i < V; i++) se += exp((double)x[i] - (double)mx);
    float lse = mx + (float)log(se);
    int tok = 0;
    if (greedy) {
        for (int i = 1; i < V; i++)
            if (x[i] > x[tok]) tok = i;
        if (keep_out) {
            memset(keep_out, 0, (size_t)V);
            keep_out[tok] = 1;
        }
    } else {
        float *s = malloc(sizeof(float) * (size_t)V);
        if (sp->temperature != 1.0f)
            for (int i = 0; i < V; i++) s[i] = x[i] / sp->temperature;
        else
            memcpy(s, x, sizeof(float) * (size_t)V);
        if (sp->top_k > 0) orc_top_k(s, V, sp->top_k);
        if (sp->top_p < 1.0f) orc_top_p(s, V, sp->top_p);
        if (sp->min_p > 0.0f) orc_min_p(s, V, sp->min_p);
        if (keep_out)
            for (int i = 0; i < V; i++) keep_out[i] = s[i] > -INFINITY;
        float m2 = max_of(s, V);
        vi_t *so = sorted_asc(s, V);
        float *e = malloc(sizeof(float) * (size_t)V);
        float *cum = malloc(sizeof(float) * (size_t)V);
        for (int i = 0; i < V; i++) e[i] = orc_expf(so[i].v - m2);
        float z;
        blocked_cumsum(e, V, cum, &z);
        float u = draw_uniform(sp->seed < 0 ? 0 : sp->seed, step);
        float target = u * z;
        int pick = V - 1;
        for (int i = 0; i < V; i++)
            if (cum[i] > target && e[i] > 0.f) { pick = i; break; }
        tok = so[pick].i;
        free(so); free(e); free(cum); free(s);
    }
    *tok_out = tok;
    if (logprob_out) *logprob_out = x[tok] - lse;
    free(x);
    return 0;
}

/* ------------------------------------------------------------ generate */

/* handle_generate_real (engine.c:360-602) without the actor: chunked
   prefill of prompt[:-1], seed forward of the last prompt token, then one
   sample + one forward per emitted token; EOS ends without emitting. */
int orc_generate(orc_model *m, const int32_t *prompt, int n, int max_new,
                 const orc_sampling *sp, int prefill_chunk, int32_t *out,
                 float *logprobs, float *margins) {
    const orc_config *c = &m->c;
    if (n <= 0 || max_new <= 0) return 0;
    if (n > c->max_pos) return -2;
    if (prefill_chunk <= 0) prefill_chunk = 512;
    orc_kv *kv = orc_kv_new(m, n + max_new + 1);
    if (!kv) return -1;
    int V = c->vocab;
    float *lg = malloc(sizeof(float) * (size_t)V);
    int32_t *ctx = malloc(sizeof(int32_t) * (size_t)(n + max_new + 1));
    memcpy(ctx, prompt, sizeof(int32_t) * (size_t)n);
    int n_ctx = n;
    int rc = 0, emitted = 0;
    for (int pos = 0; pos < n - 1; pos += prefill_chunk) {
        int len = (n - 1 - pos) < prefill_chunk ? (n - 1 - pos) : prefill_chunk;
        if (orc_forward(m, kv, prompt + pos, len, 0, NULL)) { rc = -1; goto done; }
    }
    if (orc_forward(m, kv, prompt + n - 1, 1, 1, lg)) { rc = -1; goto done; }
    while (emitted < max_new) {
        int32_t tok;
        float lp;
        orc_sample(lg, V, sp, ctx, n_ctx, (uint64_t)emitted, &tok, &lp, NULL);
        if (margins) {
            float a = -INFINITY, b = -INFINITY;
            for (int i = 0; i < V; i++) {
                if (lg[i] > a) { b = a; a = lg[i]; }
                else if (lg[i] > b) b = lg[i];
            }
            margins[emitted] = a - b;
        }
        int eos = 0;
        for (int e = 0; e < c->n_eos; e++)
            if (c->eos[e] == tok) eos = 1;
        if (eos) break;
        out[emitted] = tok;
        if (logprobs) logprobs[emitted] = lp;
        ctx[n_ctx++] = tok;
        emitted++;
        if (emitted < max_new)
            if (orc_forward(m, kv, &tok, 1, 1, lg)) { rc = -1; goto done; }
    }
    rc = emitted;
done:
    free(lg);
    free(ctx);
    orc_kv_free(kv);
    return rc;
}

/* ------------------------------------------------------ synthetic weights */
/* The benchmark's seeded MLX-format weights, restated here so the CPU
   baseline can build them without the CUDA library: element e of stream
   `seed` is the Irwin-Hall sum of 12 uniforms (24-bit halves of six
   SplitMix64 outputs, Steele/Lea/Flood 2014) scaled to N(0, std) and rounded
   to bf16; each group is MLX affine-quantized (mlx ops.cpp affine_quantize:
   the larger-magnitude edge maps exactly to a level). The CUDA library's
   generator produces the same bits (a test compares them). */
static uint64_t syn_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint16_t syn_value(uint64_t seed, uint64_t e, float std) {
    uint64_t base = syn_mix(seed ^ 0x5EED5EED5EEDull) + e * 6ull;
    uint32_t sum = 0;
    for (int i = 0; i < 6; i++) {
        uint64_t r = syn_mix(base + (uint64_t)i);
        sum += (uint32_t)(r >> 40) + (uint32_t)((r >> 16) & 0xFFFFFFu);
    }
    float z = (float)sum * (1.0f / 16777216.0f) - 6.0f;
    return f2bf(z * std);
}

typedef struct {
    uint32_t *w;
    uint16_t *s, *b;
    int cols, G;
    uint64_t seed;
    float std;
} syn_ctx;

static void syn_rows(void *vc, int r0, int r1) {
    syn_ctx *c = vc;
    const int G = c->G, ng = c->cols / G;
    float v[64];
    for (int r = r0; r < r1; r++)
        for (int g = 0; g < ng; g++) {
            float mx = -INFINITY, mn = INFINITY;
            for (int j = 0; j < G; j++) {
                v[j] = bf2f(syn_value(c->seed, (uint64_t)r * c->cols + (uint64_t)g * G + j, c->std));
                mx = v[j] > mx ? v[j] : mx;
                mn = v[j] < mn ? v[j] : mn;
            }
            int neg_edge = fabsf(mn) > fabsf(mx);
            float sc = (mx - mn) / 15.0f;
            if (sc < 1e-7f) sc = 1e-7f;
            if (!neg_edge) sc = -sc;
            float edge = neg_edge ? mn : mx;
            float q0 = nearbyintf(edge / sc);
            if (q0 != 0.0f) sc = edge / q0;
            float bi = q0 == 0.0f ? 0.0f : edge;
            uint32_t *wo = c->w + (size_t)r * (c->cols / 8) + (size_t)g * (G / 8);
            for (int k8 = 0; k8 < G / 8; k8++) {
                uint32_t word = 0;
                for (int k = 0; k < 8; k++) {
                    float q = nearbyintf((v[k8 * 8 + k] - bi) / sc);
                    q = q < 0.f ? 0.f : (q > 15.f ? 15.f : q);
                    word |= ((uint32_t)q & 0xFu) << (4 * k);
                }
                wo[k8] = word;
            }
            c->s[(size_t)r * ng + g] = f2bf(sc);
            c->b[(size_t)r * ng + g] = f2bf(bi);
        }
}

int orc_synth_quantized(uint32_t *w, uint16_t *scales, uint16_t *biases, int rows, int cols,
                        int group, uint64_t seed, float std) {
    if ((group != 32 && group != 64) || cols % group || rows <= 0) return -1;
    syn_ctx c = {w, scales, biases, cols, group, seed, std};
    parallel_for(rows, 16, syn_rows, &c);
    return 0;
}

void orc_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float std, float constant) {
    for (size_t i = 0; i < n; i++) out[i] = std > 0.f ? syn_value(seed, i, std) : f2bf(constant);
}

/* Benchmark helper: stand in for a prefill of n positions by filling the
   cache with seeded N(0, 1) keys and values (ring slot p % capacity) and
   setting every layer's offset to n, so decode can be timed at context n
   without the prefill's CPU time. */
int orc_kv_fill_synth(orc_kv *kv, int n, uint64_t seed) {
    if (!kv || n < 0) return -1;
    for (int l = 0; l < kv->layers; l++) {
        for (int h = 0; h < kv->hkv; h++)
            for (int p = 0; p < n; p++) {
                size_t row = ((size_t)h * kv->cap + (size_t)(p % kv->cap)) * kv->d;
                uint64_t e = (((uint64_t)l * kv->hkv + h) * (uint64_t)n + p) * (uint64_t)kv->d;
                for (int j = 0; j < kv->d; j++) {
                    kv->k[l][row + j] = syn_value(seed, 2 * (e + j), 1.0f);
                    kv->v[l][row + j] = syn_value(seed, 2 * (e + j) + 1, 1.0f);
                }
            }
        kv->off[l] = n;
    }
    return 0;
}
