/* libmlxd_engine: device arrays, the bridge calls of the generate loop, the
   engine model, the KV cache and the sampler over libmlxd_cuda (the surface
   is described in mlxd_engine.h). */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "mlxd_engine.h"

/* ------------------------------------------------------------ arrays */

typedef struct {
    void  *p;
    size_t bytes;
    int    refs;
} ebuf;

typedef struct {
    ebuf    *b;            /* NULL for a sampler subkey */
    int      dtype;        /* mlx_dtype */
    int      ndim;
    int      shape[4];
    int      is_key;
    int      seed;
    uint64_t step;
} earr;

static size_t dt_size(int dt) { return dt == MLX_BFLOAT16 ? 2 : 4; }

static size_t numel(const earr *a) {
    size_t n = 1;
    for (int i = 0; i < a->ndim; i++) n *= (size_t)a->shape[i];
    return n;
}

/* buffers released by mlx_array_free, reused by size; all work runs on one
   stream, so a reused buffer's old readers precede its new writers */
#define CACHE_MAX 64
static ebuf *g_cache[CACHE_MAX];
static int g_ncache;
static mlx_stream g_stream;

mlx_stream mlxbridge_gpu_stream(void) {
    if (!g_stream.ctx) {
        void *s = NULL;
        if (mlxd_cuda_stream_create(&s) == 0) g_stream.ctx = s;
    }
    return g_stream;
}

static void *stream_ptr(void) { return mlxbridge_gpu_stream().ctx; }

static ebuf *buf_get(size_t bytes) {
    if (bytes == 0) bytes = 16;
    for (int i = 0; i < g_ncache; i++)
        if (g_cache[i]->bytes == bytes) {
            ebuf *b = g_cache[i];
            g_cache[i] = g_cache[--g_ncache];
            b->refs = 1;
            return b;
        }
    ebuf *b = calloc(1, sizeof(ebuf));
    if (!b) return NULL;
    if (mlxd_cuda_alloc(&b->p, bytes)) {
        free(b);
        return NULL;
    }
    b->bytes = bytes;
    b->refs = 1;
    return b;
}

static void buf_put(ebuf *b) {
    if (!b || --b->refs > 0) return;
    if (g_ncache < CACHE_MAX) {
        g_cache[g_ncache++] = b;
        return;
    }
    mlxd_cuda_synchronize(stream_ptr());
    mlxd_cuda_free(b->p);
    free(b);
}

int mlxbridge_clear_cache(void) {
    if (g_ncache) mlxd_cuda_synchronize(stream_ptr());
    for (int i = 0; i < g_ncache; i++) {
        mlxd_cuda_free(g_cache[i]->p);
        free(g_cache[i]);
    }
    g_ncache = 0;
    return 0;
}

static mlx_array wrap(earr *a) { return (mlx_array){a}; }

static earr *new_arr(int dtype, int ndim, const int *shape) {
    if (ndim < 0 || ndim > 4) return NULL;
    earr *a = calloc(1, sizeof(earr));
    if (!a) return NULL;
    a->dtype = dtype;
    a->ndim = ndim;
    for (int i = 0; i < ndim; i++) a->shape[i] = shape[i];
    a->b = buf_get(numel(a) * dt_size(dtype));
    if (!a->b) {
        free(a);
        return NULL;
    }
    return a;
}

mlx_array mlx_array_new(void) { return (mlx_array){NULL}; }

int mlx_array_free(mlx_array a) {
    earr *e = a.ctx;
    if (!e) return 0;
    buf_put(e->b);
    free(e);
    return 0;
}

mlx_array mlx_array_new_data(const void *data, const int *shape, int dim, mlx_dtype dtype) {
    if (!data || (dtype != MLX_INT32 && dtype != MLX_UINT32 && dtype != MLX_FLOAT32 && dtype != MLX_BFLOAT16))
        return mlx_array_new();
    earr *a = new_arr(dtype, dim, shape);
    if (!a) return mlx_array_new();
    /* pageable source: the call returns once the bytes are staged */
    if (mlxd_cuda_upload(a->b->p, data, numel(a) * dt_size(dtype), stream_ptr())) {
        mlx_array_free(wrap(a));
        return mlx_array_new();
    }
    return wrap(a);
}

int mlx_reshape(mlx_array *res, mlx_array a, const int *shape, size_t shape_num, mlx_stream s) {
    (void)s;
    earr *e = a.ctx;
    if (!res || !e || !e->b || shape_num > 4) return -1;
    earr *r = calloc(1, sizeof(earr));
    if (!r) return -1;
    *r = *e;
    r->ndim = (int)shape_num;
    for (size_t i = 0; i < shape_num; i++) r->shape[i] = shape[i];
    if (numel(r) != numel(e)) {
        free(r);
        return -1;
    }
    e->b->refs++;
    mlx_array_free(*res);
    *res = wrap(r);
    return 0;
}

size_t mlx_array_ndim(mlx_array a) { return a.ctx ? (size_t)((earr *)a.ctx)->ndim : 0; }
int mlx_array_dim(mlx_array a, int dim) {
    earr *e = a.ctx;
    return e && dim >= 0 && dim < e->ndim ? e->shape[dim] : 0;
}
mlx_dtype mlx_array_dtype(mlx_array a) { return a.ctx ? (mlx_dtype)((earr *)a.ctx)->dtype : MLX_FLOAT32; }
void *mlxd_array_data(mlx_array a) {
    earr *e = a.ctx;
    return e && e->b ? e->b->p : NULL;
}

int mlxbridge_get_shape(mlx_array arr, int *dims, int max_dims) {
    earr *e = arr.ctx;
    if (!e) return -1;
    for (int i = 0; i < e->ndim && i < max_dims; i++) dims[i] = e->shape[i];
    return e->ndim;
}

/* the work is enqueued already; an empty handle is the reference's failure */
int mlxbridge_async_eval(mlx_array a) { return a.ctx ? 0 : -1; }
int mlxbridge_async_eval_n(const mlx_array *arrs, size_t n) {
    for (size_t i = 0; i < n; i++)
        if (!arrs[i].ctx) return -1;
    return 0;
}

int mlxbridge_item_int32(int32_t *out, mlx_array a) {
    earr *e = a.ctx;
    if (!out || !e || !e->b || (e->dtype != MLX_INT32 && e->dtype != MLX_UINT32) || numel(e) < 1) return -1;
    return mlxd_cuda_read_token((const int32_t *)e->b->p, out, stream_ptr());
}

int mlxbridge_item_float32(float *out, mlx_array a) {
    earr *e = a.ctx;
    if (!out || !e || !e->b || numel(e) < 1) return -1;
    if (e->dtype == MLX_FLOAT32 || e->dtype == MLX_BFLOAT16) {
        uint32_t bits = 0;
        if (mlxd_cuda_read_token((const int32_t *)e->b->p, (int32_t *)&bits, stream_ptr())) return -1;
        if (e->dtype == MLX_BFLOAT16) bits <<= 16;
        memcpy(out, &bits, 4);
        return 0;
    }
    return -1;
}

int mlxbridge_synchronize(mlx_stream s) { return mlxd_cuda_synchronize(s.ctx ? s.ctx : stream_ptr()); }
int mlxbridge_get_active_memory(size_t *out) {
    if (!out) return -1;
    *out = mlxd_cuda_active_memory();
    return 0;
}
int mlxbridge_get_peak_memory(size_t *out) {
    if (!out) return -1;
    *out = mlxd_cuda_peak_memory();
    return 0;
}

/* ------------------------------------------------------------ model */

static void copy_err(char *err, size_t errlen, const char *what) {
    if (err && errlen) snprintf(err, errlen, "%s: %s", what, mlxd_cuda_last_error());
}

int engine_model_load(engine_model_t *em, const char *model_dir, char *err, size_t errlen) {
    if (!em || !model_dir) return -1;
    memset(em, 0, sizeof(*em));
    if (model_config_load(&em->cfg, model_dir, err, errlen)) return -1;
    if (engine_model_check_supported(&em->cfg, err, errlen)) return -1;
    mlxd_model_config mc;
    if (model_config_to_cuda(&em->cfg, 0, 1, &mc, err, errlen)) return -1;
    mlxd_checkpoint ck;
    if (mlxd_checkpoint_open(&ck, model_dir, &em->cfg, err, errlen)) return -1;
    const int rc = mlxd_cuda_model_create(&em->m, &mc, ck.tensors, ck.n_tensors);
    mlxd_checkpoint_close(&ck);
    if (rc) {
        copy_err(err, errlen, "model upload");
        memset(em, 0, sizeof(*em));
        return -1;
    }
    em->stream = mlxbridge_gpu_stream();
    return 0;
}

void engine_model_free(engine_model_t *em) {
    if (!em) return;
    if (em->m) mlxd_cuda_model_destroy(em->m);
    memset(em, 0, sizeof(*em));
}

/* ------------------------------------------------------------ KV cache */

int kvcache_init(kvcache_t *kv, int num_layers) {
    if (!kv || num_layers <= 0) return -1;
    memset(kv, 0, sizeof(*kv));
    kv->entries = calloc((size_t)num_layers, sizeof(kv_entry_t));
    if (!kv->entries) return -1;
    kv->num_layers = num_layers;
    return 0;
}

void kvcache_free(kvcache_t *kv) {
    if (!kv) return;
    if (kv->dev) mlxd_cuda_kv_destroy(kv->dev);
    free(kv->entries);
    memset(kv, 0, sizeof(*kv));
}

int kvcache_layer_offset(const kvcache_t *kv, int layer) {
    if (!kv || layer < 0 || layer >= kv->num_layers) return -1;
    return kv->entries[layer].offset;
}

int kvcache_capacity(const kvcache_t *kv, int layer) {
    if (!kv || layer < 0 || layer >= kv->num_layers) return -1;
    return kv->entries[layer].capacity;
}

static int window_of(const kvcache_t *kv) {
    const model_config_t *c = &kv->em->cfg;
    return !strcmp(c->model_type, "mistral") && c->has_sliding_window ? c->sliding_window : 0;
}

/* a device cache of `cap` slots; the rows written so far move over */
static int kv_realloc(kvcache_t *kv, int cap) {
    mlxd_kv *nk = NULL;
    if (mlxd_cuda_kv_create(&nk, kv->em->m, cap)) return -1;
    void *st = stream_ptr();
    int moved = 0;
    if (kv->dev) {
        const int hkv = kv->em->cfg.num_key_value_heads, D = kv->em->cfg.head_dim;
        for (int l = 0; l < kv->num_layers; l++) {
            const int n = kv->entries[l].offset;
            if (!n) continue;
            ebuf *tk = buf_get((size_t)hkv * n * D * 2), *tv = buf_get((size_t)hkv * n * D * 2);
            int rc = !tk || !tv || mlxd_cuda_kv_gather(kv->dev, l, 0, 0, n, tk->p, st) ||
                     mlxd_cuda_kv_gather(kv->dev, l, 1, 0, n, tv->p, st) ||
                     mlxd_cuda_kv_write(nk, l, 0, n, tk->p, tv->p, st);
            buf_put(tk);
            buf_put(tv);
            if (rc) {
                mlxd_cuda_kv_destroy(nk);
                return -1;
            }
            moved = n > moved ? n : moved;
        }
        if (mlxd_cuda_synchronize(st)) {
            mlxd_cuda_kv_destroy(nk);
            return -1;
        }
        mlxd_cuda_kv_destroy(kv->dev);
    }
    kv->dev = nk;
    if (mlxd_cuda_kv_set_offset(nk, kv->entries[0].offset, st)) return -1;
    for (int l = 0; l < kv->num_layers; l++) {
        kv->entries[l].capacity = cap;
        kv->entries[l].n_kv_heads = kv->em->cfg.num_key_value_heads;
        kv->entries[l].head_dim = kv->em->cfg.head_dim;
    }
    return 0;
}

int kvcache_bind(kvcache_t *kv, const engine_model_t *em) {
    if (!kv || !em || !em->m || kv->num_layers != em->cfg.num_hidden_layers) return -1;
    if (kv->dev) return kv->em == em ? 0 : -1;
    kv->em = em;
    const int w = window_of(kv);
    /* a sliding window keeps a ring (window + one 512-token chunk); other
       caches start at 256 slots and grow */
    return kv_realloc(kv, w > 0 ? w + 511 : 256);
}

/* room for n more positions at every layer (full caches grow) */
static int kv_room(kvcache_t *kv, int n) {
    if (window_of(kv) > 0) return 0;
    int need = 0;
    for (int l = 0; l < kv->num_layers; l++)
        if (kv->entries[l].offset + n > need) need = kv->entries[l].offset + n;
    const int cap = kv->entries[0].capacity;
    if (need <= cap) return 0;
    int nc = cap * 2 > need ? cap * 2 : need;
    nc = (nc + 255) / 256 * 256;
    const int maxp = kv->em->cfg.max_position_embeddings;
    if (maxp > 0 && nc > maxp) nc = maxp;
    if (nc < need) return -1;
    return kv_realloc(kv, nc);
}

static int make_view(const kvcache_t *kv, int layer, int is_value, int start, int len, mlx_array *out) {
    const int shape[4] = {1, kv->em->cfg.num_key_value_heads, len, kv->em->cfg.head_dim};
    earr *a = new_arr(MLX_BFLOAT16, 4, shape);
    if (!a) return -1;
    if (len > 0 && mlxd_cuda_kv_gather(kv->dev, layer, is_value, start, len, a->b->p, stream_ptr())) {
        mlx_array_free(wrap(a));
        return -1;
    }
    mlx_array_free(*out);
    *out = wrap(a);
    return 0;
}

static int view_range(const kvcache_t *kv, int layer, int max_kv, int q_len, int *start, int *len) {
    const int end = kv->entries[layer].offset;
    int s = max_kv > 0 && q_len == 1 && end > max_kv ? end - max_kv : 0;
    if (end - s > kv->entries[layer].capacity) s = end - kv->entries[layer].capacity;   /* ring */
    *start = s;
    *len = end - s;
    return 0;
}

int kvcache_update(kvcache_t *kv, int layer, mlx_array new_k, mlx_array new_v, int max_kv, mlx_array *k_view,
                   mlx_array *v_view, mlx_stream s) {
    (void)s;
    earr *k = new_k.ctx, *v = new_v.ctx;
    if (!kv || !kv->dev || layer < 0 || layer >= kv->num_layers || !k || !v || !k_view || !v_view) return -1;
    const int hkv = kv->em->cfg.num_key_value_heads, D = kv->em->cfg.head_dim;
    if (k->dtype != MLX_BFLOAT16 || v->dtype != MLX_BFLOAT16 || k->ndim != 4 || v->ndim != 4 || k->shape[0] != 1 ||
        k->shape[1] != hkv || k->shape[3] != D || memcmp(k->shape, v->shape, sizeof k->shape))
        return -1;
    const int n = k->shape[2];
    if (kv_room(kv, n)) return -1;
    const int off = kv->entries[layer].offset;
    if (mlxd_cuda_kv_write(kv->dev, layer, off, n, k->b->p, v->b->p, stream_ptr())) return -1;
    kv->entries[layer].offset = off + n;
    kv->entries[layer].initialized = true;
    /* once every layer reached the same position, a model_forward appends
       after it */
    int same = 1;
    for (int l = 1; l < kv->num_layers; l++) same &= kv->entries[l].offset == kv->entries[0].offset;
    if (same && mlxd_cuda_kv_set_offset(kv->dev, kv->entries[0].offset, stream_ptr())) return -1;
    int st, len;
    view_range(kv, layer, max_kv, n, &st, &len);
    mlx_array kt = mlx_array_new(), vt = mlx_array_new();
    if (make_view(kv, layer, 0, st, len, &kt) || make_view(kv, layer, 1, st, len, &vt)) {
        mlx_array_free(kt);
        mlx_array_free(vt);
        return -1;
    }
    mlx_array_free(*k_view);
    mlx_array_free(*v_view);
    *k_view = kt;
    *v_view = vt;
    return 0;
}

int kvcache_view(const kvcache_t *kv, int layer, int max_kv, int q_len, mlx_array *k_view, mlx_array *v_view,
                 mlx_stream s) {
    (void)s;
    if (!kv || !kv->dev || layer < 0 || layer >= kv->num_layers || !kv->entries[layer].initialized || !k_view ||
        !v_view)
        return -1;
    int st, len;
    view_range(kv, layer, max_kv, q_len, &st, &len);
    mlx_array kt = mlx_array_new(), vt = mlx_array_new();
    if (make_view(kv, layer, 0, st, len, &kt) || make_view(kv, layer, 1, st, len, &vt)) {
        mlx_array_free(kt);
        mlx_array_free(vt);
        return -1;
    }
    mlx_array_free(*k_view);
    mlx_array_free(*v_view);
    *k_view = kt;
    *v_view = vt;
    return 0;
}

int model_forward(engine_model_t *em, mlx_array ids, kvcache_t *kv, bool want_logits, mlx_array *logits_out) {
    earr *ia = ids.ctx;
    if (!em || !em->m || !kv || !ia || !ia->b || (ia->dtype != MLX_INT32 && ia->dtype != MLX_UINT32) ||
        (want_logits && !logits_out))
        return -1;
    const int n = (int)numel(ia);
    if (n <= 0) return -1;
    if (!kv->dev && kvcache_bind(kv, em)) return -1;
    if (kv->em != em || kv_room(kv, n)) return -1;
    earr *lg = NULL;
    if (want_logits) {
        const int shape[3] = {1, 1, em->cfg.vocab_size};
        lg = new_arr(MLX_BFLOAT16, 3, shape);
        if (!lg) return -1;
    }
    if (mlxd_cuda_forward(em->m, kv->dev, (const int32_t *)ia->b->p, n, 1, want_logits, lg ? lg->b->p : NULL,
                          em->stream.ctx)) {
        if (lg) mlx_array_free(wrap(lg));
        return -1;
    }
    for (int l = 0; l < kv->num_layers; l++) {
        kv->entries[l].offset += n;
        kv->entries[l].initialized = true;
    }
    if (lg) {
        mlx_array_free(*logits_out);
        *logits_out = wrap(lg);
    }
    return 0;
}

/* ------------------------------------------------------------ sampler */

int sampler_key_init(sampler_key_t *k, int seed) {
    if (!k) return -1;
    k->key = mlx_array_new();
    k->seeded = false;
    if (seed < 0) return 0;
    earr *a = calloc(1, sizeof(earr));
    if (!a) return -1;
    a->is_key = 1;
    a->seed = seed;
    k->key = wrap(a);
    k->seeded = true;
    return 0;
}

/* the subkey names draw `step` of the seed's stream; the key moves on */
int sampler_key_next(sampler_key_t *k, mlx_array *subkey_out, mlx_stream s) {
    (void)s;
    if (!k || !subkey_out) return -1;
    if (!k->seeded) {
        *subkey_out = mlx_array_new();
        return 0;
    }
    earr *key = k->key.ctx, *sub = calloc(1, sizeof(earr));
    if (!sub) return -1;
    *sub = *key;
    key->step++;
    *subkey_out = wrap(sub);
    return 0;
}

void sampler_key_free(sampler_key_t *k) {
    if (!k) return;
    mlx_array_free(k->key);
    k->key = mlx_array_new();
    k->seeded = false;
}

sampling_params_t sampling_resolve(const sampling_params_t *req, unsigned set_mask, const model_config_t *cfg) {
    sampling_params_t out = SAMPLING_PARAMS_DEFAULT;
    if (set_mask & SAMPLING_SET_TEMPERATURE) out.temperature = req->temperature;
    else if (cfg && cfg->has_gen_temperature) out.temperature = cfg->gen_temperature;
    if (set_mask & SAMPLING_SET_TOP_P) out.top_p = req->top_p;
    else if (cfg && cfg->has_gen_top_p) out.top_p = cfg->gen_top_p;
    if (set_mask & SAMPLING_SET_TOP_K) out.top_k = req->top_k;
    else if (cfg && cfg->has_gen_top_k) out.top_k = cfg->gen_top_k;
    if (set_mask & SAMPLING_SET_MIN_P) out.min_p = req->min_p;
    if (set_mask & SAMPLING_SET_SEED) out.seed = req->seed;
    return out;
}

/* unseeded draws take consecutive steps of stream 0 */
static uint64_t g_unseeded_step;

int sampler_sample_lazy(mlx_array logits, const sampling_params_t *sp, mlx_array subkey, bool want_logprob,
                        mlx_stream s, mlx_array *tok_out, mlx_array *logprob_out) {
    earr *la = logits.ctx, *key = subkey.ctx;
    if (!la || !la->b || !sp || !tok_out || (want_logprob && !logprob_out) ||
        (la->dtype != MLX_BFLOAT16 && la->dtype != MLX_FLOAT32) || la->ndim < 1)
        return -1;
    const int V = la->shape[la->ndim - 1];
    const size_t rows = numel(la) / (size_t)V;
    const char *row = (const char *)la->b->p + (rows - 1) * (size_t)V * dt_size(la->dtype);
    mlxd_sampling ms = {sp->temperature, sp->top_p, sp->top_k, sp->min_p, key ? key->seed : -1, 1.0f, 0};
    const uint64_t step = key ? key->step : g_unseeded_step++;
    const int one = 1;
    earr *t = new_arr(MLX_INT32, 1, &one), *lp = want_logprob ? new_arr(MLX_FLOAT32, 1, &one) : NULL;
    if (!t || (want_logprob && !lp)) goto fail;
    if (mlxd_cuda_sample(row, la->dtype == MLX_BFLOAT16 ? MLXD_BF16 : MLXD_F32, V, &ms, NULL, 0, step,
                         (int32_t *)t->b->p, lp ? (float *)lp->b->p : NULL, NULL, s.ctx ? s.ctx : stream_ptr()))
        goto fail;
    mlx_array_free(*tok_out);
    *tok_out = wrap(t);
    if (want_logprob) {
        mlx_array_free(*logprob_out);
        *logprob_out = wrap(lp);
    }
    return 0;
fail:
    if (t) mlx_array_free(wrap(t));
    if (lp) mlx_array_free(wrap(lp));
    return -1;
}
