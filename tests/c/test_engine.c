/* C11 driver of libmlxd_engine, built and run by tests/test_engine_c_gpu.py.
 *
 *   test_engine generate DIR MAX_NEW CHUNK TEMP TOP_K TOP_P SEED ID...
 *       the generate loop of the reference (src/engine/engine.c:360-602):
 *       chunked prefill of ids[:-1], the seed forward, then the pipelined
 *       decode (sample the pending logits lazily, enqueue the next forward,
 *       async_eval both, read the token); prints "TOKENS ..." and
 *       "LOGPROBS ..." (stops at EOS like the reference)
 *   test_engine async DIR MAX_NEW ID...
 *       the same greedy decode through mlxd_cuda_step_async /
 *       mlxd_cuda_read_token on the library's own handles
 *   test_engine kv DIR ID...
 *       model_forward on the ids, then kvcache_view of every layer against
 *       mlxd_cuda_kv_read, and a kvcache_update / kvcache_view round trip on
 *       a second cache
 *   test_engine load DIR
 *       engine_model_load only: prints "LOAD OK" or "LOAD ERROR <message>"
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "mlxd_engine.h"

#define CHECK(cond, ...)                          \
    do {                                          \
        if (!(cond)) {                            \
            fprintf(stderr, "FAIL: " __VA_ARGS__); \
            fprintf(stderr, " (%s)\n", mlxd_cuda_last_error()); \
            exit(1);                              \
        }                                         \
    } while (0)

static mlx_array ids_array(const int32_t *ids, int n) {
    const int shape[2] = {1, n};
    return mlx_array_new_data(ids, shape, 2, MLX_INT32);
}

static int is_eos(const model_config_t *c, int32_t id) {
    for (int i = 0; i < c->num_eos_tokens; i++)
        if (c->eos_token_ids[i] == id) return 1;
    return 0;
}

static void load(engine_model_t *em, const char *dir) {
    char err[512] = "";
    CHECK(mlxd_cuda_init(0) == 0, "init");
    CHECK(engine_model_load(em, dir, err, sizeof err) == 0, "engine_model_load: %s", err);
}

static int run_generate(int argc, char **argv) {
    if (argc < 10) return 2;
    engine_model_t em;
    load(&em, argv[2]);
    const int max_new = atoi(argv[3]), chunk = atoi(argv[4]);
    sampling_params_t req = {(float)atof(argv[5]), (float)atof(argv[7]), atoi(argv[6]), 0.0f, atoi(argv[8])};
    sampling_params_t sp =
        sampling_resolve(&req, SAMPLING_SET_TEMPERATURE | SAMPLING_SET_TOP_K | SAMPLING_SET_TOP_P | SAMPLING_SET_SEED,
                         &em.cfg);
    const int n = argc - 9;
    int32_t *ids = malloc(sizeof(int32_t) * (size_t)n);
    for (int i = 0; i < n; i++) ids[i] = atoi(argv[9 + i]);
    const bool want_lp = true;

    kvcache_t kv;
    CHECK(kvcache_init(&kv, em.cfg.num_hidden_layers) == 0, "kvcache_init");
    sampler_key_t skey;
    CHECK(sampler_key_init(&skey, sp.seed) == 0, "sampler_key_init");
    mlx_array pending = mlx_array_new();
    for (int pos = 0; pos < n - 1; pos += chunk) {
        const int len = n - 1 - pos < chunk ? n - 1 - pos : chunk;
        mlx_array a = ids_array(ids + pos, len);
        CHECK(model_forward(&em, a, &kv, false, NULL) == 0, "prefill forward");
        mlx_array_free(a);
        mlxbridge_clear_cache();
    }
    CHECK(kvcache_layer_offset(&kv, 0) == n - 1, "prefill offset %d", kvcache_layer_offset(&kv, 0));
    mlx_array last = ids_array(ids + n - 1, 1);
    CHECK(model_forward(&em, last, &kv, true, &pending) == 0, "seed forward");
    mlx_array_free(last);

    int32_t *toks = malloc(sizeof(int32_t) * (size_t)max_new);
    float *lps = malloc(sizeof(float) * (size_t)max_new);
    int emitted = 0;
    while (emitted < max_new) {
        mlx_array subkey = mlx_array_new();
        CHECK(sampler_key_next(&skey, &subkey, em.stream) == 0, "key_next");
        mlx_array tok = mlx_array_new(), lp = mlx_array_new();
        CHECK(sampler_sample_lazy(pending, &sp, subkey, want_lp, em.stream, &tok, &lp) == 0, "sample");
        mlx_array_free(subkey);
        mlx_array_free(pending);
        pending = mlx_array_new();
        mlx_array next = mlx_array_new();
        int have_next = 0;
        if (emitted + 1 < max_new) {
            const int shape[2] = {1, 1};
            mlx_array step_ids = mlx_array_new();
            CHECK(mlx_reshape(&step_ids, tok, shape, 2, em.stream) == 0, "reshape");
            CHECK(model_forward(&em, step_ids, &kv, true, &next) == 0, "decode forward");
            mlx_array batch[3] = {tok, next, lp};
            CHECK(mlxbridge_async_eval_n(batch, 3) == 0, "async_eval");
            mlx_array_free(step_ids);
            have_next = 1;
        } else {
            mlx_array batch[2] = {tok, lp};
            CHECK(mlxbridge_async_eval_n(batch, 2) == 0, "async_eval");
        }
        int32_t id = -1;
        float lpv = 0.f;
        CHECK(mlxbridge_item_int32(&id, tok) == 0, "item_int32");
        CHECK(mlxbridge_item_float32(&lpv, lp) == 0, "item_float32");
        mlx_array_free(tok);
        mlx_array_free(lp);
        if (is_eos(&em.cfg, id)) {
            if (have_next) mlx_array_free(next);
            break;
        }
        toks[emitted] = id;
        lps[emitted] = lpv;
        emitted++;
        if (!have_next) break;
        pending = next;
    }
    mlx_array_free(pending);
    printf("TOKENS");
    for (int i = 0; i < emitted; i++) printf(" %d", toks[i]);
    printf("\nLOGPROBS");
    for (int i = 0; i < emitted; i++) printf(" %.9g", lps[i]);
    printf("\nOFFSET %d\n", kvcache_layer_offset(&kv, 0));
    sampler_key_free(&skey);
    kvcache_free(&kv);
    mlxbridge_clear_cache();
    engine_model_free(&em);
    free(ids);
    free(toks);
    free(lps);
    return 0;
}

static int run_async(int argc, char **argv) {
    if (argc < 5) return 2;
    engine_model_t em;
    load(&em, argv[2]);
    const int max_new = atoi(argv[3]), n = argc - 4;
    int32_t *ids = malloc(sizeof(int32_t) * (size_t)n);
    for (int i = 0; i < n; i++) ids[i] = atoi(argv[4 + i]);
    mlxd_kv *kv = NULL;
    CHECK(mlxd_cuda_kv_create(&kv, em.m, n + max_new + 8) == 0, "kv_create");
    void *st = em.stream.ctx;
    if (n > 1) CHECK(mlxd_cuda_forward(em.m, kv, ids, n - 1, 0, 0, NULL, st) == 0, "prefill");
    int32_t *dtok = NULL;
    CHECK(mlxd_cuda_alloc((void **)&dtok, sizeof(int32_t) * 2) == 0, "alloc");
    CHECK(mlxd_cuda_upload(dtok, ids + n - 1, 4, st) == 0, "upload");
    mlxd_sampling sp = {0.0f, 1.0f, -1, 0.0f, -1, 1.0f, 0};
    /* one step ahead: step e + 1 is enqueued before token e is read */
    CHECK(mlxd_cuda_step_async(em.m, kv, dtok, &sp, NULL, 0, 0, dtok + 1, NULL, st) == 0, "step_async");
    printf("TOKENS");
    for (int e = 0; e < max_new; e++) {
        const int cur = (e + 1) & 1, nxt = e & 1;
        if (e + 1 < max_new)
            CHECK(mlxd_cuda_step_async(em.m, kv, dtok + cur, &sp, NULL, 0, (uint64_t)(e + 1), dtok + nxt, NULL,
                                       st) == 0,
                  "step_async");
        int32_t t = -1;
        /* token e sits in the slot step e + 1 read from, before step e + 1 ends */
        CHECK(mlxd_cuda_read_token(dtok + cur, &t, st) == 0, "read_token");
        printf(" %d", t);
    }
    printf("\n");
    mlxd_cuda_free(dtok);
    mlxd_cuda_kv_destroy(kv);
    engine_model_free(&em);
    free(ids);
    return 0;
}

static int run_kv(int argc, char **argv) {
    if (argc < 4) return 2;
    engine_model_t em;
    load(&em, argv[2]);
    const int n = argc - 3;
    int32_t *ids = malloc(sizeof(int32_t) * (size_t)n);
    for (int i = 0; i < n; i++) ids[i] = atoi(argv[3 + i]);
    kvcache_t kv;
    CHECK(kvcache_init(&kv, em.cfg.num_hidden_layers) == 0, "kvcache_init");
    mlx_array a = ids_array(ids, n);
    CHECK(model_forward(&em, a, &kv, false, NULL) == 0, "forward");
    mlx_array_free(a);
    const int H = em.cfg.num_key_value_heads, D = em.cfg.head_dim;
    size_t elems = (size_t)H * n * D;
    uint16_t *want = malloc(elems * 2), *got = malloc(elems * 2);
    for (int l = 0; l < em.cfg.num_hidden_layers; l++) {
        mlx_array kview = mlx_array_new(), vview = mlx_array_new();
        CHECK(kvcache_view(&kv, l, 0, n, &kview, &vview, em.stream) == 0, "kvcache_view");
        CHECK(mlx_array_dim(kview, 2) == n && mlx_array_dim(kview, 1) == H, "view shape");
        for (int v = 0; v < 2; v++) {
            int rows = 0;
            CHECK(mlxd_cuda_kv_read(kv.dev, l, v, want, &rows) == 0 && rows == n, "kv_read");
            CHECK(mlxd_cuda_download(got, mlxd_array_data(v ? vview : kview), elems * 2, em.stream.ctx) == 0,
                  "download");
            CHECK(mlxd_cuda_synchronize(em.stream.ctx) == 0, "sync");
            CHECK(memcmp(want, got, elems * 2) == 0, "layer %d %s view differs", l, v ? "value" : "key");
        }
        /* decode-step trim: the last 3 rows */
        if (n > 3) {
            mlx_array k3 = mlx_array_new(), v3 = mlx_array_new();
            CHECK(kvcache_view(&kv, l, 3, 1, &k3, &v3, em.stream) == 0 && mlx_array_dim(k3, 2) == 3, "trim");
            mlx_array_free(k3);
            mlx_array_free(v3);
        }
        mlx_array_free(kview);
        mlx_array_free(vview);
    }
    /* update / view round trip on a second cache: layer 1's rows written
       into layer 0 of the new cache come back unchanged */
    kvcache_t kv2;
    CHECK(kvcache_init(&kv2, em.cfg.num_hidden_layers) == 0 && kvcache_bind(&kv2, &em) == 0, "bind");
    const int L1 = em.cfg.num_hidden_layers > 1 ? 1 : 0;
    mlx_array k1 = mlx_array_new(), v1 = mlx_array_new(), kv_k = mlx_array_new(), kv_v = mlx_array_new();
    CHECK(kvcache_view(&kv, L1, 0, n, &k1, &v1, em.stream) == 0, "view");
    CHECK(kvcache_update(&kv2, 0, k1, v1, 0, &kv_k, &kv_v, em.stream) == 0, "kvcache_update");
    CHECK(kvcache_layer_offset(&kv2, 0) == n && kvcache_layer_offset(&kv2, L1 ? 1 : 0) == (L1 ? 0 : n),
          "offsets");
    CHECK(mlxd_cuda_download(got, mlxd_array_data(kv_v), elems * 2, em.stream.ctx) == 0, "download");
    CHECK(mlxd_cuda_synchronize(em.stream.ctx) == 0, "sync");
    int rows = 0;
    CHECK(mlxd_cuda_kv_read(kv.dev, L1, 1, want, &rows) == 0, "kv_read");
    CHECK(memcmp(want, got, elems * 2) == 0, "update round trip differs");
    mlx_array_free(k1);
    mlx_array_free(v1);
    mlx_array_free(kv_k);
    mlx_array_free(kv_v);
    kvcache_free(&kv2);
    kvcache_free(&kv);
    mlxbridge_clear_cache();
    engine_model_free(&em);
    free(want);
    free(got);
    free(ids);
    printf("KV OK\n");
    return 0;
}

int main(int argc, char **argv) {
    if (argc < 3) {
        fprintf(stderr, "usage: test_engine generate|async|kv|load DIR ...\n");
        return 2;
    }
    if (!strcmp(argv[1], "generate")) return run_generate(argc, argv);
    if (!strcmp(argv[1], "async")) return run_async(argc, argv);
    if (!strcmp(argv[1], "kv")) return run_kv(argc, argv);
    if (!strcmp(argv[1], "load")) {
        engine_model_t em;
        char err[512] = "";
        CHECK(mlxd_cuda_init(0) == 0, "init");
        if (engine_model_load(&em, argv[2], err, sizeof err)) {
            printf("LOAD ERROR %s\n", err);
            return 0;
        }
        printf("LOAD OK\n");
        engine_model_free(&em);
        return 0;
    }
    return 2;
}
