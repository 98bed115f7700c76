/* Model directory loading for libmlxd_engine: config.json and
   generation_config.json (reference src/model/model.c:667-1031, the dense
   families on the path), the support gate (src/engine/emodel.c:22-150), and
   the safetensors shards with the reference's validation
   (src/model/weights.c:20-192 shard enumeration, :752-940 validation,
   :651-750 expected set). Host only: nothing here touches the GPU. */
#define _POSIX_C_SOURCE 200809L
#include <dirent.h>
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "json.h"
#include "mlxd_engine.h"

#define FAIL(...)                                             \
    do {                                                      \
        if (err && errlen) snprintf(err, errlen, __VA_ARGS__); \
        goto fail;                                            \
    } while (0)

static char *join(const char *dir, const char *name) {
    size_t a = strlen(dir), b = strlen(name);
    char *p = malloc(a + b + 2);
    if (!p) return NULL;
    memcpy(p, dir, a);
    p[a] = '/';
    memcpy(p + a + 1, name, b + 1);
    return p;
}

static int is_file(const char *p) {
    struct stat st;
    return stat(p, &st) == 0 && S_ISREG(st.st_mode);
}

/* ------------------------------------------------------------ config */

enum { FAM_NONE = 0, FAM_QWEN3 = MLXD_QWEN3, FAM_LLAMA = MLXD_LLAMA, FAM_MISTRAL = MLXD_MISTRAL,
       FAM_QWEN3_5 = MLXD_QWEN3_5 };

static int family_of(const char *t) {
    if (!strcmp(t, "qwen3")) return FAM_QWEN3;
    if (!strcmp(t, "llama")) return FAM_LLAMA;
    if (!strcmp(t, "mistral")) return FAM_MISTRAL;
    if (!strcmp(t, "qwen3_5") || !strcmp(t, "qwen3_5_text")) return FAM_QWEN3_5;
    return FAM_NONE;
}

static void read_eos(const json_val *v, model_config_t *c) {
    if (!v) return;
    if (v->type == JSON_NUM) {
        c->num_eos_tokens = 1;
        c->eos_token_ids[0] = (int)v->num;
    } else if (v->type == JSON_ARR) {
        c->num_eos_tokens = 0;
        for (int i = 0; i < v->n && c->num_eos_tokens < 8; i++)
            if (v->items[i]->type == JSON_NUM) c->eos_token_ids[c->num_eos_tokens++] = (int)v->items[i]->num;
    }
}

int model_config_load(model_config_t *c, const char *dir, char *err, size_t errlen) {
    json_val *cj = NULL, *gj = NULL;
    char *path = NULL;
    if (!c || !dir) return -1;
    memset(c, 0, sizeof(*c));
    path = join(dir, "config.json");
    if (!path) FAIL("out of memory");
    cj = json_parse_file(path, err, errlen);
    if (!cj || cj->type != JSON_OBJ) FAIL("failed to load config from %s", dir);
    const char *mt = json_str(cj, "model_type");
    if (!mt) FAIL("config.json: model_type missing");
    snprintf(c->model_type, sizeof c->model_type, "%s", mt);
    c->vocab_size = json_int(cj, "vocab_size", 0);
    c->hidden_size = json_int(cj, "hidden_size", 0);
    c->num_hidden_layers = json_int(cj, "num_hidden_layers", 0);
    c->num_attention_heads = json_int(cj, "num_attention_heads", 0);
    c->num_key_value_heads = json_int(cj, "num_key_value_heads", c->num_attention_heads);
    c->max_position_embeddings = json_int(cj, "max_position_embeddings", 0);
    c->intermediate_size = json_int(cj, "intermediate_size", 0);
    if (c->vocab_size <= 0 || c->hidden_size <= 0 || c->num_hidden_layers <= 0 || c->num_attention_heads <= 0 ||
        c->num_key_value_heads <= 0)
        FAIL("config.json: missing or invalid core dimensions");
    c->head_dim = json_int(cj, "head_dim", 0);
    if (c->head_dim <= 0) c->head_dim = c->hidden_size / c->num_attention_heads;
    c->rms_norm_eps = (float)json_double(cj, "rms_norm_eps", 1e-6);
    c->rope_theta = (float)json_double(cj, "rope_theta", 1e6);
    c->partial_rotary_factor = (float)json_double(cj, "partial_rotary_factor", 1.0);
    /* a flat rope_parameters object (qwen3_5) carries theta and the partial
       factor; nested per-attention-type parameters are another family's */
    const json_val *rp = json_get(cj, "rope_parameters");
    if (rp && rp->type == JSON_OBJ) {
        int nested = 0;
        for (int i = 0; i < rp->n; i++) nested |= rp->items[i]->type == JSON_OBJ;
        if (!nested) {
            c->rope_theta = (float)json_double(rp, "rope_theta", c->rope_theta);
            c->partial_rotary_factor = (float)json_double(rp, "partial_rotary_factor", c->partial_rotary_factor);
        }
    }
    const json_val *rs = json_get(cj, "rope_scaling");
    if (rs && rs->type == JSON_OBJ) {
        const char *rt = json_str(rs, "rope_type");
        if (!rt) rt = json_str(rs, "type");
        if (rt) snprintf(c->rope_scaling_type, sizeof c->rope_scaling_type, "%s", rt);
        c->rope_scaling_factor = (float)json_double(rs, "factor", 1.0);
        c->rope_low_freq_factor = (float)json_double(rs, "low_freq_factor", 1.0);
        c->rope_high_freq_factor = (float)json_double(rs, "high_freq_factor", 1.0);
        c->rope_original_max_position_embeddings = json_int(rs, "original_max_position_embeddings", 0);
    }
    const json_val *sw = json_get(cj, "sliding_window");
    if (sw && sw->type == JSON_NUM && sw->num > 0) {
        c->has_sliding_window = true;
        c->sliding_window = (int)sw->num;
    }
    c->attention_bias = json_bool(cj, "attention_bias", 0);
    const json_val *q = json_get(cj, "quantization");
    if (!q) q = json_get(cj, "quantization_config");
    if (q && q->type == JSON_OBJ) {
        c->quant_bits = json_int(q, "bits", 0);
        c->quant_group_size = json_int(q, "group_size", 64);
    }
    c->tie_word_embeddings = json_bool(cj, "tie_word_embeddings", 0);
    const int fam = family_of(c->model_type);
    c->has_qk_norm = fam == FAM_QWEN3 || fam == FAM_QWEN3_5;
    c->attn_output_gate = json_bool(cj, "attn_output_gate", fam == FAM_QWEN3_5);
    const char *act = json_str(cj, "hidden_act");
    if (!act) act = json_str(cj, "hidden_activation");
    c->hidden_act_silu = !act || !strcmp(act, "silu") || !strcmp(act, "swish");
    c->num_experts = json_int(cj, "num_experts", json_int(cj, "num_local_experts", 0));
    read_eos(json_get(cj, "eos_token_id"), c);
    free(path);
    path = join(dir, "generation_config.json");
    if (path && is_file(path)) {
        gj = json_parse_file(path, NULL, 0);
        if (gj && gj->type == JSON_OBJ) {
            const json_val *v;
            if ((v = json_get(gj, "temperature")) && v->type == JSON_NUM) {
                c->has_gen_temperature = true;
                c->gen_temperature = (float)v->num;
            }
            if ((v = json_get(gj, "top_p")) && v->type == JSON_NUM) {
                c->has_gen_top_p = true;
                c->gen_top_p = (float)v->num;
            }
            if ((v = json_get(gj, "top_k")) && v->type == JSON_NUM) {
                c->has_gen_top_k = true;
                c->gen_top_k = (int)v->num;
            }
            if (!c->num_eos_tokens) read_eos(json_get(gj, "eos_token_id"), c);
        }
    }
    free(path);
    json_free(cj);
    json_free(gj);
    return 0;
fail:
    free(path);
    json_free(cj);
    json_free(gj);
    return -1;
}

#define REJECT(cond, msg)                                          \
    do {                                                           \
        if (cond) {                                                \
            if (err && errlen) snprintf(err, errlen, "%s", msg);   \
            return -1;                                             \
        }                                                          \
    } while (0)

/* the dense checks every family on the path shares */
static int reject_common(const model_config_t *c, char *err, size_t errlen, int allow_window, int allow_partial,
                         int allow_gate) {
    REJECT(c->attention_bias, "attention_bias not supported");
    REJECT(!allow_window && c->has_sliding_window, "sliding window attention not supported");
    REJECT(c->num_experts > 0, "MoE models not supported");
    REJECT(!c->hidden_act_silu, "only SiLU activation supported");
    REJECT(!allow_partial && c->partial_rotary_factor != 1.0f, "partial rotary embedding not supported");
    REJECT(!allow_gate && c->attn_output_gate, "attention output gate not supported");
    return 0;
}

int engine_model_check_supported(const model_config_t *c, char *err, size_t errlen) {
    if (!c) return -1;
    const char *rt = c->rope_scaling_type;
    switch (family_of(c->model_type)) {
    case FAM_QWEN3:
        if (reject_common(c, err, errlen, 0, 0, 0)) return -1;
        REJECT(rt[0], "RoPE scaling not supported");
        break;
    case FAM_LLAMA:
        if (reject_common(c, err, errlen, 0, 0, 0)) return -1;
        REJECT(rt[0] && strcmp(rt, "linear") && strcmp(rt, "llama3") && strcmp(rt, "default"),
               "unsupported RoPE scaling type");
        REJECT(!strcmp(rt, "linear"), "linear RoPE scaling not supported by the CUDA path");
        if (!strcmp(rt, "llama3")) {
            REJECT(c->rope_scaling_factor <= 0.0f, "llama3 rope_scaling_factor must be > 0");
            REJECT(c->rope_original_max_position_embeddings <= 0,
                   "llama3 rope_original_max_position_embeddings must be > 0");
            REJECT(c->rope_low_freq_factor <= 0.0f, "llama3 rope_low_freq_factor must be > 0");
            REJECT(c->rope_high_freq_factor <= c->rope_low_freq_factor,
                   "llama3 rope_high_freq_factor must be > rope_low_freq_factor");
        }
        REJECT(c->has_qk_norm, "qk_norm not supported for llama");
        break;
    case FAM_MISTRAL:
        if (reject_common(c, err, errlen, 1, 0, 0)) return -1;
        REJECT(c->has_qk_norm, "qk_norm not supported for mistral");
        REJECT(rt[0], "RoPE scaling not supported");
        break;
    case FAM_QWEN3_5: {
        if (reject_common(c, err, errlen, 0, 1, 1)) return -1;
        REJECT(c->partial_rotary_factor <= 0.0f || c->partial_rotary_factor > 1.0f,
               "partial_rotary_factor must be in (0, 1]");
        const int dims = (int)((float)c->head_dim * c->partial_rotary_factor);
        REJECT(dims < 2 || (dims & 1), "partial_rotary_factor yields invalid rope dims (must be even, >= 2)");
        REJECT(rt[0], "RoPE scaling not supported");
        REJECT(!c->attn_output_gate, "qwen3_5 requires attn_output_gate");
        break;
    }
    default:
        REJECT(1, "unsupported model family (only qwen3/llama/qwen3_5/mistral dense supported)");
    }
    REJECT(c->quant_bits != 0 && c->quant_bits != 4, "only 4-bit quantization supported");
    REJECT(c->quant_bits == 4 && c->quant_group_size != 32 && c->quant_group_size != 64,
           "quantization group size must be 32 or 64");
    return 0;
}

int model_config_to_cuda(const model_config_t *c, int tp_rank, int tp_size, mlxd_model_config *o, char *err,
                         size_t errlen) {
    if (!c || !o) return -1;
    if (engine_model_check_supported(c, err, errlen)) return -1;
    memset(o, 0, sizeof(*o));
    o->family = family_of(c->model_type);
    o->vocab = c->vocab_size;
    o->hidden = c->hidden_size;
    o->layers = c->num_hidden_layers;
    o->n_heads = c->num_attention_heads;
    o->n_kv_heads = c->num_key_value_heads;
    o->head_dim = c->head_dim;
    o->inter = c->intermediate_size;
    o->max_pos = c->max_position_embeddings;
    o->eps = c->rms_norm_eps;
    o->rope_theta = c->rope_theta;
    o->qk_norm = c->has_qk_norm;
    o->tie = c->tie_word_embeddings;
    o->attn_gate = c->attn_output_gate;
    o->rope_dims = c->partial_rotary_factor != 1.0f ? (int)((float)c->head_dim * c->partial_rotary_factor)
                                                    : c->head_dim;
    if (!strcmp(c->rope_scaling_type, "llama3")) {
        o->rope_llama3 = 1;
        o->rope_factor = c->rope_scaling_factor;
        o->rope_lo = c->rope_low_freq_factor;
        o->rope_hi = c->rope_high_freq_factor;
        o->rope_orig_max = c->rope_original_max_position_embeddings;
    }
    o->window = o->family == MLXD_MISTRAL && c->has_sliding_window ? c->sliding_window : 0;
    o->qbits = c->quant_bits;
    o->qgroup = c->quant_bits ? c->quant_group_size : 64;
    o->n_eos = c->num_eos_tokens;
    for (int i = 0; i < c->num_eos_tokens && i < 8; i++) o->eos[i] = c->eos_token_ids[i];
    o->tp_rank = tp_rank;
    o->tp_size = tp_size;
    return 0;
}

/* ------------------------------------------------------------ shards */

static int cmp_str(const void *a, const void *b) { return strcmp(*(char *const *)a, *(char *const *)b); }

typedef struct {
    char **v;
    int n, cap;
} strlist;

static int sl_push(strlist *l, char *s) {
    if (l->n == l->cap) {
        int nc = l->cap ? 2 * l->cap : 16;
        char **nv = realloc(l->v, sizeof(char *) * (size_t)nc);
        if (!nv) return -1;
        l->v = nv;
        l->cap = nc;
    }
    l->v[l->n++] = s;
    return 0;
}

static void sl_free(strlist *l) {
    for (int i = 0; i < l->n; i++) free(l->v[i]);
    free(l->v);
    l->v = NULL;
    l->n = l->cap = 0;
}

static int ends_with(const char *s, const char *suf) {
    size_t a = strlen(s), b = strlen(suf);
    return a >= b && !strcmp(s + a - b, suf);
}

/* 0 ok, 1 no index, -2 invalid index; files (sorted, unique) and the index's
   tensor names */
static int shards_from_index(const char *dir, strlist *files, strlist *keys) {
    char *ip = join(dir, "model.safetensors.index.json");
    if (!ip) return -2;
    if (!is_file(ip)) {
        free(ip);
        return 1;
    }
    json_val *doc = json_parse_file(ip, NULL, 0);
    free(ip);
    const json_val *wm = json_get(doc, "weight_map");
    if (!wm || wm->type != JSON_OBJ) {
        json_free(doc);
        return -2;
    }
    for (int i = 0; i < wm->n; i++) {
        const json_val *fv = wm->items[i];
        if (fv->type != JSON_STR) continue;
        const char *f = fv->str;
        if (strlen(f) < 13 || strchr(f, '/') || !strncmp(f, "..", 2) || !ends_with(f, ".safetensors")) goto bad;
        char *k = strdup(wm->keys[i]);
        if (!k || sl_push(keys, k)) goto bad;
        int dup = 0;
        for (int j = 0; j < files->n && !dup; j++) {
            const char *b = strrchr(files->v[j], '/');
            dup = !strcmp(b ? b + 1 : files->v[j], f);
        }
        if (dup) continue;
        char *full = join(dir, f);
        if (!full || sl_push(files, full)) goto bad;
    }
    json_free(doc);
    if (!files->n) return -2;
    qsort(files->v, (size_t)files->n, sizeof(char *), cmp_str);
    return 0;
bad:
    json_free(doc);
    return -2;
}

static int shards_glob(const char *dir, strlist *files) {
    char *single = join(dir, "model.safetensors");
    if (single && is_file(single)) return sl_push(files, single);
    free(single);
    DIR *d = opendir(dir);
    if (!d) return -1;
    struct dirent *e;
    while ((e = readdir(d))) {
        if (strlen(e->d_name) < 13 || !ends_with(e->d_name, ".safetensors")) continue;
        char *full = join(dir, e->d_name);
        if (!full) break;
        if (!is_file(full) || sl_push(files, full)) free(full);
    }
    closedir(d);
    if (!files->n) return -1;
    qsort(files->v, (size_t)files->n, sizeof(char *), cmp_str);
    return 0;
}

static int find_tensor(const mlxd_checkpoint *ck, const char *name) {
    for (int i = 0; i < ck->n_tensors; i++)
        if (!strcmp(ck->tensors[i].name, name)) return i;
    return -1;
}

static int has_prefix(const mlxd_checkpoint *ck, const char *p) {
    size_t n = strlen(p);
    for (int i = 0; i < ck->n_tensors; i++)
        if (!strncmp(ck->tensors[i].name, p, n)) return 1;
    return 0;
}

static int dtype_of(const char *s, int *size) {
    if (!strcmp(s, "BF16")) { *size = 2; return MLXD_BF16; }
    if (!strcmp(s, "F32")) { *size = 4; return MLXD_F32; }
    if (!strcmp(s, "U32")) { *size = 4; return MLXD_U32; }
    return 0;
}

/* one shard: map it, read its header, append its tensors */
static int load_shard(mlxd_checkpoint *ck, const char *path, char *err, size_t errlen) {
    json_val *hdr = NULL;
    int fd = open(path, O_RDONLY);
    if (fd < 0) FAIL("shard file not found: %s", path);
    struct stat st;
    if (fstat(fd, &st) || st.st_size < 8) {
        close(fd);
        FAIL("failed to load %s", path);
    }
    const size_t size = (size_t)st.st_size;
    unsigned char *base = mmap(NULL, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (base == MAP_FAILED) FAIL("failed to map %s", path);
    void **nm = realloc(ck->maps, sizeof(void *) * (size_t)(ck->n_maps + 1));
    size_t *ns = realloc(ck->map_sizes, sizeof(size_t) * (size_t)(ck->n_maps + 1));
    if (nm) ck->maps = nm;
    if (ns) ck->map_sizes = ns;
    if (!nm || !ns) {
        munmap(base, size);
        FAIL("out of memory");
    }
    ck->maps[ck->n_maps] = base;
    ck->map_sizes[ck->n_maps++] = size;
    uint64_t hl = 0;
    for (int i = 0; i < 8; i++) hl |= (uint64_t)base[i] << (8 * i);
    if (hl == 0 || hl > size - 8 || hl > (100u << 20)) FAIL("failed to load %s: bad header length", path);
    hdr = json_parse((const char *)base + 8, (size_t)hl, err, errlen);
    if (!hdr || hdr->type != JSON_OBJ) FAIL("failed to load %s: bad header", path);
    const size_t data0 = 8 + (size_t)hl;
    for (int i = 0; i < hdr->n; i++) {
        const char *name = hdr->keys[i];
        if (!strcmp(name, "__metadata__")) continue;
        const json_val *t = hdr->items[i];
        const char *ds = json_str(t, "dtype");
        const json_val *shape = json_get(t, "shape"), *off = json_get(t, "data_offsets");
        int esz = 0;
        const int dt = ds ? dtype_of(ds, &esz) : 0;
        if (!dt) FAIL("tensor \"%s\" in %s has unsupported dtype %s", name, path, ds ? ds : "(none)");
        if (!shape || shape->type != JSON_ARR || shape->n > 4 || !off || off->type != JSON_ARR || off->n != 2)
            FAIL("tensor \"%s\" in %s: bad shape or offsets", name, path);
        if (find_tensor(ck, name) >= 0) FAIL("duplicate tensor \"%s\" in shard %s", name, path);
        mlxd_tensor T;
        memset(&T, 0, sizeof T);
        T.dtype = dt;
        T.ndim = shape->n;
        size_t numel = 1;
        for (int d = 0; d < shape->n; d++) {
            const double v = json_num(shape->items[d], -1);
            if (v < 0) FAIL("tensor \"%s\" in %s: bad shape", name, path);
            T.shape[d] = (int64_t)v;
            numel *= (size_t)v;
        }
        const double a = json_num(off->items[0], -1), b = json_num(off->items[1], -1);
        if (a < 0 || b < a || data0 + (size_t)b > size || (size_t)(b - a) != numel * (size_t)esz)
            FAIL("tensor \"%s\" in %s: data offsets out of range", name, path);
        T.data = base + data0 + (size_t)a;
        T.name = strdup(name);
        mlxd_tensor *nt = realloc(ck->tensors, sizeof(mlxd_tensor) * (size_t)(ck->n_tensors + 1));
        if (!T.name || !nt) {
            free((void *)T.name);
            FAIL("out of memory");
        }
        ck->tensors = nt;
        ck->tensors[ck->n_tensors++] = T;
    }
    json_free(hdr);
    return 0;
fail:
    json_free(hdr);
    return -1;
}

static int is_float(int dt) { return dt == MLXD_BF16 || dt == MLXD_F32; }

/* weights_validate_expected: one projection (base name) of the family */
static int check_proj(const mlxd_checkpoint *ck, const model_config_t *c, const char *base, char *err,
                      size_t errlen) {
    char w[300], s[300], b[300];
    snprintf(w, sizeof w, "%s.weight", base);
    snprintf(s, sizeof s, "%s.scales", base);
    snprintf(b, sizeof b, "%s.biases", base);
    const int iw = find_tensor(ck, w);
    if (iw < 0) FAIL("missing expected tensor \"%s\"", w);
    if (ck->tensors[iw].dtype == MLXD_U32) {
        if (c->quant_bits <= 0) FAIL("tensor \"%s\" is uint32 but config has no quantization", w);
        const int is = find_tensor(ck, s), ib = find_tensor(ck, b);
        if (is < 0 || ib < 0) FAIL("quantized tensor \"%s\" missing scales/biases", base);
        if (!is_float(ck->tensors[is].dtype)) FAIL("scales \"%s\" has non-float dtype", s);
        if (!is_float(ck->tensors[ib].dtype)) FAIL("biases \"%s\" has non-float dtype", b);
    } else if (!is_float(ck->tensors[iw].dtype)) {
        FAIL("tensor \"%s\" has unexpected dtype (expected float or uint32)", w);
    }
    return 0;
fail:
    return -1;
}

static int check_norm(const mlxd_checkpoint *ck, const char *name, char *err, size_t errlen) {
    const int i = find_tensor(ck, name);
    if (i < 0) FAIL("missing expected tensor \"%s\"", name);
    if (!is_float(ck->tensors[i].dtype)) FAIL("norm tensor \"%s\" has non-float dtype", name);
    return 0;
fail:
    return -1;
}

static int validate(const mlxd_checkpoint *ck, const model_config_t *c, const strlist *index_keys, char *err,
                    size_t errlen) {
    char name[300];
    for (int i = 0; i < index_keys->n; i++)
        if (find_tensor(ck, index_keys->v[i]) < 0)
            FAIL("index declares tensor \"%s\" but it was not found in shards", index_keys->v[i]);
    for (int l = 0; l < c->num_hidden_layers; l++) {
        snprintf(name, sizeof name, "model.layers.%d.", l);
        if (!has_prefix(ck, name)) FAIL("missing tensors for layer %d", l);
    }
    if (find_tensor(ck, "model.embed_tokens.weight") < 0) FAIL("missing model.embed_tokens.weight");
    if (c->quant_bits > 0) {
        int found = 0;
        for (int i = 0; i < ck->n_tensors; i++) {
            const char *k = ck->tensors[i].name;
            if (!ends_with(k, ".scales")) continue;
            snprintf(name, sizeof name, "%.*s.weight", (int)(strlen(k) - 7), k);
            const int iw = find_tensor(ck, name);
            if (iw < 0) continue;
            if (ck->tensors[iw].dtype != MLXD_U32) FAIL("quantized weight %s has dtype %d, expected uint32", name,
                                                        ck->tensors[iw].dtype);
            found = 1;
        }
        if (!found)
            FAIL("quantized config (bits=%d) but no quantized weights found (expected uint32 dtype with "
                 "scales/biases)", c->quant_bits);
    }
    for (int i = 0; i < ck->n_tensors; i++) {
        const char *k = ck->tensors[i].name;
        const int sc = ends_with(k, ".scales"), bi = ends_with(k, ".biases");
        if (!sc && !bi) continue;
        const int bl = (int)strlen(k) - 7;
        snprintf(name, sizeof name, "%.*s.weight", bl, k);
        if (find_tensor(ck, name) < 0)
            FAIL("orphan %s for \"%.*s\" (base .weight missing)", sc ? ".scales" : ".biases", bl, k);
        snprintf(name, sizeof name, "%.*s.%s", bl, k, sc ? "biases" : "scales");
        if (find_tensor(ck, name) < 0)
            FAIL("orphan %s for \"%.*s\" (missing %s)", sc ? ".scales" : ".biases", bl, k,
                 sc ? ".biases" : ".scales");
    }
    static const char *const projs[] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                                        "self_attn.o_proj", "mlp.gate_proj",    "mlp.up_proj",
                                        "mlp.down_proj"};
    if (check_proj(ck, c, "model.embed_tokens", err, errlen)) return -1;
    if (!c->tie_word_embeddings && check_proj(ck, c, "lm_head", err, errlen)) return -1;
    if (check_norm(ck, "model.norm.weight", err, errlen)) return -1;
    for (int l = 0; l < c->num_hidden_layers; l++) {
        for (size_t p = 0; p < sizeof projs / sizeof projs[0]; p++) {
            snprintf(name, sizeof name, "model.layers.%d.%s", l, projs[p]);
            if (check_proj(ck, c, name, err, errlen)) return -1;
        }
        static const char *const norms[] = {"input_layernorm", "post_attention_layernorm", "self_attn.q_norm",
                                            "self_attn.k_norm"};
        const int nn = c->has_qk_norm ? 4 : 2;
        for (int p = 0; p < nn; p++) {
            snprintf(name, sizeof name, "model.layers.%d.%s.weight", l, norms[p]);
            if (check_norm(ck, name, err, errlen)) return -1;
        }
    }
    return 0;
fail:
    return -1;
}

int mlxd_checkpoint_open(mlxd_checkpoint *ck, const char *dir, const model_config_t *cfg, char *err,
                         size_t errlen) {
    strlist files = {0}, keys = {0};
    if (!ck || !dir || !cfg) return -1;
    memset(ck, 0, sizeof(*ck));
    if (err && errlen) err[0] = '\0';
    const int ir = shards_from_index(dir, &files, &keys);
    if (ir == -2) FAIL("invalid model.safetensors.index.json in %s", dir);
    if (ir == 1 && shards_glob(dir, &files)) FAIL("no safetensors files found in %s", dir);
    for (int i = 0; i < files.n; i++)
        if (load_shard(ck, files.v[i], err, errlen)) goto fail;
    if (validate(ck, cfg, &keys, err, errlen)) goto fail;
    sl_free(&files);
    sl_free(&keys);
    return 0;
fail:
    sl_free(&files);
    sl_free(&keys);
    mlxd_checkpoint_close(ck);
    return -1;
}

void mlxd_checkpoint_close(mlxd_checkpoint *ck) {
    if (!ck) return;
    for (int i = 0; i < ck->n_tensors; i++) free((void *)ck->tensors[i].name);
    for (int i = 0; i < ck->n_maps; i++) munmap(ck->maps[i], ck->map_sizes[i]);
    free(ck->tensors);
    free(ck->maps);
    free(ck->map_sizes);
    memset(ck, 0, sizeof(*ck));
}
