/*
 * libmlxd_engine -- the engine-side C11 surface of tlkahn/mlxd over
 * libmlxd_cuda, so that the reference's generate loop (src/engine/engine.c,
 * handle_generate_real) builds against this header instead of mlx-c:
 *
 *   src/engine/emodel.h    engine_model_t, engine_model_check_supported,
 *                          engine_model_load, engine_model_free, model_forward
 *   src/engine/kvcache.h   kvcache_t, kvcache_init/free/layer_offset/
 *                          capacity/update/view
 *   src/engine/sampler.h   sampler_key_t, sampler_key_init/next/free,
 *                          sampling_resolve, sampler_sample_lazy
 *   src/mlxbridge/         the calls engine.c makes: mlx_array_new/free,
 *                          mlx_array_new_data, mlx_reshape,
 *                          mlxbridge_gpu_stream, mlxbridge_async_eval_n,
 *                          mlxbridge_item_int32/float32,
 *                          mlxbridge_synchronize, mlxbridge_clear_cache
 *   src/model/weights.c    the safetensors loader with its validation
 *                          (mlxd_checkpoint_open)
 *
 * mlx_array is this library's handle: a device tensor (bf16, f32, int32 or
 * u32; up to 4 dims) or a sampler subkey. Functions enqueue their work on
 * the engine stream (mlxbridge_gpu_stream) and return, which is the
 * reference's lazy evaluation: mlxbridge_async_eval_n only checks its
 * arguments, and the item reads wait for the stream. Buffers released by
 * mlx_array_free return to a cache reused in stream order (all work is on
 * one stream); mlxbridge_clear_cache frees the cache. Engine-thread only,
 * one GPU (mlxd_cuda_init selects it); tensor parallelism stays on the
 * libmlxd_cuda API.
 */
#ifndef MLXD_ENGINE_H
#define MLXD_ENGINE_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "mlxd_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- handles (mlx-c's are structs holding one pointer; so are these) ---- */
typedef struct { void *ctx; } mlx_array;
typedef struct { void *ctx; } mlx_stream;
typedef enum { MLX_UINT32 = 3, MLX_INT32 = 7, MLX_FLOAT32 = 10, MLX_BFLOAT16 = 12 } mlx_dtype;

mlx_array mlx_array_new(void);
int       mlx_array_free(mlx_array a);
/* copies `data` (host) into a new device array */
mlx_array mlx_array_new_data(const void *data, const int *shape, int dim, mlx_dtype dtype);
int       mlx_reshape(mlx_array *res, mlx_array a, const int *shape, size_t shape_num, mlx_stream s);
size_t    mlx_array_ndim(mlx_array a);
int       mlx_array_dim(mlx_array a, int dim);
mlx_dtype mlx_array_dtype(mlx_array a);
/* device address of the data (NULL for an empty handle or a subkey) */
void     *mlxd_array_data(mlx_array a);

mlx_stream mlxbridge_gpu_stream(void);
int  mlxbridge_get_shape(mlx_array arr, int *dims, int max_dims);
int  mlxbridge_async_eval(mlx_array a);
int  mlxbridge_async_eval_n(const mlx_array *arrs, size_t n);
int  mlxbridge_item_int32(int32_t *out, mlx_array a);
int  mlxbridge_item_float32(float *out, mlx_array a);
int  mlxbridge_synchronize(mlx_stream s);
int  mlxbridge_clear_cache(void);
int  mlxbridge_get_active_memory(size_t *out);
int  mlxbridge_get_peak_memory(size_t *out);

/* ---- model config (src/model/model.h: the fields on the decode path) ---- */
typedef struct {
    char  model_type[32];
    int   vocab_size, hidden_size, num_hidden_layers, num_attention_heads,
          num_key_value_heads, max_position_embeddings, intermediate_size, head_dim;
    float rms_norm_eps, rope_theta;
    char  rope_scaling_type[16];       /* "" = none */
    float rope_scaling_factor, rope_low_freq_factor, rope_high_freq_factor;
    int   rope_original_max_position_embeddings;
    float partial_rotary_factor;
    bool  has_sliding_window;
    int   sliding_window;
    bool  attention_bias;
    int   quant_bits, quant_group_size;
    bool  tie_word_embeddings;
    bool  has_qk_norm;
    bool  attn_output_gate;
    bool  hidden_act_silu;
    int   num_experts;
    int   num_eos_tokens;
    int   eos_token_ids[8];
    /* generation_config.json sampling defaults */
    bool  has_gen_temperature, has_gen_top_p, has_gen_top_k;
    float gen_temperature, gen_top_p;
    int   gen_top_k;
} model_config_t;

/* config.json (+ generation_config.json) of a model directory, the dense
   families on the path: qwen3, llama, mistral, qwen3_5 (model.c:667-1031) */
int model_config_load(model_config_t *cfg, const char *model_dir, char *err, size_t errlen);
/* the library config of a loaded model_config_t (tensor-parallel shard) */
int model_config_to_cuda(const model_config_t *cfg, int tp_rank, int tp_size, mlxd_model_config *out,
                         char *err, size_t errlen);

/* ---- checkpoint (src/model/weights.c:20-192, 752-1060) ------------------
   Shards from model.safetensors.index.json (file names checked: *.safetensors
   in the directory itself), else model.safetensors, else every
   *.safetensors (sorted). Each file is mapped read-only; tensors must be
   BF16, F32 or U32. Validation: duplicate names across shards, every name
   the index declares present, every layer and the embedding present, the
   expected projection / norm set of the family, quantized weights u32 with
   float scales and biases, no orphan scales or biases. */
typedef struct {
    mlxd_tensor *tensors;
    int          n_tensors;
    void       **maps;
    size_t      *map_sizes;
    int          n_maps;
} mlxd_checkpoint;
int  mlxd_checkpoint_open(mlxd_checkpoint *ck, const char *model_dir, const model_config_t *cfg,
                          char *err, size_t errlen);
void mlxd_checkpoint_close(mlxd_checkpoint *ck);

/* ---- engine model (src/engine/emodel.h:11-28) --------------------------- */
typedef struct engine_model {
    model_config_t cfg;
    mlxd_model    *m;
    mlx_stream     stream;
    bool           stub;
} engine_model_t;

typedef struct {
    int  offset;        /* positions written (rope offset of the next token) */
    int  capacity;
    int  n_kv_heads;    /* recorded on first update */
    int  head_dim;
    bool initialized;
} kv_entry_t;

typedef struct {
    kv_entry_t *entries;   /* one per layer */
    int         num_layers;
    mlxd_kv    *dev;       /* the device cache, made by the first update */
    const engine_model_t *em;
} kvcache_t;

int  engine_model_check_supported(const model_config_t *cfg, char *err, size_t errlen);
int  engine_model_load(engine_model_t *em, const char *model_dir, char *err, size_t errlen);
void engine_model_free(engine_model_t *em);
/* ids [1, n] int32 (device); appends n positions to kv; *logits_out (a live
   handle, replaced on success) gets the last position's logits [1, 1, V]
   bf16 when want_logits */
int  model_forward(engine_model_t *em, mlx_array ids, kvcache_t *kv, bool want_logits,
                   mlx_array *logits_out);

/* ---- KV cache (src/engine/kvcache.h:11-51) ------------------------------ */
int  kvcache_init(kvcache_t *kv, int num_layers);
void kvcache_free(kvcache_t *kv);
int  kvcache_layer_offset(const kvcache_t *kv, int layer);
int  kvcache_capacity(const kvcache_t *kv, int layer);
/* new_k / new_v [1, H, n, D] bf16 appended at the layer's offset; views
   [1, H, len, D] of the layer after the update, the last max_kv rows on
   one-token updates when max_kv > 0 (copies; the cache needs a model bound
   by a model_forward, or kvcache_bind) */
int  kvcache_update(kvcache_t *kv, int layer, mlx_array new_k, mlx_array new_v, int max_kv,
                    mlx_array *k_view, mlx_array *v_view, mlx_stream s);
int  kvcache_view(const kvcache_t *kv, int layer, int max_kv, int q_len, mlx_array *k_view,
                  mlx_array *v_view, mlx_stream s);
/* makes the device cache for em now (model_forward does it on first use) */
int  kvcache_bind(kvcache_t *kv, const engine_model_t *em);

/* ---- sampler (src/engine/sampler.h:11-50, src/core/types.h:21-42) ------- */
typedef struct {
    float temperature;
    float top_p;
    int   top_k;
    float min_p;
    int   seed;
} sampling_params_t;
#define SAMPLING_PARAMS_DEFAULT \
    ((sampling_params_t){.temperature = 1.0f, .top_p = 1.0f, .top_k = -1, .min_p = 0.0f, .seed = -1})
#define SAMPLING_SET_TEMPERATURE (1u << 0)
#define SAMPLING_SET_TOP_P       (1u << 1)
#define SAMPLING_SET_TOP_K       (1u << 2)
#define SAMPLING_SET_MIN_P       (1u << 3)
#define SAMPLING_SET_SEED        (1u << 4)

typedef struct { mlx_array key; bool seeded; } sampler_key_t;
int  sampler_key_init(sampler_key_t *k, int seed);
int  sampler_key_next(sampler_key_t *k, mlx_array *subkey_out, mlx_stream s);
void sampler_key_free(sampler_key_t *k);
sampling_params_t sampling_resolve(const sampling_params_t *req, unsigned set_mask,
                                   const model_config_t *cfg);
/* temperature, top_k, top_p, min_p, categorical draw on the last row of
   logits; temperature < 0.01 is greedy. *tok_out: int32 [1];
   *logprob_out: f32 [1] when want_logprob */
int  sampler_sample_lazy(mlx_array logits, const sampling_params_t *sp, mlx_array subkey,
                         bool want_logprob, mlx_stream s, mlx_array *tok_out,
                         mlx_array *logprob_out);

#ifdef __cplusplus
}
#endif

#endif /* MLXD_ENGINE_H */
