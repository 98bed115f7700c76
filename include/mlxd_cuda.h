/*
 * libmlxd_cuda -- C ABI of the B200 (sm_100a) decoder step for mlxd.
 *
 * Replaces the mlx-c bridge of tlkahn/mlxd (src/mlxbridge/mlxbridge.h:9-42)
 * and the mlx calls behind src/engine/{forward,emodel,kvcache,sampler}.h.
 * Plain C types only: pointers, sizes, ints, floats. Every function that can
 * fail returns 0 on success and -1 on failure with a message readable through
 * mlxd_cuda_last_error() (the MLXB_CHECK / log_error pattern of
 * src/mlxbridge/mlxbridge.c:14-20). Out-parameters are written only on
 * success ("freed and replaced on success, unchanged on failure",
 * src/engine/forward.h:11-12). All calls for one model must come from one
 * host thread (the engine thread, src/engine/engine.h:124-138).
 */
#ifndef MLXD_CUDA_H
#define MLXD_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtypes and families ---------------------------------------------- */
enum { MLXD_BF16 = 1, MLXD_F32 = 2, MLXD_U32 = 3, MLXD_I32 = 4 };
enum { MLXD_QWEN3 = 1, MLXD_LLAMA = 2, MLXD_MISTRAL = 3, MLXD_QWEN3_5 = 4 };

/* ---- errors ------------------------------------------------------------ */
/* Last error message of the calling thread ("" when none). */
const char *mlxd_cuda_last_error(void);

/* ---- device and streams (mlxbridge.c:6-8 gpu stream, :126-132 sync) ---- */
int mlxd_cuda_init(int device);
int mlxd_cuda_device_count(int *n);
int mlxd_cuda_stream_create(void **stream);
int mlxd_cuda_stream_destroy(void *stream);
int mlxd_cuda_synchronize(void *stream);   /* NULL = whole device */

/* ---- memory (mlxbridge.c:134-178 active/peak/cache limits) ------------- */
int    mlxd_cuda_alloc(void **dptr, size_t bytes);
int    mlxd_cuda_free(void *dptr);
int    mlxd_cuda_upload(void *dst, const void *host_src, size_t bytes, void *stream);
int    mlxd_cuda_download(void *host_dst, const void *src, size_t bytes, void *stream);
int    mlxd_cuda_memset(void *dst, int value, size_t bytes, void *stream);
size_t mlxd_cuda_active_memory(void);
size_t mlxd_cuda_peak_memory(void);

/* ---- model (emodel.h:11-28, model.h model_config_t subset) -------------- */
typedef struct {
    int   family;              /* MLXD_QWEN3 / _LLAMA / _MISTRAL / _QWEN3_5 */
    int   vocab, hidden, layers, n_heads, n_kv_heads, head_dim, inter, max_pos;
    float eps, rope_theta;
    int   qk_norm;             /* per-head RMSNorm of q and k (qwen3) */
    int   tie;                 /* lm_head = embed_tokens */
    int   attn_gate;           /* qwen3_5 attention output gate */
    int   rope_dims;           /* rotated dims (partial rotary) */
    int   rope_llama3;         /* llama3 frequency rule */
    float rope_factor, rope_lo, rope_hi;
    int   rope_orig_max;
    int   window;              /* > 0: sliding window on every layer */
    int   qbits, qgroup;       /* qbits 0 = dense bf16 weights; 4 = MLX affine */
    int   n_eos;
    int   eos[8];
    int   tp_rank, tp_size;    /* tensor-parallel shard of this process */
} mlxd_model_config;

/* One named tensor of an MLX-format checkpoint (weights.h:71-76 triplets are
   passed as their three tensors: NAME.weight u32, NAME.scales, NAME.biases). */
typedef struct {
    const char *name;
    int         dtype;         /* MLXD_BF16 / MLXD_F32 / MLXD_U32 */
    int         ndim;
    int64_t     shape[4];
    const void *data;
    int         on_device;     /* data is a device pointer of this GPU */
} mlxd_tensor;

typedef struct mlxd_model mlxd_model;
typedef struct mlxd_kv mlxd_kv;

/* engine_model_load's upload half (emodel.c:176-211): validates the tensor
   set like weights_get_triplet (weights.c:1053-1088), repacks quantized
   projections into the kernels' layouts (decode row blocks, prefill GEMM
   tiles) and keeps only this rank's shard. */
int  mlxd_cuda_model_create(mlxd_model **out, const mlxd_model_config *cfg,
                            const mlxd_tensor *tensors, int n_tensors);
void mlxd_cuda_model_destroy(mlxd_model *m);
size_t mlxd_cuda_model_weight_bytes(const mlxd_model *m);
/* Tensor parallel: bind an NCCL communicator (unique id bytes from rank 0,
   128 bytes) before the first forward when tp_size > 1. Collective: every
   rank calls it. It also maps every rank's exchange mailbox into every
   other rank (CUDA IPC): one-token steps combine their row-parallel partials,
   greedy argmax keys and, for sampling, the logits shards through those
   mailboxes inside the step, with no NCCL call; chunked prefill uses NCCL.
   A one-token step whose peer does not arrive within about a second per
   exchange fails (-1, "gave up waiting for a peer GPU"); forward then
   synchronises its stream to report it. */
int  mlxd_cuda_model_tp_init(mlxd_model *m, const void *nccl_unique_id);
int  mlxd_cuda_nccl_unique_id(void *out128);
/* Tensor-parallel shard plan, host only (no device call). The reference has
   no multi-GPU path (one mlx stream, src/engine/engine.c:360-602); this is
   the partition mlxd_cuda_model_create applies when tp_size > 1: q, k, v,
   gate, up and lm_head are split by rows (heads, intermediate, vocab), o and
   down by columns (row-parallel, on quantisation-group boundaries). Writes
   ranges[8][4] = {row0, rows, col0, cols} for q, k, v, o, gate, up, down,
   lm_head of the full matrices; -1 (last_error set) when `size` does not
   divide the heads, intermediate or vocab. */
int  mlxd_cuda_tp_plan(const mlxd_model_config *cfg, int rank, int size, int *ranges);

/* ---- KV cache (kvcache.h:11-51) ----------------------------------------
   Preallocated per-layer [Hkv][capacity][D] bf16 storage. With a sliding
   window the storage is a ring of `capacity` slots (position p in slot
   p % capacity) and attention covers positions (p - window, p]. */
int  mlxd_cuda_kv_create(mlxd_kv **out, const mlxd_model *m, int capacity);
void mlxd_cuda_kv_destroy(mlxd_kv *kv);
int  mlxd_cuda_kv_offset(const mlxd_kv *kv, int layer);    /* kvcache_layer_offset */
int  mlxd_cuda_kv_capacity(const mlxd_kv *kv, int layer);  /* kvcache_capacity */
int  mlxd_cuda_kv_reset(mlxd_kv *kv);
/* kvcache_view: copy the live rows of one layer, oldest first, as bf16 bits
   [Hkv][n][D] into host memory; *n_out = rows copied. */
int  mlxd_cuda_kv_read(mlxd_kv *kv, int layer, int is_value, uint16_t *host_out,
                       int *n_out);

/* kvcache_update / kvcache_view (kvcache.c:98-180) for callers that drive
   layers themselves: rows [pos, pos + n) of one layer (ring slots
   (pos + i) % capacity) from / to contiguous device arrays [Hkv][n][D]
   (bf16), enqueued on `stream`. kv_set_offset sets the position the next
   forward appends at (every layer). */
int  mlxd_cuda_kv_write(mlxd_kv *kv, int layer, int pos, int n, const void *k_dev,
                        const void *v_dev, void *stream);
int  mlxd_cuda_kv_gather(mlxd_kv *kv, int layer, int is_value, int pos, int n,
                         void *dst_dev, void *stream);
int  mlxd_cuda_kv_set_offset(mlxd_kv *kv, int offset, void *stream);

/* ---- forward (model_forward, emodel.c:221-337) --------------------------
   ids: n token ids (host or device memory). Appends n positions to kv.
   want_logits: write the last position's logits (bf16 [V]) to logits_dev
   (device memory); with tp_size > 1 each rank writes its vocab shard. */
int mlxd_cuda_forward(mlxd_model *m, mlxd_kv *kv, const int32_t *ids, int n,
                      int ids_on_device, int want_logits, void *logits_dev,
                      void *stream);

/* ---- single ops (forward.h dense subset) -------------------------------- */
typedef struct mlxd_linear mlxd_linear;
/* fwd_linear's weight triplet (forward.c:11-63) uploaded into the tile
   layout: w u32 [out][in/8]; scales/biases [out][in/group] (sdtype). */
int  mlxd_cuda_linear_create(mlxd_linear **out, const uint32_t *w, const void *scales,
                             const void *biases, int sdtype, int rows, int cols,
                             int group, int on_device);
void mlxd_cuda_linear_destroy(mlxd_linear *l);
/* y[S][out] (bf16) = x[S][in] (bf16) . deq(W)^T in the library's projection
   arithmetic (each group of 64 or 32 inputs in fixed point on its largest
   magnitude's grid, exact integer group sums, f64 combination, one rounding
   to bf16): S == 1 on the decode kernel, S > 1 on the chunk kernels, with
   identical bits per row. Device pointers. */
int  mlxd_cuda_linear(const mlxd_linear *l, const void *x, int S, void *y, void *stream);
/* One-token y[out] = x[in] . deq(W)^T that allocates nothing (no counterpart
   in the reference): the same projection and bits as mlxd_cuda_linear with
   S == 1, for callers that cannot allocate device memory when they call it:
   code inside a caching allocator's callback (allocating would re-enter it)
   and serving loops that hold all HBM under a fixed plan (a cudaMalloc there
   can fail, and it synchronises the device). The workspace of the generic
   kernel (the input staged in per-group fixed point, 4 bytes per column plus
   16 per group) lives in one static device array of 2 MiB + 64 KiB, held by
   every GPU that loads the library and shared by every call on it; an input
   wider than 262144 columns is rejected with -1 and a message. The first
   call on each device looks the array up and should come before any stream
   capture. Calls whose kernels can overlap on the GPU (unordered streams)
   race on the array. Device pointers. */
int  mlxd_cuda_linear_noalloc(const mlxd_linear *l, const void *x, void *y, void *stream);
/* qGEMV measurement (no reference counterpart; the decode-GEMV microbenchmark):
   launches the decode GEMV of n projections round-robin, iters rounds, on an
   internal stream bracketed by CUDA events; *ms_out = mean ms per launch.
   x: device bf16 input of max(cols); y: device output of max(rows). */
int  mlxd_cuda_linear_timed(const mlxd_linear *const *ls, int n, int iters, const void *x,
                            void *y, float *ms_out);
/* The same with every launch chained to the previous one by programmatic
   dependent launch (a launch's CTAs start and load their first weights while
   the previous one finishes), the launch mode of the decode step's graph
   (no reference counterpart). */
int  mlxd_cuda_linear_timed_chained(const mlxd_linear *const *ls, int n, int iters,
                                    const void *x, void *y, float *ms_out);
/* fwd_rmsnorm (forward.c:186-219) over rows of n; device pointers */
int  mlxd_cuda_rmsnorm(const void *x, int rows, int n, const void *w, float eps,
                       void *y, void *stream);

/* ---- sampler (sampler.h:11-50) ------------------------------------------ */
typedef struct {
    float temperature;          /* < 0.01: greedy */
    float top_p;                /* >= 1: off; <= 0: top-1 */
    int   top_k;                /* <= 0 or >= V: off */
    float min_p;                /* <= 0: off */
    int   seed;                 /* < 0: unseeded (stream 0) */
    float repetition_penalty;   /* 1 or <= 0: off (mlx-lm rule) */
    int   repetition_context;   /* last R context tokens */
} mlxd_sampling;

/* sampler_sample_lazy (sampler.c:269-380) on one row of logits (device,
   bf16 or f32). ctx_dev: n_ctx context token ids (device) for the repetition
   penalty. step: index of this draw in the request's random stream.
   Writes the token (device int32), its raw logprob (device f32, optional)
   and the final candidate mask (device u8 [V], optional). */
int mlxd_cuda_sample(const void *logits_dev, int dtype, int V, const mlxd_sampling *sp,
                     const int32_t *ctx_dev, int n_ctx, uint64_t step,
                     int32_t *tok_dev, float *logprob_dev, uint8_t *keep_dev,
                     void *stream);

/* The pipelined decode loop's pair (engine.c:470-560 over
   mlxbridge_async_eval_n + mlxbridge_item_int32, mlxbridge.c:88-124):
   step_async enqueues on `stream` the forward of the token in tok_in_dev
   (device int32) at the cache's next position and the choice of the next
   token (the sampler with sp, context ctx_dev[n_ctx] for the repetition
   penalty and draw index `step`; temperature < 0.01 is greedy) into
   tok_out_dev, with its raw logprob when logprob_dev is given, and returns
   without waiting; it may be called again with tok_out_dev as the next input
   before the token is read. read_token waits for the stream's work up to the
   call and reads one token into host memory. */
int mlxd_cuda_step_async(mlxd_model *m, mlxd_kv *kv, const int32_t *tok_in_dev,
                         const mlxd_sampling *sp, const int32_t *ctx_dev, int n_ctx,
                         uint64_t step, int32_t *tok_out_dev, float *logprob_dev,
                         void *stream);
int mlxd_cuda_read_token(const int32_t *tok_dev, int32_t *out, void *stream);

/* ---- generate (handle_generate_real, engine.c:360-602) ------------------
   Chunked prefill of prompt[:-1] (chunk tokens per forward), seed forward of
   the last prompt token, then decode with one-step lookahead: step e's
   forward is enqueued before step e-1's token is read back (4 bytes).
   Stops at an EOS id (not emitted) or after max_new tokens. prompt/out/
   logprobs are host memory. Returns the count of emitted tokens, or -1.
   timing (optional, host, 4 + max_new doubles): [0] prefill ms and [1]
   decode ms (device events), [2] tokens emitted, [3] host wall ms of the
   decode loop (launch of the first step to the last token in host memory),
   [4 + e] device time in ms from the end of prefill to the end of step e. */
int mlxd_cuda_generate(mlxd_model *m, mlxd_kv *kv, const int32_t *prompt, int n,
                       int max_new, const mlxd_sampling *sp, int chunk,
                       int32_t *out, float *logprobs, double *timing);

/* Cancellation and hooks of handle_generate_real (engine_gen_hooks_t,
   engine.h:96-120; poll sites engine.c:406-470). shutdown and cancelled are
   ints read with acquire loads (the layout of C11 atomic_int); NULL is never
   set. At every site: poll -> hook -> re-poll -> work. Sites: before each
   prefill chunk (on_prefill_chunk(ud, pos, chunk_len), pos = absolute token
   index), after the prefill before the seed step (on_before_seed), and
   before each decode step is enqueued (on_decode_step(ud, step), step = the
   count of tokens chosen before it). A set flag ends the request at that
   site: steps already enqueued finish and their tokens are emitted (a stop
   at step s's site leaves s tokens), `stopped` becomes 1 and the emitted
   count is returned. Hooks run on the calling thread and may block; they
   must not call this library for the same model. Under tensor parallelism
   every rank must stop at the same site (a hook can agree the decision
   across ranks); a rank that stops alone makes its peers' next step fail
   after the exchange's bounded wait. */
typedef struct {
    const int *shutdown;
    const int *cancelled;
    void (*on_prefill_chunk)(void *ud, int pos, int chunk_len);
    void (*on_decode_step)(void *ud, int step);
    void (*on_before_seed)(void *ud);
    void *ud;
    int stopped;               /* out */
} mlxd_gen_control;
int mlxd_cuda_generate_ctl(mlxd_model *m, mlxd_kv *kv, const int32_t *prompt, int n,
                           int max_new, const mlxd_sampling *sp, int chunk,
                           int32_t *out, float *logprobs, double *timing,
                           mlxd_gen_control *ctl);

/* ---- synthetic MLX-format weights (bench and tests) ---------------------
   Fills w (u32 [rows][cols/8]), scales, biases (bf16 [rows][cols/group]) in
   device memory with N(0, std) values (Irwin-Hall sum of 12 uniforms from
   SplitMix64 on (seed, element)) rounded to bf16, then MLX affine 4-bit
   quantisation. dense_bf16 variant fills a bf16 matrix. Bit-identical to the
   host functions below. */
int mlxd_cuda_synth_quantized(uint32_t *w, uint16_t *scales, uint16_t *biases, int rows,
                              int cols, int group, uint64_t seed, float std, void *stream);
int mlxd_cuda_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float std,
                         float constant, void *stream);
void mlxd_host_synth_quantized(uint32_t *w, uint16_t *scales, uint16_t *biases, int rows,
                               int cols, int group, uint64_t seed, float std);
void mlxd_host_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float std, float constant);

#ifdef __cplusplus
}
#endif
#endif
