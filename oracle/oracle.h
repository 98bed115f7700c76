/*
 * CPU oracle for the mlxd per-token decoder step.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, op by op and with the
 * same bf16 rounding points, what tlkahn/mlxd computes through mlx-c for one
 * forward step (src/engine/forward.c, src/engine/emodel.c), its KV cache
 * (src/engine/kvcache.c) and its sampler (src/engine/sampler.c). It is the
 * checker for the CUDA library (libmlxd_cuda) and the timed CPU baseline.
 * The product path never links, loads or calls it.
 *
 * Pinning: the oracle is checked against the reference's own golden vectors
 * (tests/test_engine_gpu.c:21-23 greedy sequence, tests/test_qwen3_5_goldens_gpu.c
 * logits, tests/test_rope_llama3.c frequency vector, tests/test_sampler_gpu.c
 * known-answer sets, tests/test_mlxbridge_gpu.c:563-642 quantized matmul).
 * The arithmetic itself lives in the un-vendored third-party mlx (>= 0.31.2) /
 * mlx-c (>= 0.6.0); the restated algorithms are named at each function.
 */
#ifndef MLXD_ORACLE_H
#define MLXD_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_QWEN3 = 1, ORC_LLAMA = 2, ORC_MISTRAL = 3, ORC_QWEN3_5 = 4 };
enum { ORC_BF16 = 1, ORC_F32 = 2, ORC_U32 = 3 };

typedef struct {
    int   family;
    int   vocab, hidden, layers, n_heads, n_kv_heads, head_dim, inter, max_pos;
    float eps, rope_theta;
    int   qk_norm;        /* qwen3 / qwen3_5 */
    int   tie;            /* lm_head is embed_tokens */
    int   attn_gate;      /* qwen3_5: q_proj emits [queries | gate] per head */
    int   rope_dims;      /* rotated dims per head (partial rotary) */
    int   rope_llama3;    /* custom freqs from the llama3 rule */
    float rope_factor, rope_lo, rope_hi;
    int   rope_orig_max;
    int   window;         /* >0: every layer is local with this window */
    int   qbits, qgroup;  /* qbits == 0: dense bf16 weights */
    int   n_eos;
    int   eos[8];
} orc_config;

typedef struct orc_model orc_model;
typedef struct orc_kv orc_kv;

/* thread count for the pthread pool (0 = all online cores) */
void orc_set_threads(int n);
int  orc_get_threads(void);

orc_model *orc_model_new(const orc_config *cfg);
/* copies the data; dtype one of ORC_BF16/ORC_F32/ORC_U32 */
int  orc_model_set_tensor(orc_model *m, const char *name, int dtype,
                          const int64_t *shape, int ndim, const void *data);
/* resolves every tensor the forward needs; -1 with a message on a gap */
int  orc_model_finalize(orc_model *m, char *err, int errlen);
void orc_model_free(orc_model *m);

orc_kv *orc_kv_new(const orc_model *m, int capacity);
void    orc_kv_free(orc_kv *kv);
int     orc_kv_offset(const orc_kv *kv, int layer);
/* copy one layer's cache rows [0, offset) out as bf16 bits [Hkv][offset][D] */
int     orc_kv_read(const orc_kv *kv, int layer, int is_value, uint16_t *out);

/* model_forward (emodel.c:221-337): ids[S] -> last-position logits as the
   float values of bf16 numbers (logits_out may be NULL when !want_logits). */
int orc_forward(orc_model *m, orc_kv *kv, const int32_t *ids, int S,
                int want_logits, float *logits_out);
/* same, but also writes the final hidden state of every position (bf16 bits,
   [S][H]) before the final norm; for layer-level parity checks */
int orc_forward_hidden(orc_model *m, orc_kv *kv, const int32_t *ids, int S,
                       uint16_t *hidden_out);

/* ---- single ops (forward.c), for kernel-level parity ---- */
/* fwd_linear (forward.c:11-63): y[S][out] (bf16 bits) = x[S][in] . deq(W)^T.
   quantized: w u32 [out][in/8], scales/biases [out][in/group] of sdtype.
   exact_dequant != 0: factorised f32 product (mlx qmv); 0: weights rounded to
   bf16 after dequantisation (mlx qmm tile load). */
void orc_qlinear(const uint16_t *x, int S, int in, int out,
                 const uint32_t *w, const void *scales, const void *biases,
                 int sdtype, int group, int exact_dequant, uint16_t *y);
void orc_dense_linear(const uint16_t *x, int S, int in, int out,
                      const uint16_t *w, uint16_t *y);
/* fwd_rmsnorm (forward.c:186-219) over rows of length n */
void orc_rmsnorm(const uint16_t *x, int rows, int n, const uint16_t *w,
                 float eps, uint16_t *y);
/* mlx_fast_rope traditional=false on one head vector (forward.c:427-456) */
void orc_rope(uint16_t *x, int D, int dims, int pos, float theta,
              const float *freqs);
/* allowed[i][j] of the attention mask for q_len queries over kv_len keys
   (window 0 = plain causal); -1 on invalid sizes (q_len > kv_len) */
int  orc_window_mask(int q_len, int kv_len, int window, uint8_t *out);
int  orc_rope_llama3_freqs(float theta, float factor, float lo, float hi,
                           int orig_max, int head_dim, float *out);
/* MLX affine quantisation (mlx ops.cpp affine_quantize); w f32 [rows][cols] */
void orc_affine_quantize(const float *w, int rows, int cols, int group,
                         uint32_t *wq, float *scales, float *biases);
void orc_dequantize_row(const uint32_t *w, const void *s, const void *b,
                        int sdtype, int cols, int group, float *out);

/* ---- sampler (sampler.c) ---- */
typedef struct {
    float temperature;
    float top_p;
    int   top_k;
    float min_p;
    int   seed;                  /* < 0: unseeded */
    float repetition_penalty;    /* <= 0 or 1: off */
    int   repetition_context;    /* last R context tokens */
} orc_sampling;

/* one sampling step over f32 logits[V]. ctx = context tokens (prompt +
   generated so far) for the repetition penalty. step = 0-based draw index
   (the counter of the draw's random stream). keep_out (optional, V bytes)
   receives the final candidate mask. Returns 0 / -1. */
int orc_sample(const float *logits, int V, const orc_sampling *sp,
               const int32_t *ctx, int n_ctx, uint64_t step,
               int32_t *tok_out, float *logprob_out, uint8_t *keep_out);
/* individual filters on f32 logits in place (-inf = masked) */
void orc_top_k(float *x, int V, int k);
void orc_top_p(float *x, int V, float p);
void orc_min_p(float *x, int V, float mp);
/* own exponential (Cody-Waite reduction + degree-7 Taylor, fmaf) shared
   bit for bit with the CUDA sampler */
float orc_expf(float x);

/* engine generate loop (engine.c:360-602): chunked prefill of prompt[:-1],
   seed forward, decode with sampling; stops at EOS or max_new.
   Returns the number of tokens written to out (EOS not emitted). */
int orc_generate(orc_model *m, const int32_t *prompt, int n, int max_new,
                 const orc_sampling *sp, int prefill_chunk,
                 int32_t *out, float *logprobs, float *margins);

/* seeded synthetic MLX-format weights (the benchmark's generator, restated
   so the CPU baseline needs no CUDA library); same bits as libmlxd_cuda's */
int  orc_synth_quantized(uint32_t *w, uint16_t *scales, uint16_t *biases, int rows, int cols,
                         int group, uint64_t seed, float std);
void orc_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float std, float constant);
/* stands in for a prefill of n positions (seeded N(0,1) keys/values): decode
   timing at context n */
int  orc_kv_fill_synth(orc_kv *kv, int n, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
