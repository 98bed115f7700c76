// Host-side launchers of the device kernels (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "internal.h"

namespace mlxd {

int num_sms();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel, device
// and size; false (error set) when the runtime refuses
bool smem_allowed(const void *kern, size_t bytes);

// ---- projections (qgemv.cu). Every launcher computes the group-exact
// arithmetic (gemv_i8.cuh): identical bits for decode, prefill and shards.
enum { PRO_PLAIN = 0, PRO_RMSNORM = 1 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3, EPI_PARTIAL = 4 };
struct GemvArgs {
    const uint8_t *ti8, *sbi;   // decode layout (set by qgemv)
    int rows, cols;
    const uint16_t *x;          // bf16 [S][cols]
    const uint16_t *norm_w;     // PRO_RMSNORM
    float eps;
    uint16_t *y;                // bf16 [S][rows] (EPI_SWIGLU: [S][rows/2])
    double *yf;                 // EPI_PARTIAL: f64 [S][rows] (the unrounded row values)
    const uint16_t *residual;   // EPI_RESIDUAL
    unsigned long long *amax;   // EPI_ARGMAX
    int row_offset;             // EPI_ARGMAX: global index of row 0
    void *gws;                  // generic path: workspace (generic_ws_bytes)
    size_t gws_bytes;
    int grid_cap;               // decode layout: at most this many CTAs (0: one per SM)
    int res_early;              // EPI_RESIDUAL: the residual was complete before the producer of
                                // x started, so a chained launch requests it before its wait
    // EPI_PARTIAL inside a tensor-parallel decode step (decode layout only):
    // each row value leaves as a 16-byte line {low word, epoch, high word,
    // epoch} at tp_line[p] + 4 row for every rank p (tp.cu), epoch =
    // *tp_seq * tp_mul + tp_add; yf is not written
    uint32_t *tp_line[8];
    int tp_n;
    const unsigned *tp_seq;
    unsigned tp_mul, tp_add;
};
// one token (decode); PDL-chained when pdl
int qgemv(const QMat &W, int pro, int epi, GemvArgs a, cudaStream_t st, bool pdl);
// S tokens on the generic kernels (any format)
int qgemm_generic(const QMat &W, int pro, int epi, GemvArgs a, int S, void *ws, size_t ws_bytes,
                  cudaStream_t st);
size_t generic_ws_bytes(const QMat &W, int S, int pro);
// decode layout (ti8/sbi) of a fast matrix from its MLX arrays; gateup: the
// MLX rows alternate 64 gate and 64 up rows
int build_decode_layout(QMat &M, bool gateup, cudaStream_t st);
// the one-token projection with its workspace in a static device array
// instead of a caller-provided allocation; -1 when the matrix needs more
int qgemv_static_scratch(const QMat &W, const uint16_t *x, uint16_t *y, cudaStream_t st);

// ---- prefill projections on tcgen05 (qgemm_tc.cu): same arithmetic
bool qgemm_tc_eligible(const QMat &W, int S, int epi);
int qgemm_tc(const QMat &W, const uint16_t *x, int S, int epi, const uint16_t *res, uint16_t *y, double *yf,
             void *ws, size_t ws_bytes, cudaStream_t st);
size_t qgemm_tc_ws_bytes(int S, int cols);
int qgemm_tc_timeouts();

// ---- small ops (ops.cu)
int embed_rows(const Embed &e, int H, int group, int vocab, const int32_t *ids, int S, uint16_t *h,
               cudaStream_t st);
int rmsnorm_rows(const uint16_t *x, int rows, int n, const uint16_t *w, float eps, uint16_t *y,
                 cudaStream_t st);
// prefill: q/k norm + rope + kv append for S tokens at positions pos0..pos0+S-1
struct RopeArgs {
    int D, rope_dims;
    const float *cs;     // device cos/sin table [positions][rope_dims/2][2]
};
int qk_rope_append(const uint16_t *qkv, int S, int qdim, int hq, int hkv, int gate,
                   const uint16_t *qn, const uint16_t *kn, float eps, RopeArgs r, int pos0,
                   uint16_t *q_out, uint16_t *kc, uint16_t *vc, int cap, cudaStream_t st);
// h = bf16(h + bf16(sum of f64 partials in rank order)) (tensor-parallel residual)
int add_partials(uint16_t *h_out, const uint16_t *h_in, const double *part, int nranks, size_t stride,
                 size_t n, cudaStream_t st);

// ---- tensor parallel exchanges of the decode step (tp.cu)
int tp_setup(mlxd_model *m);       // collective over the model's NCCL communicator
void tp_free(mlxd_model *m);
// out = bf16(res + bf16(sum of the ranks' f64 partials)); idx: the exchange's
// index in the step (0 .. 2L-1)
int tp_sum(mlxd_model *m, const double *part, const uint16_t *res, uint16_t *out, int idx, cudaStream_t st,
           bool pdl);
// greedy: the largest of the ranks' argmax keys -> token; position + 1,
// step counter + 1
// the row-parallel projection's send half of exchange idx, for its GEMV
// epilogue (GemvArgs tp_*), and the receive half: out = bf16(res + bf16(sum
// over ranks of the lines)); only for decode-layout projections
int tp_send_args(mlxd_model *m, int idx, GemvArgs &a);
int tp_recv(mlxd_model *m, const uint16_t *res, uint16_t *out, int idx, cudaStream_t st, bool pdl);
int tp_argmax(mlxd_model *m, unsigned long long *amax, int32_t *d_pos, int32_t *token, cudaStream_t st, bool pdl);
// every rank's logits shard into every rank's full row (tp_full_logits)
int tp_gather_logits(mlxd_model *m, const uint16_t *logits, cudaStream_t st, bool pdl);
uint16_t *tp_full_logits(mlxd_model *m);
// device step counter: every one-token step that is not greedy-fused
// advances it in its final kernel
unsigned *tp_seq(mlxd_model *m);
int tp_timeouts(mlxd_model *m);

// ---- attention (attention.cu)
struct AttnDecodeArgs {
    const uint16_t *qkv;     // [qdim + 2*hkv*D]
    int qdim, gate;
    const uint16_t *qn, *kn;
    float eps;
    RopeArgs rope;
    uint16_t *kc, *vc;       // layer cache [hkv][cap][D]
    int cap, window;
    const int32_t *d_pos;
    int hq, hkv;
    uint16_t *out;           // [hq*D]
    // the step's block results ([hkv][nbmax][rep] (m, l) and [..][D] o) and
    // one arrival counter per kv head (zero between launches)
    float *part_o, *part_l, *part_m;
    int *cnt;
    int nbmax;               // blocks the attended span can touch
};
size_t attention_decode_part_floats(int nbmax, int hkv, int rep, int D);
bool attention_decode_supported(int D, int rep, int rope_dims);
int attention_decode(const AttnDecodeArgs &a, cudaStream_t st, bool pdl);
// SMs the decode attention kernel holds (one CTA each)
int attention_decode_sms(const AttnDecodeArgs &a);
int attention_timeouts();
// prefill (S queries at positions pos0..): q [S][hq][D]; gate [S][qdim] or null
size_t attention_prefill_scratch(int S, int pos0, int window, int hq, int D);
int attention_prefill(const uint16_t *q, int S, int pos0, const uint16_t *kc,
                      const uint16_t *vc, int cap, int window, int hq, int hkv, int D,
                      const uint16_t *gate_src, int qdim, uint16_t *out, float *scr, size_t scr_floats,
                      cudaStream_t st);

// ---- sampler (sampler.cu)
// The sampler's scratch for rows of up to V logits, owned by its caller (one
// per model); d_nctx / d_step (optional): the context length and the draw's
// step read from device memory, so that the launches can be replayed from a
// CUDA graph
struct SampWork;
SampWork *samp_work_create(int V);
void samp_work_destroy(SampWork *w);
int samp_work_capacity(const SampWork *w);   // logits per row it holds
int sample(SampWork *w, const void *logits, int dtype, int V, const mlxd_sampling &sp, const int32_t *ctx,
           int n_ctx, uint64_t step, int32_t *tok, float *lp, uint8_t *keep, cudaStream_t st,
           const int32_t *d_nctx = nullptr, const unsigned long long *d_step = nullptr);

}  // namespace mlxd
