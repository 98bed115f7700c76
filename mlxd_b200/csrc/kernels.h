// Host-side launchers of the device kernels (internal).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "internal.h"

namespace mlxd {

// ---- repack (qgemv.cu)
// MLX-format triplet rows [r0, r0+nrows) x cols [c0, c0+ncols) of a source
// with row strides ldw (u32 words) / lds (scale elements), written as
// destination row blocks dst_rb0 + dst_rb_stride * i.
int repack_quant(QMat &dst, const uint32_t *w, const void *s, const void *b, int sdtype,
                 int ldw, int lds, int r0, int nrows, int c0, int dst_rb0, int dst_rb_stride,
                 cudaStream_t st);

// ---- decode GEMV (qgemv.cu)
enum { PRO_PLAIN = 0, PRO_RMSNORM = 1 };
enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3, EPI_PARTIAL_F32 = 4 };
struct GemvArgs {
    const uint8_t *tiles;
    const uint8_t *sb;
    const uint8_t *sb8;         // fast-path scale/bias records (set by qgemv)
    const uint8_t *ti8, *sbi;   // integer-MMA layout (set by qgemv)
    int rows, cols;
    const uint16_t *x;          // bf16 [cols]
    const uint16_t *norm_w;     // PRO_RMSNORM
    float eps;
    uint16_t *y;                // bf16 [rows] (EPI_SWIGLU: [rows/2])
    float *yf;                  // EPI_PARTIAL_F32: f32 [rows]
    const uint16_t *residual;   // EPI_RESIDUAL
    unsigned long long *amax;   // EPI_ARGMAX
    int row_offset;             // EPI_ARGMAX: global index of row 0
    float *ws;                  // split row-block partials [units][slots][16 or 32]
    int *cnt;                   // per-unit arrival counters (zero between launches)
    int ws_slots;               // set by the launcher
    PfList pf;                  // weight-stream ranges this launch requests into L2
    int grid_cap;               // at most this many CTAs (0: one per SM)
    int res_early;              // EPI_RESIDUAL: the residual was complete before the producer of
                                // x started, so a chained launch requests it before its wait
};
int qgemv(const QMat &W, int pro, int epi, GemvArgs a, cudaStream_t st, bool pdl);
// the arrays (pointer, bytes) that the decode GEMV of W reads, in order
void qgemv_stream(const QMat &W, std::vector<std::pair<const unsigned char *, size_t>> &out);
// workspace floats one matrix needs (units -> counters)
size_t gemv_workspace_floats(int rows, int cols, int group, int epi, int sms, int *units);
int num_sms();
// decode GEMV (EPI_STORE) with its workspace in a static device array instead
// of a caller-provided allocation; -1 when the matrix needs more than it holds
int qgemv_static_scratch(const QMat &W, const uint16_t *x, uint16_t *y, cudaStream_t st);

// ---- persistent decode step (megastep.cu)
int megastep_setup(mlxd_model *m);          // 0 also when the model is not eligible
void megastep_free(mlxd_model *m);
bool megastep_ready(const mlxd_model *m, const mlxd_kv *kv);
int megastep_launch(mlxd_model *m, mlxd_kv *kv, const int32_t *ids_dev, uint16_t *logits, bool argmax,
                    cudaStream_t st);
int megastep_timeouts(mlxd_model *m);

// ---- prefill GEMM / dense (qgemm.cu)
// y[S][rows] = x[S][cols] . W^T with epilogue (STORE/RESIDUAL/SWIGLU)
int linear_multi(const QMat &W, const uint16_t *x, int S, uint16_t *y, int epi,
                 const uint16_t *residual, float *yf, cudaStream_t st);
// the same on tcgen05 (qgemm_tc.cu) for group-64 bf16-scale matrices with
// rows a multiple of 128; timeouts: nonzero once a launch gave up a wait
bool qgemm_tc_eligible(const QMat &W, int S);
int qgemm_tc(const QMat &W, const uint16_t *x, int S, uint16_t *y, int epi, const uint16_t *res, float *yf,
             cudaStream_t st);
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
int add_residual(uint16_t *h, const uint16_t *y, size_t n, cudaStream_t st);

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
    float *part;
    int *count;
    int nsplit;
    uint16_t *out;           // [hq*D]
    PfList pf;               // weight-stream ranges this launch requests into L2
};
int attention_decode(const AttnDecodeArgs &a, cudaStream_t st, bool pdl);
// the tensor-core decode kernel (one cluster per kv head): 0 launched, 1 not
// applicable to the shape or device, -1 error
int attention_decode_tc(const AttnDecodeArgs &a, cudaStream_t st, bool pdl);
// SMs the decode attention kernel holds (one CTA each) for this shape; 0 when
// the tensor-core kernel does not serve it
int attention_decode_tc_sms(const AttnDecodeArgs &a);
// prefill (S queries at positions pos0..): q [S][hq][D]; gate [S][qdim] or null
int attention_prefill(const uint16_t *q, int S, int pos0, const uint16_t *kc,
                      const uint16_t *vc, int cap, int window, int hq, int hkv, int D,
                      const uint16_t *gate_src, int qdim, uint16_t *out, cudaStream_t st);

// ---- sampler (sampler.cu)
// d_nctx / d_step (optional): the context length and the draw's step read
// from device memory instead of n_ctx / step, so that the launches can be
// replayed from a CUDA graph; sample_reserve(V) then runs before the capture
int sample(const void *logits, int dtype, int V, const mlxd_sampling &sp, const int32_t *ctx,
           int n_ctx, uint64_t step, int32_t *tok, float *lp, uint8_t *keep, cudaStream_t st,
           const int32_t *d_nctx = nullptr, const unsigned long long *d_step = nullptr);
int sample_reserve(int V);
int argmax_decode(const unsigned long long *amax, int32_t *tok, cudaStream_t st);

}  // namespace mlxd
