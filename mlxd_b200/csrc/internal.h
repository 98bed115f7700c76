// Internal structures of libmlxd_cuda (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>
#include <string>
#include <vector>

#include "../../include/mlxd_cuda.h"

namespace mlxd {

void set_error(const char *fmt, ...);
bool cuda_ok(cudaError_t e, const char *what);
#define MLXD_CHECK(call) do { if (!::mlxd::cuda_ok((call), #call)) return -1; } while (0)

void *dev_alloc(size_t bytes);      // tracked cudaMalloc (nullptr + error on failure)
void dev_free(void *p);

// A projection in device memory. Every quantized matrix keeps its MLX
// arrays (w u32 [rows][cols/8], scales/biases [rows][cols/group] of sdtype);
// a fused gate|up matrix stores alternating 64-row blocks of gate and up
// rows. Matrices of the fast format (group 64, bf16 scales, cols a multiple
// of 512) also carry the decode layout: ti8, tiles of 16 rows x 64 columns
// whose lane words are the u8 A fragments of two mma.m16n8k32 (low nibbles:
// columns 0-31, high nibbles: 32-63), and sbi, per (16 rows, 8 groups) 16
// records of 32 B: (s, b) of rows g, g+8 for the four groups 2j + h that
// lanes (g, 2h) and (g, 2h+1) scale. Dense matrices keep bf16 [rows][cols].
struct QMat {
    int rows = 0, cols = 0;     // out, in
    int group = 64;
    int sdtype = MLXD_BF16;     // scale/bias dtype
    bool quant = true;
    uint32_t *w = nullptr;
    void *s = nullptr, *b = nullptr;
    uint8_t *ti8 = nullptr, *sbi = nullptr;
    uint16_t *dense = nullptr;
    bool fast() const {
        return quant && group == 64 && sdtype == MLXD_BF16 && cols % 512 == 0 && rows % 16 == 0;
    }
    size_t w_bytes() const { return quant ? (size_t)rows * cols / 2 : (size_t)rows * cols * 2; }
    size_t sb_bytes() const {   // scales + biases
        return quant ? (size_t)rows * (cols / group) * (sdtype == MLXD_F32 ? 8 : 4) : 0;
    }
    size_t ti8_bytes() const { return (size_t)rows * cols / 2; }
    size_t sbi_bytes() const { return (size_t)rows * cols / 16; }
    // bytes one decode step streams from HBM for this matrix
    size_t stream_bytes() const { return ti8 ? ti8_bytes() + sbi_bytes() : w_bytes() + sb_bytes(); }
};

struct Layer {
    QMat qkv, o, gateup, down;
    uint16_t *ln1 = nullptr, *ln2 = nullptr, *qn = nullptr, *kn = nullptr;
};

// MLX-format embedding table kept for the row gather.
struct Embed {
    bool quant = true;
    int sdtype = MLXD_BF16;
    uint32_t *w = nullptr;   // [V][H/8]
    void *s = nullptr, *b = nullptr;   // [V][H/G]
    uint16_t *dense = nullptr;         // [V][H]
};

}  // namespace mlxd

namespace mlxd {
struct SampWork;
}

struct mlxd_model {
    mlxd_model_config c;
    int hq, hkv, qdim;          // local heads, q rows per token (x2 with gate)
    int inter_local;            // local intermediate (tp shard)
    int vocab_local, vocab_off; // lm_head shard
    std::vector<mlxd::Layer> L;
    mlxd::QMat lm;
    mlxd::Embed embed;
    uint16_t *norm = nullptr;
    float *freqs = nullptr;     // llama3 freqs [D/2] (device) or null
    // decode scratch
    uint16_t *h = nullptr, *h1 = nullptr, *qkv = nullptr, *att = nullptr, *act = nullptr;
    uint16_t *logits = nullptr;
    unsigned long long *amax = nullptr;  // fused argmax key
    int32_t *token = nullptr;   // device token slot
    float *lp = nullptr;        // device logprob slot
    double *part_h = nullptr;   // [tp_size][hidden] f64 partials (tensor parallel)
    void *gws = nullptr;        // generic projection workspace (decode)
    size_t gws_bytes = 0;
    float *rope_cs = nullptr;   // [positions][rope_dims/2][2] cos/sin
    int rope_positions = 0;
    mlxd::SampWork *samp = nullptr;   // sampler scratch of this model
    // generate loop state
    int32_t *ctx = nullptr;     // context ids (prompt + generated)
    int32_t *n_ctx = nullptr;
    int ctx_cap = 0;
    unsigned long long *d_step = nullptr;   // sampled decoding: the draw's step
    void *graph_exec = nullptr; // cudaGraphExec_t of one decode step (greedy or sampled)
    const void *graph_kv = nullptr;
    unsigned long long graph_kv_serial = 0;   // a cache freed and another created at the same
                                              // address must not replay the old graph
    bool graph_lp = false;
    bool graph_sampled = false;
    mlxd_sampling graph_sp = {};   // the settings a sampled graph was captured with
    // prefill scratch (grown on demand)
    int pre_cap = 0;
    uint16_t *p_h = nullptr, *p_x = nullptr, *p_qkv = nullptr, *p_q = nullptr, *p_att = nullptr,
             *p_act = nullptr, *p_tmp = nullptr;
    int32_t *p_ids = nullptr;
    double *p_part = nullptr;   // [S][hidden] f64 partials (tensor parallel)
    void *p_ws = nullptr;       // projection workspace of a chunk
    size_t p_ws_bytes = 0;
    float *p_scr = nullptr;     // attention scratch of a chunk
    size_t p_scr_floats = 0;
    cudaStream_t stream = nullptr;
    // tensor parallel
    void *nccl = nullptr;       // ncclComm_t when tp_size > 1
    void *tp = nullptr;         // NVLink mailboxes of the decode step's exchanges (tp.cu)
    size_t weight_bytes = 0;
};

struct mlxd_kv {
    int layers, hkv, d, cap;
    int window;                 // ring buffer when > 0
    int offset;                 // absolute positions written (host mirror)
    uint16_t *k = nullptr, *v = nullptr;   // [L][hkv][cap][d]
    int32_t *d_pos = nullptr;   // device copy of offset (position of the next token)
    unsigned long long serial = 0;   // unique per created cache (keys the decode graph)
    // decode attention's per-step block results and arrival counters
    float *att_part = nullptr;
    int *att_cnt = nullptr;
    int att_nbmax = 0, att_rep = 0;
};
