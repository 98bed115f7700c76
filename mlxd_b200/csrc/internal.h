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

// Byte ranges of the weight stream that one decode launch requests into L2
// (multiples of 16 bytes, 16-byte aligned); n = 0: none.
constexpr int PF_MAX = 8;
struct PfList {
    const unsigned char *p[PF_MAX];
    unsigned int bytes[PF_MAX];
    int n;
};

void *dev_alloc(size_t bytes);      // tracked cudaMalloc (nullptr + error on failure)
void dev_free(void *p);

// A projection in device memory. Quantized matrices live in the tile layout
// written by repack: for row block rb (16 rows) and group g, 32 lanes of
// group/4 bytes each (tiles), plus 8 scale/bias records per tile (sb).
struct QMat {
    int rows = 0, cols = 0;     // out, in (rows a multiple of 16)
    int group = 64;
    int sdtype = MLXD_BF16;     // scale/bias dtype
    bool quant = true;
    uint8_t *tiles = nullptr;
    uint8_t *sb = nullptr;
    // decode fast path (group 64, bf16 scales, cols/64 a multiple of 8): the
    // same scales/biases regrouped per row block and block of 8 groups, one
    // 16-byte record per lane: (s,b) of rows g, g+8 x groups 2t, 2t+1
    uint8_t *sb8 = nullptr;
    // integer-MMA decode layout (same eligibility as sb8): tiles whose lane
    // words carry the u8 A fragments of two m16n8k32 MMAs (low nibbles: group
    // columns 0-31, high nibbles: 32-63), and per (row block, block of 8
    // groups) 16 records of 32 B: (s, b) of rows g, g+8 for the four groups
    // 2j + h (j = 0..3) that lanes (g, 2h) and (g, 2h+1) scale
    uint8_t *ti8 = nullptr;
    uint8_t *sbi = nullptr;
    uint16_t *dense = nullptr;  // [rows][cols] bf16 when !quant
    size_t tile_bytes() const { return (size_t)rows / 16 * (cols / group) * 32 * (group / 4); }
    size_t sb_bytes() const {
        return (size_t)rows / 16 * (cols / group) * 8 * (sdtype == MLXD_F32 ? 16 : 8);
    }
    bool fast8() const { return quant && group == 64 && sdtype == MLXD_BF16 && (cols / 64) % 8 == 0; }
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
    float *part = nullptr;      // attention split partials
    int *att_count = nullptr;   // per kv head split completion counters
    unsigned long long *amax = nullptr;  // fused argmax key
    int32_t *token = nullptr;   // device token slot
    float *lp = nullptr;        // device logprob slot
    float *part_h = nullptr;    // [hidden] f32 partial (tensor parallel)
    float *gemv_ws = nullptr;   // decode GEMV split row-block partials
    int *gemv_cnt = nullptr;    // decode GEMV per-unit counters
    float *rope_cs = nullptr;   // [positions][rope_dims/2][2] cos/sin
    int rope_positions = 0;
    int nsplit = 16;
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
    float *p_part = nullptr;
    cudaStream_t stream = nullptr;
    // persistent single-kernel decode step (megastep.cu) when eligible
    void *mega = nullptr;
    // tensor parallel
    void *nccl = nullptr;       // ncclComm_t when tp_size > 1
    size_t weight_bytes = 0;
};

struct mlxd_kv {
    int layers, hkv, d, cap;
    int window;                 // ring buffer when > 0
    int offset;                 // absolute positions written (host mirror)
    uint16_t *k = nullptr, *v = nullptr;   // [L][hkv][cap][d]
    int32_t *d_pos = nullptr;   // device copy of offset (position of the next token)
    unsigned long long serial = 0;   // unique per created cache (keys the decode graph)
};
