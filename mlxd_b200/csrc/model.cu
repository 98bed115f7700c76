// Model upload, KV cache, forward orchestration, generate loop: the C ABI of
// libmlxd_cuda behind src/engine/{emodel,kvcache,sampler,engine}.c.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <nccl.h>
#include <nvtx3/nvToolsExt.h>

#include "internal.h"
#include "kernels.h"

using namespace mlxd;

// ------------------------------------------------------------- small kernels

namespace mlxd {

__global__ void set_pos_kernel(int32_t *d_pos, int v) { *d_pos = v; }

// end of one decode step: advance the position; with the fused argmax, turn
// the winning key into the token id and clear the key for the next step
__global__ void step_finish_kernel(int32_t *d_pos, unsigned long long *amax, int32_t *token, unsigned *tp_seq) {
    *d_pos += 1;
    if (tp_seq) *tp_seq += 1u;
    if (amax) {
        *token = (int32_t)(0xFFFFFFFFu - (uint32_t)(*amax & 0xFFFFFFFFull));
        *amax = 0ull;
    }
}

__global__ void append_token_kernel(int32_t *ctx, int idx, const int32_t *token) { ctx[idx] = *token; }

// sampled decoding inside a CUDA graph: append the drawn token to the
// context list and advance the context length and the draw's step
__global__ void sampled_step_kernel(int32_t *ctx, int32_t *n_ctx, const int32_t *token,
                                    unsigned long long *d_step) {
    ctx[*n_ctx] = *token;
    *n_ctx += 1;
    *d_step += 1;
}

// raw logprob of the chosen token: x[tok] - logsumexp(x)
__global__ void logprob_kernel(const uint16_t *logits, int V, const int32_t *tok, float *lp) {
    __shared__ float sh[32];
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x)
        mx = fmaxf(mx, __uint_as_float((uint32_t)logits[i] << 16));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) mx = fmaxf(mx, sh[i]);
    __syncthreads();
    float s = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x)
        s += expf(__uint_as_float((uint32_t)logits[i] << 16) - mx);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
        *lp = __uint_as_float((uint32_t)logits[*tok] << 16) - (mx + logf(t));
    }
}

}  // namespace mlxd

struct mlxd_linear {
    QMat W;
    void *ws = nullptr;   // generic-path workspace
    size_t ws_bytes = 0;
};

// ---------------------------------------------------------------- helpers

namespace {

struct TensorSet {
    std::unordered_map<std::string, const mlxd_tensor *> by_name;
    const mlxd_tensor *get(const std::string &n) const {
        auto it = by_name.find(n);
        return it == by_name.end() ? nullptr : it->second;
    }
};

size_t tensor_elems(const mlxd_tensor *t) {
    size_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= (size_t)t->shape[i];
    return n;
}
size_t dt_size(int dt) { return dt == MLXD_BF16 ? 2 : 4; }

// weights_get_triplet (weights.c:1053-1088): {base}.weight + optional
// scales/biases; a partial triplet is an error.
struct Triplet {
    const mlxd_tensor *w = nullptr, *s = nullptr, *b = nullptr;
    bool quant = false;
    int rows = 0, cols = 0;
};

int get_triplet(const TensorSet &ts, const std::string &base, int group, Triplet &out) {
    out = Triplet{};
    out.w = ts.get(base + ".weight");
    out.s = ts.get(base + ".scales");
    out.b = ts.get(base + ".biases");
    if (!out.w) {
        set_error("missing tensor %s.weight", base.c_str());
        return -1;
    }
    if ((out.s == nullptr) != (out.b == nullptr)) {
        set_error("partial quantized triplet %s", base.c_str());
        return -1;
    }
    if (out.w->ndim != 2) {
        set_error("%s.weight must be 2-D", base.c_str());
        return -1;
    }
    out.quant = out.s != nullptr;
    out.rows = (int)out.w->shape[0];
    if (out.quant) {
        if (out.w->dtype != MLXD_U32) {
            set_error("%s.weight: quantized weight must be U32", base.c_str());
            return -1;
        }
        out.cols = (int)out.w->shape[1] * 8;
        if (out.s->dtype != out.b->dtype || (out.s->dtype != MLXD_BF16 && out.s->dtype != MLXD_F32) ||
            out.s->ndim != 2 || out.b->ndim != 2 || out.s->shape[0] != out.rows ||
            out.s->shape[1] * group != out.cols || out.b->shape[0] != out.rows || out.b->shape[1] != out.s->shape[1]) {
            set_error("%s: scales/biases shape or dtype mismatch", base.c_str());
            return -1;
        }
    } else {
        if (out.w->dtype != MLXD_BF16) {
            set_error("%s.weight: dense weight must be BF16", base.c_str());
            return -1;
        }
        out.cols = (int)out.w->shape[1];
    }
    return 0;
}

// one source block of rows [r0, r0+nr) x cols [c0, c0+ncols of the matrix)
// into a matrix: at destination rows dst_row0.. (il = 0), or as the gate
// (il = 1) / up (il = 2) rows of a fused gate|up matrix (64-row blocks of
// gate and up alternate)
struct Piece {
    Triplet t;
    int r0, nr, c0;
    int dst_row0;
    int il;
};

int copy_rows(void *dst, size_t dst_pitch, const void *src, size_t src_pitch, size_t width, int rows,
              cudaStream_t st) {
    MLXD_CHECK(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width, rows, cudaMemcpyDefault, st));
    return 0;
}

int place_piece(QMat &M, const Piece &p, cudaStream_t st) {
    const int G = M.group;
    const int ng = M.quant ? M.cols / G : 0, sng = M.quant ? p.t.cols / G : 0;
    const size_t es = M.quant ? dt_size(M.sdtype) : 2;
    auto copy_block = [&](int src_row, int dst_row, int n) -> int {
        if (M.quant) {
            if (copy_rows(M.w + (size_t)dst_row * (M.cols / 8), (size_t)M.cols / 2,
                          (const uint32_t *)p.t.w->data + (size_t)src_row * (p.t.cols / 8) + p.c0 / 8,
                          (size_t)p.t.cols / 2, (size_t)M.cols / 2, n, st) ||
                copy_rows((char *)M.s + (size_t)dst_row * ng * es, ng * es,
                          (const char *)p.t.s->data + ((size_t)src_row * sng + p.c0 / G) * es, sng * es, ng * es, n,
                          st) ||
                copy_rows((char *)M.b + (size_t)dst_row * ng * es, ng * es,
                          (const char *)p.t.b->data + ((size_t)src_row * sng + p.c0 / G) * es, sng * es, ng * es, n,
                          st))
                return -1;
        } else {
            if (copy_rows(M.dense + (size_t)dst_row * M.cols, (size_t)M.cols * 2,
                          (const uint16_t *)p.t.w->data + (size_t)src_row * p.t.cols + p.c0, (size_t)p.t.cols * 2,
                          (size_t)M.cols * 2, n, st))
                return -1;
        }
        return 0;
    };
    if (p.il == 0) return copy_block(p.r0, p.dst_row0, p.nr);
    if (p.nr % 64) {
        set_error("gate/up shard of %d rows is not a multiple of 64", p.nr);
        return -1;
    }
    for (int c = 0; c < p.nr / 64; c++)
        if (copy_block(p.r0 + 64 * c, 128 * c + (p.il == 2 ? 64 : 0), 64)) return -1;
    return 0;
}

int build_qmat(QMat &M, int rows, int cols, int group, const std::vector<Piece> &pcs, bool gateup,
               cudaStream_t st) {
    M.rows = rows;
    M.cols = cols;
    M.group = group;
    M.quant = pcs[0].t.quant;
    for (auto &p : pcs)
        if (p.t.quant != M.quant) {
            set_error("mixed quantized and dense projections in one fused matrix");
            return -1;
        }
    if (M.quant) {
        M.sdtype = pcs[0].t.s->dtype;
        for (auto &p : pcs)
            if (p.t.s->dtype != M.sdtype) {
                set_error("mixed scale dtypes in one fused matrix");
                return -1;
            }
        if (cols % group || cols % 8) {
            set_error("projection %dx%d does not split into groups of %d", rows, cols, group);
            return -1;
        }
        M.w = (uint32_t *)dev_alloc(M.w_bytes());
        M.s = dev_alloc(M.sb_bytes() / 2);
        M.b = dev_alloc(M.sb_bytes() / 2);
        if (!M.w || !M.s || !M.b) return -1;
    } else {
        M.dense = (uint16_t *)dev_alloc(M.w_bytes());
        if (!M.dense) return -1;
    }
    for (auto &p : pcs)
        if (place_piece(M, p, st)) return -1;
    return build_decode_layout(M, gateup, st);
}

void free_qmat(QMat &M) {
    dev_free(M.w);
    dev_free(M.s);
    dev_free(M.b);
    dev_free(M.ti8);
    dev_free(M.sbi);
    dev_free(M.dense);
    M = QMat{};
}

uint16_t *upload_vec(TensorSet &ts, const std::string &name, int n, cudaStream_t st) {
    const mlxd_tensor *t = ts.get(name);
    if (!t || t->dtype != MLXD_BF16 || (int)tensor_elems(t) != n) {
        set_error("missing or bad tensor %s", name.c_str());
        return nullptr;
    }
    uint16_t *p = (uint16_t *)dev_alloc((size_t)n * 2);
    if (!p) return nullptr;
    if (cudaMemcpyAsync(p, t->data, (size_t)n * 2, cudaMemcpyDefault, st) != cudaSuccess) {
        set_error("upload of %s failed", name.c_str());
        return nullptr;
    }
    return p;
}

// fwd_rope_llama3_freqs (forward.c:323-358)
int llama3_freqs(const mlxd_model_config &c, std::vector<float> &out) {
    if (c.head_dim < 2 || (c.head_dim & 1) || c.rope_factor <= 0 || c.rope_orig_max <= 0 ||
        c.rope_lo <= 0 || c.rope_hi <= c.rope_lo) {
        set_error("invalid llama3 rope parameters");
        return -1;
    }
    double base = c.rope_theta, f = c.rope_factor, lf = c.rope_lo, hf = c.rope_hi, old = c.rope_orig_max;
    double low_wl = old / lf, high_wl = old / hf;
    out.resize(c.head_dim / 2);
    for (int i = 0; i < c.head_dim / 2; i++) {
        double fr = pow(base, 2.0 * i / (double)c.head_dim);
        double wl = 2.0 * M_PI * fr;
        if (wl > low_wl) fr = fr * f;
        else if (wl > high_wl) {
            double sm = (old / wl - lf) / (hf - lf);
            fr = fr / ((1.0 - sm) / f + sm);
        }
        out[i] = (float)fr;
    }
    return 0;
}

// the one-kernel-per-op decode step serves head dims 64/128 with 1, 2, 4
// or 8 query heads per kv head; other models decode through the generic
// forward (one position)
bool fast_decode_ok(const mlxd_model *m) {
    return attention_decode_supported(m->c.head_dim, m->hq / m->hkv, m->c.rope_dims);
}

ncclComm_t comm_of(mlxd_model *m) { return (ncclComm_t)m->nccl; }

// the row-parallel projection's f64 partials summed over the ranks (in
// place), then h_out = bf16(h_in + bf16(sum)): the sum of exact partials of
// the group-exact arithmetic, so the result equals one GPU's bit for bit
int reduce_partials(mlxd_model *m, double *part, size_t n, uint16_t *h_out, const uint16_t *h_in, cudaStream_t st) {
    ncclResult_t r = ncclAllReduce(part, part, n, ncclFloat64, ncclSum, comm_of(m), st);
    if (r != ncclSuccess) {
        set_error("ncclAllReduce: %s", ncclGetErrorString(r));
        return -1;
    }
    return add_partials(h_out, h_in, part, 1, n, n, st);
}

size_t proj_ws_bytes(const mlxd_model *m, int S) {
    size_t b = 0;
    auto need = [&](const QMat &W) {
        size_t x = qgemm_tc_eligible(W, S, EPI_STORE) ? qgemm_tc_ws_bytes(S, W.cols) : generic_ws_bytes(W, S, PRO_PLAIN);
        if (x > b) b = x;
    };
    for (auto &L : m->L) {
        need(L.qkv);
        need(L.o);
        need(L.gateup);
        need(L.down);
    }
    need(m->lm);
    return b;
}

int ensure_prefill(mlxd_model *m, int S) {
    if (S <= m->pre_cap) return 0;
    dev_free(m->p_h); dev_free(m->p_x); dev_free(m->p_qkv); dev_free(m->p_q);
    dev_free(m->p_att); dev_free(m->p_act); dev_free(m->p_tmp); dev_free(m->p_ids);
    dev_free(m->p_part); dev_free(m->p_ws);
    m->p_h = m->p_x = m->p_qkv = m->p_q = m->p_att = m->p_act = m->p_tmp = nullptr;
    m->p_ids = nullptr;
    m->p_part = nullptr;
    m->p_ws = nullptr;
    m->pre_cap = 0;
    const mlxd_model_config &c = m->c;
    int D = c.head_dim;
    size_t qkvw = (size_t)m->qdim + 2 * (size_t)m->hkv * D;
    m->p_h = (uint16_t *)dev_alloc((size_t)S * c.hidden * 2);
    m->p_x = (uint16_t *)dev_alloc((size_t)S * c.hidden * 2);
    m->p_qkv = (uint16_t *)dev_alloc((size_t)S * qkvw * 2);
    m->p_q = (uint16_t *)dev_alloc((size_t)S * m->hq * D * 2);
    m->p_att = (uint16_t *)dev_alloc((size_t)S * m->hq * D * 2);
    m->p_act = (uint16_t *)dev_alloc((size_t)S * m->inter_local * 2);
    m->p_tmp = (uint16_t *)dev_alloc((size_t)S * c.hidden * 2);
    m->p_ids = (int32_t *)dev_alloc((size_t)S * 4);
    m->p_part = c.tp_size > 1 ? (double *)dev_alloc((size_t)S * c.hidden * 8) : nullptr;
    m->p_ws_bytes = proj_ws_bytes(m, S);
    m->p_ws = dev_alloc(m->p_ws_bytes);
    if (!m->p_h || !m->p_x || !m->p_qkv || !m->p_q || !m->p_att || !m->p_act || !m->p_tmp || !m->p_ids ||
        (c.tp_size > 1 && !m->p_part) || !m->p_ws)
        return -1;
    m->pre_cap = S;
    return 0;
}

int ensure_attn_scratch(mlxd_model *m, int S, int pos0, int window) {
    const size_t need = attention_prefill_scratch(S, pos0, window, m->hq, m->c.head_dim);
    if (need <= m->p_scr_floats) return 0;
    dev_free(m->p_scr);
    m->p_scr = (float *)dev_alloc(need * 4);
    m->p_scr_floats = m->p_scr ? need : 0;
    return m->p_scr ? 0 : -1;
}

// y[S] = W x[S] with the epilogue; S == 1 on the decode kernels
int linear_any(mlxd_model *m, const QMat &W, const uint16_t *x, int S, int epi, uint16_t *y, const uint16_t *res,
               double *yf, cudaStream_t st) {
    GemvArgs a = {};
    a.x = x;
    a.y = y;
    a.yf = yf;
    a.residual = res;
    if (S == 1) {
        a.gws = m->gws;
        a.gws_bytes = m->gws_bytes;
        return qgemv(W, PRO_PLAIN, epi, a, st, false);
    }
    if (qgemm_tc_eligible(W, S, epi)) return qgemm_tc(W, x, S, epi, res, y, yf, m->p_ws, m->p_ws_bytes, st);
    return qgemm_generic(W, PRO_PLAIN, epi, a, S, m->p_ws, m->p_ws_bytes, st);
}

}  // namespace

// ------------------------------------------------------------------ forward

namespace mlxd {

// one token through every layer with the fused decode kernels
// a row-parallel projection whose decode GEMV sends its rows' exchange lines
// itself (decode layout); others go through tp_sum's f64 partials
static bool tp_fused(const QMat &W) { return W.ti8 && W.sbi && W.fast(); }

static int decode_step(mlxd_model *m, mlxd_kv *kv, const int32_t *ids_dev, bool want_logits,
                       uint16_t *logits_out, bool argmax, cudaStream_t st, bool pdl) {
    const mlxd_model_config &c = m->c;
    int H = c.hidden, D = c.head_dim;
    bool tp = c.tp_size > 1;
    if (embed_rows(m->embed, H, c.qgroup, c.vocab, ids_dev, 1, m->h, st)) return -1;
    size_t layer_elems = (size_t)kv->hkv * kv->cap * D;
    for (int l = 0; l < c.layers; l++) {
        Layer &L = m->L[l];
        GemvArgs a = {};
        a.gws = m->gws;
        a.gws_bytes = m->gws_bytes;
        a.x = m->h;
        a.norm_w = L.ln1;
        a.eps = c.eps;
        a.y = m->qkv;
        if (qgemv(L.qkv, PRO_RMSNORM, EPI_STORE, a, st, pdl)) return -1;
        AttnDecodeArgs ad = {};
        ad.qkv = m->qkv;
        ad.qdim = m->qdim;
        ad.gate = c.attn_gate;
        ad.qn = c.qk_norm ? L.qn : nullptr;
        ad.kn = c.qk_norm ? L.kn : nullptr;
        ad.eps = c.eps;
        ad.rope = RopeArgs{D, c.rope_dims, m->rope_cs};
        ad.kc = kv->k + (size_t)l * layer_elems;
        ad.vc = kv->v + (size_t)l * layer_elems;
        ad.cap = kv->cap;
        ad.window = kv->window;
        ad.d_pos = kv->d_pos;
        ad.hq = m->hq;
        ad.hkv = m->hkv;
        ad.out = m->att;
        if (kv->att_rep != m->hq / m->hkv || kv->d != D) {
            set_error("KV cache made for another model shape");
            return -1;
        }
        {
            const size_t per = (size_t)kv->hkv * kv->att_nbmax * kv->att_rep;
            ad.part_o = kv->att_part;
            ad.part_l = kv->att_part + per * D;
            ad.part_m = ad.part_l + per;
            ad.cnt = kv->att_cnt;
            ad.nbmax = kv->att_nbmax;
        }
        if (attention_decode(ad, st, pdl)) return -1;
        GemvArgs o = {};
        // the o projection runs on the SMs that attention leaves free (one
        // attention CTA per SM), its CTAs resident with their weights loaded
        // while attention runs, instead of a third of them starting cold after it
        if (pdl) {
            const int att_sms = attention_decode_sms(ad), sms = num_sms();
            if (att_sms > 0 && sms - att_sms >= sms / 4) o.grid_cap = sms - att_sms;
        }
        o.gws = m->gws;
        o.gws_bytes = m->gws_bytes;
        o.x = m->att;
        if (tp && tp_fused(L.o)) {
            // the GEMV's epilogue sends its rows; the exchange kernel receives
            if (tp_send_args(m, 2 * l, o) || qgemv(L.o, PRO_PLAIN, EPI_PARTIAL, o, st, pdl) ||
                tp_recv(m, m->h, m->h1, 2 * l, st, pdl))
                return -1;
        } else if (tp) {
            o.yf = m->part_h;
            if (qgemv(L.o, PRO_PLAIN, EPI_PARTIAL, o, st, pdl)) return -1;
            if (tp_sum(m, m->part_h, m->h, m->h1, 2 * l, st, pdl)) return -1;
        } else {
            o.y = m->h1;
            o.residual = m->h;
            o.res_early = 1;   // written by the previous layer's down GEMV (or the embedding)
            if (qgemv(L.o, PRO_PLAIN, EPI_RESIDUAL, o, st, pdl)) return -1;
        }
        GemvArgs gu = {};
        gu.gws = m->gws;
        gu.gws_bytes = m->gws_bytes;
        gu.x = m->h1;
        gu.norm_w = L.ln2;
        gu.eps = c.eps;
        gu.y = m->act;
        if (qgemv(L.gateup, PRO_RMSNORM, EPI_SWIGLU, gu, st, pdl)) return -1;
        GemvArgs dn = {};
        dn.gws = m->gws;
        dn.gws_bytes = m->gws_bytes;
        dn.x = m->act;
        if (tp && tp_fused(L.down)) {
            if (tp_send_args(m, 2 * l + 1, dn) || qgemv(L.down, PRO_PLAIN, EPI_PARTIAL, dn, st, pdl) ||
                tp_recv(m, m->h1, m->h, 2 * l + 1, st, pdl))
                return -1;
        } else if (tp) {
            dn.yf = m->part_h;
            if (qgemv(L.down, PRO_PLAIN, EPI_PARTIAL, dn, st, pdl)) return -1;
            if (tp_sum(m, m->part_h, m->h1, m->h, 2 * l + 1, st, pdl)) return -1;
        } else {
            dn.y = m->h;
            dn.residual = m->h1;
            dn.res_early = 1;   // written by the o GEMV, two launches back
            if (qgemv(L.down, PRO_PLAIN, EPI_RESIDUAL, dn, st, pdl)) return -1;
        }
    }
    if (want_logits) {
        GemvArgs lg = {};
        lg.gws = m->gws;
        lg.gws_bytes = m->gws_bytes;
        lg.x = m->h;
        lg.norm_w = m->norm;
        lg.eps = c.eps;
        lg.y = logits_out;
        lg.amax = m->amax;
        lg.row_offset = m->vocab_off;
        if (qgemv(m->lm, PRO_RMSNORM, argmax ? EPI_ARGMAX : EPI_STORE, lg, st, pdl)) return -1;
        // greedy over the vocabulary shards: the largest key of all ranks
        if (argmax && tp) return tp_argmax(m, m->amax, kv->d_pos, m->token, st, pdl);
    }
    step_finish_kernel<<<1, 1, 0, st>>>(kv->d_pos, argmax ? m->amax : nullptr, m->token, tp ? tp_seq(m) : nullptr);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

// S tokens through the generic kernels (prefill chunks; models the decode
// kernels do not serve)
static int generic_forward(mlxd_model *m, mlxd_kv *kv, const int32_t *ids_dev, int S, bool want_logits,
                           uint16_t *logits_out, cudaStream_t st) {
    const mlxd_model_config &c = m->c;
    int H = c.hidden, D = c.head_dim;
    bool tp = c.tp_size > 1;
    if (ensure_prefill(m, S)) return -1;
    int pos0 = kv->offset;
    if (ensure_attn_scratch(m, S, pos0, kv->window)) return -1;
    if (embed_rows(m->embed, H, c.qgroup, c.vocab, ids_dev, S, m->p_h, st)) return -1;
    size_t layer_elems = (size_t)kv->hkv * kv->cap * D;
    for (int l = 0; l < c.layers; l++) {
        Layer &L = m->L[l];
        uint16_t *kc = kv->k + (size_t)l * layer_elems, *vc = kv->v + (size_t)l * layer_elems;
        if (rmsnorm_rows(m->p_h, S, H, L.ln1, c.eps, m->p_x, st)) return -1;
        if (linear_any(m, L.qkv, m->p_x, S, EPI_STORE, m->p_qkv, nullptr, nullptr, st)) return -1;
        if (qk_rope_append(m->p_qkv, S, m->qdim, m->hq, m->hkv, c.attn_gate, c.qk_norm ? L.qn : nullptr,
                           c.qk_norm ? L.kn : nullptr, c.eps, RopeArgs{D, c.rope_dims, m->rope_cs}, pos0,
                           m->p_q, kc, vc, kv->cap, st))
            return -1;
        if (attention_prefill(m->p_q, S, pos0, kc, vc, kv->cap, kv->window, m->hq, m->hkv, D,
                              c.attn_gate ? m->p_qkv : nullptr, m->qdim, m->p_att, m->p_scr, m->p_scr_floats, st))
            return -1;
        if (tp) {
            if (linear_any(m, L.o, m->p_att, S, EPI_PARTIAL, nullptr, nullptr, m->p_part, st)) return -1;
            if (reduce_partials(m, m->p_part, (size_t)S * H, m->p_h, m->p_h, st)) return -1;
        } else if (linear_any(m, L.o, m->p_att, S, EPI_RESIDUAL, m->p_h, m->p_h, nullptr, st)) {
            return -1;
        }
        if (rmsnorm_rows(m->p_h, S, H, L.ln2, c.eps, m->p_x, st)) return -1;
        if (linear_any(m, L.gateup, m->p_x, S, EPI_SWIGLU, m->p_act, nullptr, nullptr, st)) return -1;
        if (tp) {
            if (linear_any(m, L.down, m->p_act, S, EPI_PARTIAL, nullptr, nullptr, m->p_part, st)) return -1;
            if (reduce_partials(m, m->p_part, (size_t)S * H, m->p_h, m->p_h, st)) return -1;
        } else if (linear_any(m, L.down, m->p_act, S, EPI_RESIDUAL, m->p_h, m->p_h, nullptr, st)) {
            return -1;
        }
    }
    if (want_logits) {
        const uint16_t *last = m->p_h + (size_t)(S - 1) * H;
        if (rmsnorm_rows(last, 1, H, m->norm, c.eps, m->p_x, st)) return -1;
        if (linear_any(m, m->lm, m->p_x, 1, EPI_STORE, logits_out, nullptr, nullptr, st)) return -1;
    }
    set_pos_kernel<<<1, 1, 0, st>>>(kv->d_pos, pos0 + S);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

static int check_room(const mlxd_model *m, const mlxd_kv *kv, int n) {
    if (kv->offset + n > m->rope_positions) {
        set_error("position %d beyond the %d positions of this model's RoPE table", kv->offset + n,
                  m->rope_positions);
        return -1;
    }
    if (kv->window <= 0 && kv->offset + n > kv->cap) {
        set_error("KV cache full: %d + %d > capacity %d", kv->offset, n, kv->cap);
        return -1;
    }
    if (kv->window > 0 && n > kv->cap - kv->window + 1) {
        set_error("chunk of %d tokens does not fit the ring (capacity %d, window %d)", n, kv->cap,
                  kv->window);
        return -1;
    }
    return 0;
}

static int forward_dev(mlxd_model *m, mlxd_kv *kv, const int32_t *ids_dev, int n, bool want_logits,
                       uint16_t *logits_out, cudaStream_t st) {
    if (check_room(m, kv, n)) return -1;
    int rc;
    if (n == 1 && fast_decode_ok(m))
        rc = decode_step(m, kv, ids_dev, want_logits, logits_out, false, st, false);
    else
        rc = generic_forward(m, kv, ids_dev, n, want_logits, logits_out, st);
    if (rc) return -1;
    kv->offset += n;
    return 0;
}

}  // namespace mlxd

// ------------------------------------------------------------------ C ABI

extern "C" {

int mlxd_cuda_tp_plan(const mlxd_model_config *cfg, int rank, int size, int *r) {
    if (!cfg || !r || size < 1 || rank < 0 || rank >= size) {
        set_error("tp_plan: bad arguments");
        return -1;
    }
    const mlxd_model_config &c = *cfg;
    if (c.n_heads % size || c.n_kv_heads % size || c.inter % size || c.vocab % size) {
        set_error("tensor-parallel degree %d does not divide heads/intermediate/vocab", size);
        return -1;
    }
    const int D = c.head_dim, H = c.hidden;
    const int ql = c.n_heads / size * D * (c.attn_gate ? 2 : 1), kl = c.n_kv_heads / size * D;
    const int oc = c.n_heads / size * D, il = c.inter / size, vl = c.vocab / size;
    const int plan[8][4] = {{rank * ql, ql, 0, H},     {rank * kl, kl, 0, H},     {rank * kl, kl, 0, H},
                            {0, H, rank * oc, oc},     {rank * il, il, 0, H},     {rank * il, il, 0, H},
                            {0, H, rank * il, il},     {rank * vl, vl, 0, H}};
    for (int i = 0; i < 8; i++)
        for (int j = 0; j < 4; j++) r[4 * i + j] = plan[i][j];
    return 0;
}

int mlxd_cuda_model_create(mlxd_model **out, const mlxd_model_config *cfg, const mlxd_tensor *tensors,
                           int n_tensors) {
    if (!out || !cfg || (!tensors && n_tensors)) {
        set_error("model_create: null argument");
        return -1;
    }
    const mlxd_model_config &c = *cfg;
    int tp = c.tp_size > 0 ? c.tp_size : 1, rank = c.tp_size > 0 ? c.tp_rank : 0;
    if (c.family < MLXD_QWEN3 || c.family > MLXD_QWEN3_5) {
        set_error("unsupported model family %d", c.family);
        return -1;
    }
    if (c.hidden <= 0 || c.layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
        c.vocab <= 0 || c.inter <= 0 || c.n_heads % c.n_kv_heads) {
        set_error("invalid model dimensions");
        return -1;
    }
    if (c.qbits != 0 && c.qbits != 4) {
        set_error("only 4-bit affine quantisation is supported (bits=%d)", c.qbits);
        return -1;
    }
    if (c.qbits == 4 && c.qgroup != 32 && c.qgroup != 64) {
        set_error("quantisation group %d not supported (32 or 64)", c.qgroup);
        return -1;
    }
    int plan[8][4];   // this rank's rows/columns of q, k, v, o, gate, up, down, lm_head
    if (mlxd_cuda_tp_plan(&c, rank, tp, &plan[0][0])) return -1;
    if (c.rope_dims <= 0 || c.rope_dims > c.head_dim || (c.rope_dims & 1)) {
        set_error("invalid rope dims %d", c.rope_dims);
        return -1;
    }
    if ((c.inter / tp) % 64) {
        set_error("intermediate shard %d is not a multiple of 64", c.inter / tp);
        return -1;
    }
    mlxd_model *m = new mlxd_model();
    m->c = c;
    m->c.tp_size = tp;
    m->c.tp_rank = rank;
    int G = c.qbits ? c.qgroup : 64;
    int D = c.head_dim;
    m->hq = c.n_heads / tp;
    m->hkv = c.n_kv_heads / tp;
    m->qdim = m->hq * D * (c.attn_gate ? 2 : 1);
    m->inter_local = c.inter / tp;
    m->vocab_local = c.vocab / tp;
    m->vocab_off = rank * m->vocab_local;
    cudaStream_t st = nullptr;
    TensorSet ts;
    for (int i = 0; i < n_tensors; i++) ts.by_name[tensors[i].name] = &tensors[i];
    auto fail = [&]() {
        cudaDeviceSynchronize();
        mlxd_cuda_model_destroy(m);
        return -1;
    };
    m->L.resize(c.layers);
    int qrows_full = c.n_heads * D * (c.attn_gate ? 2 : 1);
    int kvrows_full = c.n_kv_heads * D;
    for (int l = 0; l < c.layers; l++) {
        Layer &L = m->L[l];
        std::string p = "model.layers." + std::to_string(l) + ".";
        Triplet q, k, v, o, gt, up, dn;
        if (get_triplet(ts, p + "self_attn.q_proj", G, q) || get_triplet(ts, p + "self_attn.k_proj", G, k) ||
            get_triplet(ts, p + "self_attn.v_proj", G, v) || get_triplet(ts, p + "self_attn.o_proj", G, o) ||
            get_triplet(ts, p + "mlp.gate_proj", G, gt) || get_triplet(ts, p + "mlp.up_proj", G, up) ||
            get_triplet(ts, p + "mlp.down_proj", G, dn))
            return fail();
        if (q.rows != qrows_full || q.cols != c.hidden || k.rows != kvrows_full || v.rows != kvrows_full ||
            k.cols != c.hidden || v.cols != c.hidden || o.rows != c.hidden || o.cols != c.n_heads * D ||
            gt.rows != c.inter || up.rows != c.inter || gt.cols != c.hidden || up.cols != c.hidden ||
            dn.rows != c.hidden || dn.cols != c.inter) {
            set_error("layer %d: projection shapes do not match the config", l);
            return fail();
        }
        const int ql = plan[0][1], kl = plan[1][1];
        // fused q|k|v rows (column-parallel slice by heads)
        if (build_qmat(L.qkv, ql + 2 * kl, c.hidden, G,
                       {{q, plan[0][0], ql, 0, 0, 0}, {k, plan[1][0], kl, 0, ql, 0}, {v, plan[2][0], kl, 0, ql + kl, 0}},
                       false, st))
            return fail();
        // o: row-parallel (input columns of this rank's heads)
        if (build_qmat(L.o, c.hidden, plan[3][3], G, {{o, 0, c.hidden, plan[3][2], 0, 0}}, false, st)) return fail();
        // gate/up: alternating 64-row blocks
        const int il = plan[4][1];
        if (build_qmat(L.gateup, 2 * il, c.hidden, G, {{gt, plan[4][0], il, 0, 0, 1}, {up, plan[5][0], il, 0, 0, 2}},
                       true, st))
            return fail();
        if (build_qmat(L.down, c.hidden, plan[6][3], G, {{dn, 0, c.hidden, plan[6][2], 0, 0}}, false, st))
            return fail();
        if (!(L.ln1 = upload_vec(ts, p + "input_layernorm.weight", c.hidden, st))) return fail();
        if (!(L.ln2 = upload_vec(ts, p + "post_attention_layernorm.weight", c.hidden, st))) return fail();
        if (c.qk_norm) {
            if (!(L.qn = upload_vec(ts, p + "self_attn.q_norm.weight", D, st))) return fail();
            if (!(L.kn = upload_vec(ts, p + "self_attn.k_norm.weight", D, st))) return fail();
        }
    }
    // embedding (replicated, MLX format) and lm_head (vocab-parallel)
    Triplet emb;
    if (get_triplet(ts, "model.embed_tokens", G, emb)) return fail();
    if (emb.rows != c.vocab || emb.cols != c.hidden) {
        set_error("embed_tokens shape does not match the config");
        return fail();
    }
    m->embed.quant = emb.quant;
    if (emb.quant) {
        m->embed.sdtype = emb.s->dtype;
        size_t wb = tensor_elems(emb.w) * 4, sbb = tensor_elems(emb.s) * dt_size(emb.s->dtype);
        m->embed.w = (uint32_t *)dev_alloc(wb);
        m->embed.s = dev_alloc(sbb);
        m->embed.b = dev_alloc(sbb);
        if (!m->embed.w || !m->embed.s || !m->embed.b) return fail();
        if (!cuda_ok(cudaMemcpyAsync(m->embed.w, emb.w->data, wb, cudaMemcpyDefault, st), "embed upload") ||
            !cuda_ok(cudaMemcpyAsync(m->embed.s, emb.s->data, sbb, cudaMemcpyDefault, st), "embed upload") ||
            !cuda_ok(cudaMemcpyAsync(m->embed.b, emb.b->data, sbb, cudaMemcpyDefault, st), "embed upload"))
            return fail();
    } else {
        size_t b = tensor_elems(emb.w) * 2;
        m->embed.dense = (uint16_t *)dev_alloc(b);
        if (!m->embed.dense) return fail();
        if (!cuda_ok(cudaMemcpyAsync(m->embed.dense, emb.w->data, b, cudaMemcpyDefault, st), "embed upload"))
            return fail();
    }
    Triplet lm;
    if (c.tie) lm = emb;
    else if (get_triplet(ts, "lm_head", G, lm)) return fail();
    if (lm.rows != c.vocab || lm.cols != c.hidden) {
        set_error("lm_head shape does not match the config");
        return fail();
    }
    if (build_qmat(m->lm, plan[7][1], c.hidden, G, {{lm, plan[7][0], plan[7][1], 0, 0, 0}}, false, st)) return fail();
    if (!(m->norm = upload_vec(ts, "model.norm.weight", c.hidden, st))) return fail();

    // RoPE cos/sin table, computed exactly as mlx_fast_rope's angle
    // (inv_freq = 2^(-(i/half)*log2(theta)) or 1/freqs[i]; angle = pos*inv)
    {
        std::vector<float> fr;
        if (c.rope_llama3 && llama3_freqs(c, fr)) return fail();
        int half = c.rope_dims / 2;
        int npos = c.max_pos > 0 ? c.max_pos : 4096;
        if (npos > (1 << 20)) npos = 1 << 20;
        std::vector<float> cs((size_t)npos * half * 2);
        float lb = log2f(c.rope_theta);
        std::vector<float> inv(half);
        for (int i = 0; i < half; i++)
            inv[i] = c.rope_llama3 ? 1.0f / fr[i] : exp2f(-((float)i / (float)half) * lb);
        for (int p = 0; p < npos; p++) {
            float Lp = (float)p;
            for (int i = 0; i < half; i++) {
                float th = Lp * inv[i];
                cs[((size_t)p * half + i) * 2] = cosf(th);
                cs[((size_t)p * half + i) * 2 + 1] = sinf(th);
            }
        }
        m->rope_cs = (float *)dev_alloc(cs.size() * 4);
        if (!m->rope_cs) return fail();
        if (!cuda_ok(cudaMemcpy(m->rope_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope upload"))
            return fail();
        m->rope_positions = npos;
    }

    // decode scratch
    {
        size_t g = 0;
        auto need = [&](const QMat &W) {
            if (W.ti8) return;
            size_t x = generic_ws_bytes(W, 1, PRO_RMSNORM);
            if (x > g) g = x;
        };
        for (auto &L : m->L) {
            need(L.qkv);
            need(L.o);
            need(L.gateup);
            need(L.down);
        }
        need(m->lm);
        m->gws_bytes = g ? g : 256;
        m->gws = dev_alloc(m->gws_bytes);
        if (!m->gws) return fail();
    }
    size_t qkvw = (size_t)m->qdim + 2 * (size_t)m->hkv * D;
    m->h = (uint16_t *)dev_alloc((size_t)c.hidden * 2);
    m->h1 = (uint16_t *)dev_alloc((size_t)c.hidden * 2);
    m->qkv = (uint16_t *)dev_alloc(qkvw * 2);
    m->att = (uint16_t *)dev_alloc((size_t)m->hq * D * 2);
    m->act = (uint16_t *)dev_alloc((size_t)m->inter_local * 2);
    m->logits = (uint16_t *)dev_alloc((size_t)m->vocab_local * 2);
    m->amax = (unsigned long long *)dev_alloc(8);
    m->token = (int32_t *)dev_alloc(4);
    m->part_h = (double *)dev_alloc((size_t)c.hidden * 8 * tp);
    m->lp = (float *)dev_alloc(4);
    if (!m->lp || !m->h || !m->h1 || !m->qkv || !m->att || !m->act || !m->logits || !m->amax || !m->token ||
        !m->part_h)
        return fail();
    if (!cuda_ok(cudaMemset(m->amax, 0, 8), "memset")) return fail();
    if (!(m->samp = samp_work_create(c.vocab))) return fail();   // full rows (gathered under TP)
    if (!cuda_ok(cudaDeviceSynchronize(), "model upload")) return fail();
    for (auto &L : m->L)
        m->weight_bytes += L.qkv.stream_bytes() + L.o.stream_bytes() + L.gateup.stream_bytes() + L.down.stream_bytes();
    m->weight_bytes += m->lm.stream_bytes();
    *out = m;
    return 0;
}

void mlxd_cuda_model_destroy(mlxd_model *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    if (m->graph_exec) cudaGraphExecDestroy((cudaGraphExec_t)m->graph_exec);
    for (auto &L : m->L) {
        free_qmat(L.qkv);
        free_qmat(L.o);
        free_qmat(L.gateup);
        free_qmat(L.down);
        dev_free(L.ln1);
        dev_free(L.ln2);
        dev_free(L.qn);
        dev_free(L.kn);
    }
    free_qmat(m->lm);
    dev_free(m->embed.w);
    dev_free(m->embed.s);
    dev_free(m->embed.b);
    dev_free(m->embed.dense);
    dev_free(m->norm);
    dev_free(m->rope_cs);
    for (void *p : {(void *)m->h, (void *)m->h1, (void *)m->qkv, (void *)m->att, (void *)m->act,
                    (void *)m->logits, (void *)m->amax, (void *)m->token, (void *)m->part_h, (void *)m->p_h,
                    (void *)m->p_x, (void *)m->p_qkv, (void *)m->p_q, (void *)m->p_att, (void *)m->p_act,
                    (void *)m->p_tmp, (void *)m->p_ids, (void *)m->p_part, (void *)m->p_ws, (void *)m->p_scr,
                    (void *)m->ctx, (void *)m->n_ctx, (void *)m->d_step, (void *)m->lp, (void *)m->gws})
        dev_free(p);
    samp_work_destroy(m->samp);
    tp_free(m);
    if (m->stream) cudaStreamDestroy(m->stream);
    if (m->nccl) ncclCommDestroy((ncclComm_t)m->nccl);
    delete m;
}

size_t mlxd_cuda_model_weight_bytes(const mlxd_model *m) { return m ? m->weight_bytes : 0; }

int mlxd_cuda_nccl_unique_id(void *out128) {
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) {
        set_error("ncclGetUniqueId: %s", ncclGetErrorString(r));
        return -1;
    }
    memcpy(out128, &id, sizeof(id));
    return 0;
}

int mlxd_cuda_model_tp_init(mlxd_model *m, const void *uid) {
    if (!m || !uid) return -1;
    if (m->c.tp_size <= 1) return 0;
    ncclUniqueId id;
    memcpy(&id, uid, sizeof(id));
    ncclComm_t comm;
    ncclResult_t r = ncclCommInitRank(&comm, m->c.tp_size, id, m->c.tp_rank);
    if (r != ncclSuccess) {
        set_error("ncclCommInitRank: %s", ncclGetErrorString(r));
        return -1;
    }
    m->nccl = comm;
    return tp_setup(m);
}

int mlxd_cuda_kv_create(mlxd_kv **out, const mlxd_model *m, int capacity) {
    if (!out || !m || capacity <= 0) {
        set_error("kv_create: bad arguments");
        return -1;
    }
    static std::atomic<unsigned long long> kv_serial{0};
    mlxd_kv *kv = new mlxd_kv();
    kv->serial = ++kv_serial;
    kv->layers = m->c.layers;
    kv->hkv = m->hkv;
    kv->d = m->c.head_dim;
    kv->cap = capacity;
    kv->window = m->c.window;
    kv->offset = 0;
    if (kv->window > 0 && capacity < kv->window) {
        set_error("ring capacity %d smaller than the window %d", capacity, kv->window);
        delete kv;
        return -1;
    }
    size_t n = (size_t)kv->layers * kv->hkv * kv->cap * kv->d;
    kv->k = (uint16_t *)dev_alloc(n * 2);
    kv->v = (uint16_t *)dev_alloc(n * 2);
    kv->d_pos = (int32_t *)dev_alloc(4);
    // decode attention's block results: a step attends at most `span`
    // positions, which touch at most span/64 + 2 blocks
    const int span = kv->window > 0 && kv->window < kv->cap ? kv->window : kv->cap;
    kv->att_nbmax = span / 64 + 2;
    kv->att_rep = m->hq / m->hkv;
    const size_t pf = attention_decode_part_floats(kv->att_nbmax, kv->hkv, kv->att_rep, kv->d);
    kv->att_part = (float *)dev_alloc(pf * 4);
    kv->att_cnt = (int *)dev_alloc((size_t)kv->hkv * 4);
    if (!kv->k || !kv->v || !kv->d_pos || !kv->att_part || !kv->att_cnt) {
        mlxd_cuda_kv_destroy(kv);
        return -1;
    }
    if (!cuda_ok(cudaMemset(kv->d_pos, 0, 4), "memset") ||
        !cuda_ok(cudaMemset(kv->att_cnt, 0, (size_t)kv->hkv * 4), "memset")) {
        mlxd_cuda_kv_destroy(kv);
        return -1;
    }
    *out = kv;
    return 0;
}

void mlxd_cuda_kv_destroy(mlxd_kv *kv) {
    if (!kv) return;
    cudaDeviceSynchronize();
    dev_free(kv->k);
    dev_free(kv->v);
    dev_free(kv->d_pos);
    dev_free(kv->att_part);
    dev_free(kv->att_cnt);
    delete kv;
}

int mlxd_cuda_kv_offset(const mlxd_kv *kv, int layer) {
    if (!kv || layer < 0 || layer >= kv->layers) return -1;
    return kv->offset;
}

int mlxd_cuda_kv_capacity(const mlxd_kv *kv, int layer) {
    if (!kv || layer < 0 || layer >= kv->layers) return -1;
    return kv->cap;
}

int mlxd_cuda_kv_reset(mlxd_kv *kv) {
    if (!kv) return -1;
    kv->offset = 0;
    MLXD_CHECK(cudaMemset(kv->d_pos, 0, 4));
    MLXD_CHECK(cudaDeviceSynchronize());
    return 0;
}

// rows [pos, pos + n) of every kv head of one layer, ring-aware, as 2-D
// copies: dev [hkv][n][D] <-> cache slots (pos + i) % cap
static int kv_rows(mlxd_kv *kv, int layer, bool value, int pos, int n, uint16_t *dev, bool to_cache,
                   cudaStream_t st) {
    if (!kv || layer < 0 || layer >= kv->layers || pos < 0 || n < 0 || n > kv->cap || !dev) {
        set_error("kv rows: bad arguments");
        return -1;
    }
    const size_t layer_elems = (size_t)kv->hkv * kv->cap * kv->d, row = (size_t)kv->d * 2;
    uint16_t *base = (value ? kv->v : kv->k) + (size_t)layer * layer_elems;
    for (int part = 0, done = 0; done < n; part++) {
        const int slot = (pos + done) % kv->cap;
        const int len = n - done < kv->cap - slot ? n - done : kv->cap - slot;
        uint16_t *c = base + (size_t)slot * kv->d;
        uint16_t *d = dev + (size_t)done * kv->d;
        // one 2-D copy per contiguous run: hkv rows of len * D elements
        MLXD_CHECK(cudaMemcpy2DAsync(to_cache ? (void *)c : (void *)d, to_cache ? (size_t)kv->cap * row : (size_t)n * row,
                                     to_cache ? (const void *)d : (const void *)c,
                                     to_cache ? (size_t)n * row : (size_t)kv->cap * row, (size_t)len * row,
                                     (size_t)kv->hkv, cudaMemcpyDeviceToDevice, st));
        done += len;
    }
    return 0;
}

int mlxd_cuda_kv_write(mlxd_kv *kv, int layer, int pos, int n, const void *k_dev, const void *v_dev,
                       void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (kv_rows(kv, layer, false, pos, n, (uint16_t *)k_dev, true, st)) return -1;
    return kv_rows(kv, layer, true, pos, n, (uint16_t *)v_dev, true, st);
}

int mlxd_cuda_kv_gather(mlxd_kv *kv, int layer, int is_value, int pos, int n, void *dst_dev, void *stream) {
    return kv_rows(kv, layer, is_value != 0, pos, n, (uint16_t *)dst_dev, false, (cudaStream_t)stream);
}

int mlxd_cuda_kv_set_offset(mlxd_kv *kv, int offset, void *stream) {
    if (!kv || offset < 0 || (kv->window <= 0 && offset > kv->cap)) {
        set_error("kv_set_offset: bad arguments");
        return -1;
    }
    kv->offset = offset;
    set_pos_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(kv->d_pos, offset);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

int mlxd_cuda_step_async(mlxd_model *m, mlxd_kv *kv, const int32_t *tok_in_dev, const mlxd_sampling *sp,
                         const int32_t *ctx_dev, int n_ctx, uint64_t step, int32_t *tok_out_dev, float *logprob_dev,
                         void *stream) {
    if (!m || !kv || !tok_in_dev || !sp || !tok_out_dev) {
        set_error("step_async: bad arguments");
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (ensure_prefill(m, 1) || forward_dev(m, kv, tok_in_dev, 1, true, m->logits, st)) return -1;
    const uint16_t *row = m->logits;
    if (m->tp) {
        if (tp_gather_logits(m, m->logits, st, false)) return -1;
        row = tp_full_logits(m);
    }
    return sample(m->samp, row, MLXD_BF16, m->c.vocab, *sp, ctx_dev, n_ctx, step, tok_out_dev, logprob_dev, nullptr,
                  st);
}

int mlxd_cuda_read_token(const int32_t *tok_dev, int32_t *out, void *stream) {
    if (!tok_dev || !out) {
        set_error("read_token: bad arguments");
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    static thread_local int32_t *pin = nullptr;
    if (!pin) MLXD_CHECK(cudaMallocHost(&pin, 4));
    MLXD_CHECK(cudaMemcpyAsync(pin, tok_dev, 4, cudaMemcpyDeviceToHost, st));
    MLXD_CHECK(cudaStreamSynchronize(st));
    *out = *pin;
    return 0;
}

int mlxd_cuda_kv_read(mlxd_kv *kv, int layer, int is_value, uint16_t *host_out, int *n_out) {
    if (!kv || layer < 0 || layer >= kv->layers || !host_out) return -1;
    MLXD_CHECK(cudaDeviceSynchronize());
    int live = kv->offset < kv->cap ? kv->offset : kv->cap;
    int first = kv->offset - live;
    size_t layer_elems = (size_t)kv->hkv * kv->cap * kv->d;
    const uint16_t *base = (is_value ? kv->v : kv->k) + (size_t)layer * layer_elems;
    for (int h = 0; h < kv->hkv; h++)
        for (int i = 0; i < live; i++) {
            int slot = (first + i) % kv->cap;
            MLXD_CHECK(cudaMemcpy(host_out + ((size_t)h * live + i) * kv->d,
                                  base + ((size_t)h * kv->cap + slot) * kv->d, (size_t)kv->d * 2,
                                  cudaMemcpyDeviceToHost));
        }
    if (n_out) *n_out = live;
    return 0;
}

int mlxd_cuda_forward(mlxd_model *m, mlxd_kv *kv, const int32_t *ids, int n, int ids_on_device,
                      int want_logits, void *logits_dev, void *stream) {
    if (!m || !kv || !ids || n <= 0 || (want_logits && !logits_dev)) {
        set_error("forward: bad arguments");
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (ensure_prefill(m, n)) return -1;
    if (!ids_on_device) {
        for (int i = 0; i < n; i++)
            if (ids[i] < 0 || ids[i] >= m->c.vocab) {
                set_error("token id %d out of range", ids[i]);
                return -1;
            }
    }
    MLXD_CHECK(cudaMemcpyAsync(m->p_ids, ids, (size_t)n * 4,
                               ids_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    if (forward_dev(m, kv, m->p_ids, n, want_logits != 0, (uint16_t *)logits_dev, st)) return -1;
    // tensor parallel: the step waits for its exchanges, so that a peer that
    // never arrived is reported here rather than as wrong numbers
    if (m->tp) {
        if (!cuda_ok(cudaStreamSynchronize(st), "forward")) return -1;
        if (tp_timeouts(m)) {
            set_error("tensor-parallel exchange gave up waiting for a peer GPU");
            return -1;
        }
    }
    return 0;
}

// ---- single ops

int mlxd_cuda_linear_create(mlxd_linear **out, const uint32_t *w, const void *scales, const void *biases,
                            int sdtype, int rows, int cols, int group, int on_device) {
    if (!out || !w || !scales || !biases || rows <= 0 || cols <= 0 || (group != 32 && group != 64) ||
        cols % group || (sdtype != MLXD_BF16 && sdtype != MLXD_F32)) {
        set_error("linear_create: bad arguments");
        return -1;
    }
    mlxd_tensor tw = {"w", MLXD_U32, 2, {rows, cols / 8}, w, on_device};
    mlxd_tensor tsc = {"w.scales", sdtype, 2, {rows, cols / group}, scales, on_device};
    mlxd_tensor tb = {"w.biases", sdtype, 2, {rows, cols / group}, biases, on_device};
    Triplet t;
    t.w = &tw;
    t.s = &tsc;
    t.b = &tb;
    t.quant = true;
    t.rows = rows;
    t.cols = cols;
    mlxd_linear *l = new mlxd_linear();
    if (build_qmat(l->W, rows, cols, group, {{t, 0, rows, 0, 0, 0}}, false, nullptr)) {
        cudaDeviceSynchronize();
        mlxd_cuda_linear_destroy(l);
        return -1;
    }
    l->ws_bytes = generic_ws_bytes(l->W, 1, PRO_PLAIN);
    l->ws = dev_alloc(l->ws_bytes);
    if (!l->ws || !cuda_ok(cudaDeviceSynchronize(), "linear upload")) {
        mlxd_cuda_linear_destroy(l);
        return -1;
    }
    *out = l;
    return 0;
}

void mlxd_cuda_linear_destroy(mlxd_linear *l) {
    if (!l) return;
    cudaDeviceSynchronize();
    free_qmat(l->W);
    dev_free(l->ws);
    delete l;
}

int mlxd_cuda_linear(const mlxd_linear *l, const void *x, int S, void *y, void *stream) {
    if (!l || !x || !y || S <= 0) {
        set_error("linear: bad arguments");
        return -1;
    }
    mlxd_linear *ml = const_cast<mlxd_linear *>(l);
    GemvArgs a = {};
    a.x = (const uint16_t *)x;
    a.y = (uint16_t *)y;
    if (S == 1) {
        a.gws = ml->ws;
        a.gws_bytes = ml->ws_bytes;
        return qgemv(ml->W, PRO_PLAIN, EPI_STORE, a, (cudaStream_t)stream, false);
    }
    const bool tc = qgemm_tc_eligible(ml->W, S, EPI_STORE);
    const size_t need = tc ? qgemm_tc_ws_bytes(S, ml->W.cols) : generic_ws_bytes(ml->W, S, PRO_PLAIN);
    if (need > ml->ws_bytes) {
        MLXD_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
        dev_free(ml->ws);
        ml->ws = dev_alloc(need);
        ml->ws_bytes = ml->ws ? need : 0;
        if (!ml->ws) return -1;
    }
    if (tc)
        return qgemm_tc(ml->W, a.x, S, EPI_STORE, nullptr, a.y, nullptr, ml->ws, ml->ws_bytes, (cudaStream_t)stream);
    return qgemm_generic(ml->W, PRO_PLAIN, EPI_STORE, a, S, ml->ws, ml->ws_bytes, (cudaStream_t)stream);
}

int mlxd_cuda_linear_noalloc(const mlxd_linear *l, const void *x, void *y, void *stream) {
    if (!l || !x || !y) {
        set_error("linear_noalloc: null argument");
        return -1;
    }
    return qgemv_static_scratch(l->W, (const uint16_t *)x, (uint16_t *)y, (cudaStream_t)stream);
}

// pdl: each launch chained to the previous one by programmatic dependent
// launch, as the decode step's graph chains its kernels
static int linear_timed(const mlxd_linear *const *ls, int n, int iters, const void *x, void *y, bool pdl,
                        float *ms_out) {
    if (!ls || n <= 0 || iters <= 0 || !x || !y || !ms_out) return -1;
    cudaStream_t st;
    MLXD_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    int rc = 0;
    auto one = [&](int i) {
        GemvArgs g = {};
        g.x = (const uint16_t *)x;
        g.y = (uint16_t *)y;
        g.gws = ls[i]->ws;
        g.gws_bytes = ls[i]->ws_bytes;
        return qgemv(ls[i]->W, PRO_PLAIN, EPI_STORE, g, st, pdl);
    };
    for (int i = 0; i < n && !rc; i++) rc = one(i);   // warm-up
    cudaEventRecord(a, st);
    for (int it = 0; it < iters && !rc; it++)
        for (int i = 0; i < n && !rc; i++) rc = one(i);
    cudaEventRecord(b, st);
    if (!rc && cuda_ok(cudaEventSynchronize(b), "linear_timed")) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, a, b);
        *ms_out = ms / (float)(iters * n);
    } else {
        rc = -1;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaStreamDestroy(st);
    return rc;
}

int mlxd_cuda_linear_timed(const mlxd_linear *const *ls, int n, int iters, const void *x, void *y,
                           float *ms_out) {
    return linear_timed(ls, n, iters, x, y, false, ms_out);
}

int mlxd_cuda_linear_timed_chained(const mlxd_linear *const *ls, int n, int iters, const void *x, void *y,
                                   float *ms_out) {
    return linear_timed(ls, n, iters, x, y, true, ms_out);
}

int mlxd_cuda_rmsnorm(const void *x, int rows, int n, const void *w, float eps, void *y, void *stream) {
    return rmsnorm_rows((const uint16_t *)x, rows, n, (const uint16_t *)w, eps, (uint16_t *)y,
                        (cudaStream_t)stream);
}

int mlxd_cuda_sample(const void *logits_dev, int dtype, int V, const mlxd_sampling *sp, const int32_t *ctx_dev,
                     int n_ctx, uint64_t step, int32_t *tok_dev, float *logprob_dev, uint8_t *keep_dev,
                     void *stream) {
    if (!sp || V <= 0) {
        set_error("sample: bad arguments");
        return -1;
    }
    // scratch per device for the one-off entry point, sized up as needed
    static std::mutex mu;
    static std::vector<std::pair<int, SampWork *>> works;
    int dev = 0;
    MLXD_CHECK(cudaGetDevice(&dev));
    SampWork *w = nullptr;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (auto &e : works)
            if (e.first == dev) w = e.second;
        if (!w || samp_work_capacity(w) < V) {
            if (w) {
                MLXD_CHECK(cudaDeviceSynchronize());
                samp_work_destroy(w);
                for (auto &e : works)
                    if (e.first == dev) e.second = nullptr;
            }
            w = samp_work_create(V);
            if (!w) return -1;
            bool placed = false;
            for (auto &e : works)
                if (e.first == dev) {
                    e.second = w;
                    placed = true;
                }
            if (!placed) works.push_back({dev, w});
        }
    }
    return sample(w, logits_dev, dtype, V, *sp, ctx_dev, n_ctx, step, tok_dev, logprob_dev, keep_dev,
                  (cudaStream_t)stream);
}

// ---- generate (handle_generate_real, engine.c:360-602)

int mlxd_cuda_generate(mlxd_model *m, mlxd_kv *kv, const int32_t *prompt, int n, int max_new,
                       const mlxd_sampling *sp, int chunk, int32_t *out, float *logprobs, double *timing) {
    return mlxd_cuda_generate_ctl(m, kv, prompt, n, max_new, sp, chunk, out, logprobs, timing, nullptr);
}

int mlxd_cuda_generate_ctl(mlxd_model *m, mlxd_kv *kv, const int32_t *prompt, int n, int max_new,
                           const mlxd_sampling *sp, int chunk, int32_t *out, float *logprobs, double *timing,
                           mlxd_gen_control *ctl) {
    if (ctl) ctl->stopped = 0;
    // poll -> hook -> re-poll at each site (engine.c:406-470): true when a
    // flag ends the request there
    auto flagged = [ctl]() -> bool {
        return (ctl->shutdown && __atomic_load_n(ctl->shutdown, __ATOMIC_ACQUIRE)) ||
               (ctl->cancelled && __atomic_load_n(ctl->cancelled, __ATOMIC_ACQUIRE));
    };
    auto site = [&](auto &&hook) -> bool {
        if (!ctl) return false;
        if (flagged()) return ctl->stopped = 1, true;
        hook();
        if (flagged()) return ctl->stopped = 1, true;
        return false;
    };
    if (!m || !kv || !prompt || !sp || !out) {
        set_error("generate: null argument");
        return -1;
    }
    if (n <= 0 || max_new <= 0) return 0;
    if (n > m->c.max_pos && m->c.max_pos > 0) {
        set_error("prompt token count %d exceeds max_position_embeddings %d", n, m->c.max_pos);
        return -1;
    }
    if (chunk <= 0) chunk = 512;
    for (int i = 0; i < n; i++)
        if (prompt[i] < 0 || prompt[i] >= m->c.vocab) {
            set_error("prompt token id %d out of range", prompt[i]);
            return -1;
        }
    if (m->c.tp_size > 1 && !m->tp) {
        set_error("tensor-parallel model: mlxd_cuda_model_tp_init has not run");
        return -1;
    }
    cudaStream_t st = m->stream;
    if (!st) {
        MLXD_CHECK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        m->stream = st;
    }
    if (mlxd_cuda_kv_reset(kv)) return -1;
    // context list for the repetition penalty (prompt + generated); a
    // captured decode graph holds these buffers, so it goes when they do
    int ctx_cap = n + max_new + 1;
    if (ctx_cap > m->ctx_cap || !m->n_ctx || !m->d_step) {
        if (m->graph_exec) {
            cudaGraphExecDestroy((cudaGraphExec_t)m->graph_exec);
            m->graph_exec = nullptr;
        }
        dev_free(m->ctx);
        m->ctx = (int32_t *)dev_alloc((size_t)ctx_cap * 4);
        if (!m->ctx) {
            m->ctx_cap = 0;
            return -1;
        }
        m->ctx_cap = ctx_cap;
        if (!m->n_ctx) m->n_ctx = (int32_t *)dev_alloc(4);
        if (!m->d_step) m->d_step = (unsigned long long *)dev_alloc(8);
        if (!m->n_ctx || !m->d_step) return -1;
    }
    int32_t *pin = nullptr;
    MLXD_CHECK(cudaMallocHost(&pin, sizeof(int32_t) * (size_t)(n + 8) + sizeof(float) * 8));
    float *pin_lp = (float *)(pin + n + 8);
    struct PinGuard {
        void *p;
        ~PinGuard() { cudaFreeHost(p); }
    } pg{pin};
    memcpy(pin, prompt, sizeof(int32_t) * (size_t)n);
    MLXD_CHECK(cudaMemcpyAsync(m->ctx, pin, sizeof(int32_t) * (size_t)n, cudaMemcpyHostToDevice, st));
    int32_t nctx_h = n;
    MLXD_CHECK(cudaMemcpyAsync(m->n_ctx, &nctx_h, 4, cudaMemcpyHostToDevice, st));
    MLXD_CHECK(cudaMemsetAsync(m->d_step, 0, 8, st));

    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    cudaEventRecord(e0, st);
    nvtxRangePushA("prefill");
    // chunked prefill of prompt[:-1]
    for (int pos = 0; pos < n - 1; pos += chunk) {
        int len = (n - 1 - pos) < chunk ? (n - 1 - pos) : chunk;
        if (site([&] {
                if (ctl->on_prefill_chunk) ctl->on_prefill_chunk(ctl->ud, pos, len);
            }))
            break;
        if (ensure_prefill(m, len) ||
            !cuda_ok(cudaMemcpyAsync(m->p_ids, m->ctx + pos, (size_t)len * 4, cudaMemcpyDeviceToDevice, st),
                     "prefill ids") ||
            forward_dev(m, kv, m->p_ids, len, false, nullptr, st)) {
            nvtxRangePop();
            return -1;
        }
    }
    cudaEventRecord(e1, st);
    nvtxRangePop();
    // the fused greedy argmax needs the raw logits: a repetition penalty
    // (applied before greedy draws too) goes through the sampler
    const bool penalty = sp->repetition_penalty > 0.f && sp->repetition_penalty != 1.0f;
    const bool tp = m->c.tp_size > 1;
    // tensor parallel: logprobs need the whole row, so they go through the
    // gathered row and the sampler too
    const bool greedy = sp->temperature < 0.01f && !penalty && !(tp && logprobs);
    const bool fast = fast_decode_ok(m);
    // device token slot starts as the last prompt token (the seed forward)
    MLXD_CHECK(cudaMemcpyAsync(m->token, m->ctx + n - 1, 4, cudaMemcpyDeviceToDevice, st));
    int emitted = 0;
    int rc = 0;
    // one decode step (forward of m->token, then the token choice), enqueued
    auto enqueue_step = [&](int e) -> int {
        if (check_room(m, kv, 1)) return -1;
        // one CUDA graph per step: the greedy step, or the sampled step with
        // the sampler reading the context length and the draw's step from
        // device counters
        const bool sampled = !greedy;
        if (fast) {
            if (!m->graph_exec || m->graph_kv != kv || m->graph_kv_serial != kv->serial ||
                m->graph_lp != (logprobs != nullptr) || m->graph_sampled != sampled ||
                (sampled && memcmp(&m->graph_sp, sp, sizeof *sp) != 0)) {
                if (m->graph_exec) cudaGraphExecDestroy((cudaGraphExec_t)m->graph_exec);
                m->graph_exec = nullptr;
                cudaGraph_t g;
                MLXD_CHECK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
                int r = decode_step(m, kv, m->token, true, m->logits, !sampled, st, true);
                if (!r && sampled) {
                    const uint16_t *row = m->logits;
                    if (tp) {
                        r = tp_gather_logits(m, m->logits, st, true);
                        row = tp_full_logits(m);
                    }
                    if (!r)
                        r = sample(m->samp, row, MLXD_BF16, m->c.vocab, *sp, m->ctx, 0, 0, m->token,
                                   logprobs ? m->lp : nullptr, nullptr, st, m->n_ctx, m->d_step);
                    if (!r) sampled_step_kernel<<<1, 1, 0, st>>>(m->ctx, m->n_ctx, m->token, m->d_step);
                } else if (!r && logprobs) {
                    logprob_kernel<<<1, 1024, 0, st>>>(m->logits, m->vocab_local, m->token, m->lp);
                }
                cudaError_t ce = cudaStreamEndCapture(st, &g);
                if (r || ce != cudaSuccess) {
                    if (!r) set_error("graph capture: %s", cudaGetErrorString(ce));
                    if (ce == cudaSuccess) cudaGraphDestroy(g);
                    return -1;
                }
                cudaGraphExec_t ge;
                cudaError_t ie = cudaGraphInstantiate(&ge, g, 0);
                cudaGraphDestroy(g);
                if (!cuda_ok(ie, "cudaGraphInstantiate")) return -1;
                m->graph_exec = ge;
                m->graph_kv = kv;
                m->graph_kv_serial = kv->serial;
                m->graph_lp = logprobs != nullptr;
                m->graph_sampled = sampled;
                m->graph_sp = *sp;
            }
            MLXD_CHECK(cudaGraphLaunch((cudaGraphExec_t)m->graph_exec, st));
        } else {
            if (tp) {
                set_error("tensor parallelism needs the one-token decode kernels (head dim 64 or 128)");
                return -1;
            }
            if (generic_forward(m, kv, m->token, 1, true, m->logits, st)) return -1;
            if (sample(m->samp, m->logits, MLXD_BF16, m->vocab_local, *sp, m->ctx, n + e, (uint64_t)e, m->token,
                       logprobs ? m->lp : nullptr, nullptr, st))
                return -1;
            append_token_kernel<<<1, 1, 0, st>>>(m->ctx, n + e, m->token);
        }
        kv->offset += 1;
        MLXD_CHECK(cudaMemcpyAsync(pin + n + (e & 1), m->token, 4, cudaMemcpyDeviceToHost, st));
        if (logprobs) MLXD_CHECK(cudaMemcpyAsync(pin_lp + (e & 1), m->lp, 4, cudaMemcpyDeviceToHost, st));
        return 0;
    };
    std::chrono::steady_clock::time_point t0;
    bool decode_range = false;
    std::vector<cudaEvent_t> evs(2);
    cudaEventCreateWithFlags(&evs[0], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&evs[1], cudaEventDisableTiming);
    // per-step device timestamps (timing[4 + e]: end of step e, ms after prefill)
    std::vector<cudaEvent_t> tev(timing ? max_new : 0);
    for (auto &ev : tev) cudaEventCreate(&ev);
    // the host decode clock starts once the prefill has drained
    if (timing && !cuda_ok(cudaStreamSynchronize(st), "prefill")) {
        rc = -1;
        goto done;
    }
    t0 = std::chrono::steady_clock::now();
    nvtxRangePushA("decode");
    decode_range = true;
    if (ctl && ctl->stopped) goto stopped;   // during the prefill
    if (site([&] {
            if (ctl->on_before_seed) ctl->on_before_seed(ctl->ud);
        }) ||
        site([&] {
            if (ctl->on_decode_step) ctl->on_decode_step(ctl->ud, 0);
        }))
        goto stopped;
    if (enqueue_step(0)) { rc = -1; goto done; }
    cudaEventRecord(evs[0], st);
    if (timing) cudaEventRecord(tev[0], st);
    for (int e = 0; e < max_new; e++) {
        // lookahead: enqueue step e+1 before reading token e
        bool more = e + 1 < max_new;
        // the site of step e + 1; a stop there still emits token e
        if (more && site([&] {
                if (ctl->on_decode_step) ctl->on_decode_step(ctl->ud, e + 1);
            }))
            more = false;
        if (more) {
            if (enqueue_step(e + 1)) { rc = -1; goto done; }
            cudaEventRecord(evs[(e + 1) & 1], st);
            if (timing) cudaEventRecord(tev[e + 1], st);
        }
        if (!cuda_ok(cudaEventSynchronize(evs[e & 1]), "decode step")) { rc = -1; goto done; }
        int32_t tok = pin[n + (e & 1)];
        if (tok < 0 || tok >= m->c.vocab) {
            set_error("sampler produced an invalid token");
            rc = -1;
            goto done;
        }
        bool eos = false;
        for (int i = 0; i < m->c.n_eos && i < 8; i++) eos |= (m->c.eos[i] == tok);
        if (eos) break;
        out[emitted] = tok;
        if (logprobs) logprobs[emitted] = pin_lp[e & 1];
        emitted++;
        if (ctl && ctl->stopped) break;
    }
stopped:
    cudaEventRecord(e2, st);
    if (!cuda_ok(cudaStreamSynchronize(st), "generate")) rc = -1;
    if (!rc && attention_timeouts()) {
        set_error("decode attention: a launch was sized for fewer positions than it met");
        rc = -1;
    }
    if (!rc && tp_timeouts(m)) {
        set_error("tensor-parallel exchange gave up waiting for a peer GPU");
        rc = -1;
    }
    if (!rc && qgemm_tc_timeouts()) {
        set_error("prefill GEMM gave up waiting on its pipeline");
        rc = -1;
    }
    if (timing) {
        float pre = 0.f, dec = 0.f;
        cudaEventElapsedTime(&pre, e0, e1);
        cudaEventElapsedTime(&dec, e1, e2);
        timing[0] = pre;
        timing[1] = dec;
        timing[2] = emitted;
        timing[3] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        for (int e = 0; e < emitted && e < (int)tev.size(); e++) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, e1, tev[e]);
            timing[4 + e] = ms;
        }
    }
done:
    if (decode_range) nvtxRangePop();
    cudaStreamSynchronize(st);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    cudaEventDestroy(evs[0]);
    cudaEventDestroy(evs[1]);
    for (auto &ev : tev) cudaEventDestroy(ev);
    return rc ? -1 : emitted;
}

}  // extern "C"
