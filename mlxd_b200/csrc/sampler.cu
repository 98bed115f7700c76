// Sampler (sampler_sample_lazy, src/engine/sampler.c:269-380).
//
// Greedy below T = 0.01: first index of the maximum (mlx argmax), logprob from
// the raw logits. Otherwise, on f32 values: repetition penalty (build-defined;
// the reference has none -- mlx-lm's rule x>0 ? x/p : x*p over the distinct
// ids of the last R context tokens), logits / T, top_k (keep x >= k-th largest,
// ties kept; exact radix select over order-preserving keys), top_p (ascending
// order, softmax, inclusive cumsum, cutoff = smallest logit whose cumsum >
// 1-p, clamped to the max), min_p (keep x >= max + log(min_p)), then a draw by
// inverse CDF over the kept values in ascending order.
//
// Sums over the ascending order use the oracle's fixed association: the V
// sorted positions form 1024 blocks of ceil(V/1024); a running f32 sum enters
// each block at the running total of the previous blocks' block sums. Masked
// values contribute exact zeros, so when top_k leaves few survivors the sums
// are formed from the survivors alone at their virtual positions. exp is the
// shared Cody-Waite implementation, so candidate sets match the oracle bit for
// bit given identical logits. Uniforms: SplitMix64 on (seed, step).
#include <cub/cub.cuh>
#include "common.cuh"
#include "kernels.h"

namespace mlxd {

constexpr int SAMP_THREADS = 1024;
constexpr int SAMP_CAND = 4096;
constexpr int SAMP_NB = 1024;

struct SampMeta {
    float m;        // max of scaled values
    float lse;      // logsumexp of the raw (penalised) logits
    float ck;       // top-k cutoff (or -inf)
    int n_surv;     // survivors after top-k
    int mode;       // 0 greedy done, 1 candidates, 2 full sort
};

struct SampWork {
    float *xw = nullptr;      // [V] penalised raw logits
    float *sw = nullptr;      // [V] scaled + top-k masked
    float *cand_v = nullptr;  // [CAND]
    int *cand_i = nullptr;
    float *sorted_v = nullptr;  // [V] (full-sort path)
    int *sorted_i = nullptr;
    int *idx_in = nullptr;
    void *cub_tmp = nullptr;
    size_t cub_bytes = 0;
    SampMeta *meta = nullptr;
    int V = 0;
};
static SampWork g_work;

MLXD_DEV uint32_t ord_key(float v) {
    uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
MLXD_DEV float key_val(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

MLXD_DEV uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
MLXD_DEV float draw_uniform(int seed, uint64_t step) {
    uint64_t k = splitmix64(((uint64_t)(uint32_t)seed << 32) ^ 0x6d6c7864ull);
    uint64_t r = splitmix64(k + step * 0x9E3779B97F4A7C15ull);
    return __fmul_rn((float)(r >> 40), 1.0f / 16777216.0f);
}

template <typename T>
MLXD_DEV float load_logit(const void *p, int i) {
    if constexpr (sizeof(T) == 2) return bf2f(((const uint16_t *)p)[i]);
    else return ((const float *)p)[i];
}

// block reductions for 1024 threads
MLXD_DEV float block_max(float v, float *sh) {
    v = warp_max(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float r = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) r = fmaxf(r, sh[i]);
    return r;
}
MLXD_DEV float block_sum(float v, float *sh) {
    v = warp_sum(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float r = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) r += sh[i];
    return r;
}

template <typename T>
__global__ void __launch_bounds__(SAMP_THREADS) samp_prep_kernel(
    const void *logits, int V, mlxd_sampling sp, const int32_t *ctx, int n_ctx, SampWork w,
    int32_t *tok, float *lp, uint8_t *keep) {
    __shared__ float sh[32];
    __shared__ unsigned int hist[256];
    __shared__ uint32_t s_prefix;
    __shared__ int s_need;
    const int tid = threadIdx.x;
    const bool greedy = sp.temperature < 0.01f;
    for (int i = tid; i < V; i += SAMP_THREADS) w.xw[i] = load_logit<T>(logits, i);
    __syncthreads();
    if (!greedy && tid == 0 && sp.repetition_penalty > 0.f && sp.repetition_penalty != 1.0f &&
        n_ctx > 0) {
        int R = sp.repetition_context > 0 ? sp.repetition_context : n_ctx;
        int start = n_ctx > R ? n_ctx - R : 0;
        for (int i = start; i < n_ctx; i++) {
            int id = ctx[i];
            if (id < 0 || id >= V) continue;
            bool dup = false;
            for (int k = start; k < i; k++) dup |= (ctx[k] == id);
            if (dup) continue;
            float x = w.xw[id];
            w.xw[id] = x > 0.f ? __fdiv_rn(x, sp.repetition_penalty) : __fmul_rn(x, sp.repetition_penalty);
        }
    }
    __syncthreads();
    // max and logsumexp of the raw values; greedy argmax (first index)
    float mx = -INFINITY;
    unsigned long long best = 0;
    for (int i = tid; i < V; i += SAMP_THREADS) {
        float x = w.xw[i];
        mx = fmaxf(mx, x);
        unsigned long long k = ((unsigned long long)ord_key(x) << 32) | (0xFFFFFFFFu - (uint32_t)i);
        best = k > best ? k : best;
    }
    mx = block_max(mx, sh);
    float se = 0.f;
    for (int i = tid; i < V; i += SAMP_THREADS) se += expf(w.xw[i] - mx);
    se = block_sum(se, sh);
    float lse = mx + logf(se);
    if (greedy) {
        __shared__ unsigned long long sb[32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if ((tid & 31) == 0) sb[tid >> 5] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0;
            for (int i = 0; i < SAMP_THREADS / 32; i++) b = sb[i] > b ? sb[i] : b;
            int t = (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
            *tok = t;
            if (lp) *lp = w.xw[t] - lse;
            w.meta->mode = 0;
        }
        if (keep) {
            __syncthreads();
            for (int i = tid; i < V; i += SAMP_THREADS) keep[i] = 0;
            __syncthreads();
            if (tid == 0) keep[*tok] = 1;
        }
        return;
    }
    // scaled values
    for (int i = tid; i < V; i += SAMP_THREADS) {
        float x = w.xw[i];
        w.sw[i] = sp.temperature != 1.0f ? __fdiv_rn(x, sp.temperature) : x;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int i = tid; i < V; i += SAMP_THREADS) m = fmaxf(m, w.sw[i]);
    m = block_max(m, sh);
    // top-k cutoff by radix select on order-preserving keys (MSB first)
    float ck = -INFINITY;
    if (sp.top_k > 0 && sp.top_k < V) {
        if (tid == 0) {
            s_prefix = 0;
            s_need = sp.top_k;
        }
        for (int pass = 0; pass < 4; pass++) {
            int shift = 24 - 8 * pass;
            for (int b = tid; b < 256; b += SAMP_THREADS) hist[b] = 0;
            __syncthreads();
            uint32_t prefix = s_prefix;
            uint32_t pmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
            for (int i = tid; i < V; i += SAMP_THREADS) {
                uint32_t k = ord_key(w.sw[i]);
                if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFF], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int need = s_need;
                for (int b = 255; b >= 0; b--) {
                    int c = (int)hist[b];
                    if (c >= need) {
                        s_prefix = prefix | ((uint32_t)b << shift);
                        break;
                    }
                    need -= c;
                }
                s_need = need;
            }
            __syncthreads();
        }
        ck = key_val(s_prefix);
        for (int i = tid; i < V; i += SAMP_THREADS)
            if (!(w.sw[i] >= ck)) w.sw[i] = -INFINITY;
        __syncthreads();
    }
    // survivors
    __shared__ int s_cnt;
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    for (int i = tid; i < V; i += SAMP_THREADS) {
        float v = w.sw[i];
        if (v > -INFINITY) {
            int slot = atomicAdd(&s_cnt, 1);
            if (slot < SAMP_CAND) {
                w.cand_v[slot] = v;
                w.cand_i[slot] = i;
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        w.meta->m = m;
        w.meta->lse = lse;
        w.meta->ck = ck;
        w.meta->n_surv = s_cnt;
        w.meta->mode = s_cnt <= SAMP_CAND ? 1 : 2;
    }
}

// Ascending (value, index) order over a candidate list in shared memory.
__device__ void bitonic_sort_asc(float *v, int *ix, int n_pow2) {
    for (int k = 2; k <= n_pow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
                int p = i ^ j;
                if (p > i) {
                    bool up = (i & k) == 0;
                    float a = v[i], b = v[p];
                    int ia = ix[i], ib = ix[p];
                    bool gt = (a > b) || (a == b && ia > ib);
                    if (gt == up) {
                        v[i] = b; v[p] = a;
                        ix[i] = ib; ix[p] = ia;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Final stage on an ascending list of n values (the top n of V virtual
// positions), sequential in one thread with the blocked association.
__device__ void finish_sequential(const float *v, const int *ix, int n, int V, float m,
                                  const mlxd_sampling &sp, float log_mp, uint64_t step,
                                  float *out_thr, int *out_tok) {
    const int bs = max(1, (V + SAMP_NB - 1) / SAMP_NB);
    const int base = V - n;
    // softmax denominator z over the survivors
    auto blocked_total = [&](auto val_of, int from) {
        float prefix = 0.f, bt = 0.f;
        int cur = -1;
        for (int i = from; i < n; i++) {
            int b = (base + i) / bs;
            if (b != cur) {
                prefix = __fadd_rn(prefix, bt);
                bt = 0.f;
                cur = b;
            }
            bt = __fadd_rn(bt, val_of(i));
        }
        return __fadd_rn(prefix, bt);
    };
    float thr = -INFINITY;
    if (sp.top_p < 1.0f) {
        if (sp.top_p <= 0.0f) {
            thr = m;
        } else {
            float z = blocked_total([&](int i) { return own_expf(__fsub_rn(v[i], m)); }, 0);
            float t1 = __fsub_rn(1.0f, sp.top_p);
            float prefix = 0.f, bt = 0.f, run = 0.f;
            int cur = -1;
            float cut = __int_as_float(0x7f800000);
            for (int i = 0; i < n; i++) {
                int b = (base + i) / bs;
                if (b != cur) {
                    prefix = __fadd_rn(prefix, bt);
                    bt = 0.f;
                    run = prefix;
                    cur = b;
                }
                float p = __fdiv_rn(own_expf(__fsub_rn(v[i], m)), z);
                run = __fadd_rn(run, p);
                bt = __fadd_rn(bt, p);
                if (run > t1) {
                    cut = v[i];
                    break;
                }
            }
            thr = fminf(cut, m);
        }
    }
    if (sp.min_p > 0.0f) thr = fmaxf(thr, __fadd_rn(m, log_mp));
    // kept = suffix with v >= thr
    int first = 0;
    while (first < n && !(v[first] >= thr)) first++;
    int nk = n - first;
    // categorical over the kept suffix at virtual positions V-nk..V-1
    const int kbase = V - nk;
    float z2;
    {
        float prefix = 0.f, bt = 0.f;
        int cur = -1;
        for (int i = 0; i < nk; i++) {
            int b = (kbase + i) / bs;
            if (b != cur) {
                prefix = __fadd_rn(prefix, bt);
                bt = 0.f;
                cur = b;
            }
            bt = __fadd_rn(bt, own_expf(__fsub_rn(v[first + i], m)));
        }
        z2 = __fadd_rn(prefix, bt);
    }
    float u = draw_uniform(sp.seed < 0 ? 0 : sp.seed, step);
    float target = __fmul_rn(u, z2);
    int pick = n - 1;
    {
        float prefix = 0.f, bt = 0.f, run = 0.f;
        int cur = -1;
        for (int i = 0; i < nk; i++) {
            int b = (kbase + i) / bs;
            if (b != cur) {
                prefix = __fadd_rn(prefix, bt);
                bt = 0.f;
                run = prefix;
                cur = b;
            }
            float e = own_expf(__fsub_rn(v[first + i], m));
            run = __fadd_rn(run, e);
            bt = __fadd_rn(bt, e);
            if (run > target && e > 0.f) {
                pick = first + i;
                break;
            }
        }
    }
    *out_thr = thr;
    *out_tok = ix[pick];
}

__global__ void __launch_bounds__(SAMP_THREADS) samp_cand_kernel(
    int V, mlxd_sampling sp, float log_mp, uint64_t step, SampWork w, int32_t *tok, float *lp,
    uint8_t *keep, int full_scheduled) {
    __shared__ float sv[SAMP_CAND];
    __shared__ int si[SAMP_CAND];
    __shared__ float s_thr;
    __shared__ int s_tok;
    if (w.meta->mode == 2 && !full_scheduled) {
        // more tied survivors than the candidate list holds and no full sort
        // was scheduled: report an invalid token instead of a wrong one
        if (threadIdx.x == 0) *tok = -1;
        return;
    }
    if (w.meta->mode != 1) return;
    int n = w.meta->n_surv;
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        sv[i] = i < n ? w.cand_v[i] : __int_as_float(0x7f800000);
        si[i] = i < n ? w.cand_i[i] : 0x7fffffff;
    }
    __syncthreads();
    bitonic_sort_asc(sv, si, np2);
    if (threadIdx.x == 0) {
        finish_sequential(sv, si, n, V, w.meta->m, sp, log_mp, step, &s_thr, &s_tok);
        *tok = s_tok;
        if (lp) *lp = w.xw[s_tok] - w.meta->lse;
    }
    __syncthreads();
    if (keep) {
        float thr = s_thr;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            float v = w.sw[i];
            keep[i] = (v > -INFINITY && v >= thr) ? 1 : 0;
        }
    }
}

__global__ void iota_kernel(int *p, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = i;
}

// full-sort path: the ascending list lives in global memory
__global__ void samp_full_kernel(int V, mlxd_sampling sp, float log_mp, uint64_t step, SampWork w,
                                 int32_t *tok, float *lp, uint8_t *keep) {
    __shared__ float s_thr;
    __shared__ int s_tok;
    if (w.meta->mode != 2) return;
    if (threadIdx.x == 0) {
        // masked (-inf) entries sort first; survivors are the top n_surv
        int n = w.meta->n_surv;
        finish_sequential(w.sorted_v + (V - n), w.sorted_i + (V - n), n, V, w.meta->m, sp, log_mp,
                          step, &s_thr, &s_tok);
        *tok = s_tok;
        if (lp) *lp = w.xw[s_tok] - w.meta->lse;
    }
    __syncthreads();
    if (keep) {
        float thr = s_thr;
        for (int i = threadIdx.x; i < V; i += blockDim.x) {
            float v = w.sw[i];
            keep[i] = (v > -INFINITY && v >= thr) ? 1 : 0;
        }
    }
}

static int ensure_work(int V) {
    if (g_work.V >= V) return 0;
    SampWork &w = g_work;
    dev_free(w.xw); dev_free(w.sw); dev_free(w.cand_v); dev_free(w.cand_i);
    dev_free(w.sorted_v); dev_free(w.sorted_i); dev_free(w.idx_in); dev_free(w.cub_tmp);
    dev_free(w.meta);
    w = SampWork{};
    w.xw = (float *)dev_alloc(sizeof(float) * V);
    w.sw = (float *)dev_alloc(sizeof(float) * V);
    w.cand_v = (float *)dev_alloc(sizeof(float) * SAMP_CAND);
    w.cand_i = (int *)dev_alloc(sizeof(int) * SAMP_CAND);
    w.sorted_v = (float *)dev_alloc(sizeof(float) * V);
    w.sorted_i = (int *)dev_alloc(sizeof(int) * V);
    w.idx_in = (int *)dev_alloc(sizeof(int) * V);
    w.meta = (SampMeta *)dev_alloc(sizeof(SampMeta));
    size_t tmp = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, tmp, (const float *)nullptr, (float *)nullptr,
                                    (const int *)nullptr, (int *)nullptr, V);
    w.cub_tmp = dev_alloc(tmp);
    w.cub_bytes = tmp;
    if (!w.xw || !w.sw || !w.cand_v || !w.cand_i || !w.sorted_v || !w.sorted_i || !w.idx_in ||
        !w.meta || !w.cub_tmp)
        return -1;
    w.V = V;
    return 0;
}

int sample(const void *logits, int dtype, int V, const mlxd_sampling &sp, const int32_t *ctx,
           int n_ctx, uint64_t step, int32_t *tok, float *lp, uint8_t *keep, cudaStream_t st) {
    if (V <= 0 || !tok) {
        set_error("sample: bad arguments");
        return -1;
    }
    if (ensure_work(V)) return -1;
    SampWork w = g_work;
    if (dtype == MLXD_BF16)
        samp_prep_kernel<uint16_t><<<1, SAMP_THREADS, 0, st>>>(logits, V, sp, ctx, n_ctx, w, tok, lp, keep);
    else if (dtype == MLXD_F32)
        samp_prep_kernel<float><<<1, SAMP_THREADS, 0, st>>>(logits, V, sp, ctx, n_ctx, w, tok, lp, keep);
    else {
        set_error("sample: logits dtype must be bf16 or f32");
        return -1;
    }
    MLXD_CHECK(cudaGetLastError());
    if (sp.temperature < 0.01f) return 0;
    float log_mp = sp.min_p > 0.0f ? logf(sp.min_p) : 0.0f;
    // With top_k <= 1024 the survivors fit the candidate list unless more than
    // 3072 values tie at the cutoff; otherwise the whole vocabulary is sorted.
    bool need_full = !(sp.top_k > 0 && sp.top_k <= 1024);
    samp_cand_kernel<<<1, SAMP_THREADS, 0, st>>>(V, sp, log_mp, step, w, tok, lp, keep, need_full);
    MLXD_CHECK(cudaGetLastError());
    if (need_full) {
        iota_kernel<<<(V + 255) / 256, 256, 0, st>>>(w.idx_in, V);
        size_t tmp = w.cub_bytes;
        MLXD_CHECK(cub::DeviceRadixSort::SortPairs(w.cub_tmp, tmp, w.sw, w.sorted_v, w.idx_in,
                                                   w.sorted_i, V, 0, 32, st));
        samp_full_kernel<<<1, SAMP_THREADS, 0, st>>>(V, sp, log_mp, step, w, tok, lp, keep);
        MLXD_CHECK(cudaGetLastError());
    }
    return 0;
}

__global__ void argmax_decode_kernel(const unsigned long long *amax, int32_t *tok) {
    *tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(*amax & 0xFFFFFFFFull));
}

int argmax_decode(const unsigned long long *amax, int32_t *tok, cudaStream_t st) {
    argmax_decode_kernel<<<1, 1, 0, st>>>(amax, tok);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace mlxd
