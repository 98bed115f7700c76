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
//
// The passes over the vocabulary run on ceil(V / 1024) CTAs of 256 threads,
// one 1024-logit chunk each: statistics (penalty, max, argmax, partial
// logsumexp, scaling, radix pass 0), three further radix passes for top_k,
// then masking and candidate compaction. In each launch the CTA that arrives
// last (an atomic ticket, no waiting) reduces the partials; only order-free
// quantities (max, argmax key, histogram counts) decide the candidate set, so
// it does not depend on the split. The logsumexp (logprob only) combines
// per-chunk partial sums.
#include "common.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(sampler)

constexpr int SAMP_THREADS = 1024;
constexpr int SAMP_CAND = 4096;
constexpr int SAMP_NB = 1024;

constexpr int SAMP_CH = 1024;   // logits per CTA of the parallel passes
constexpr int SAMP_PT = 256;    // threads per CTA of the parallel passes

struct SampMeta {
    float m;        // max of scaled values
    float lse;      // logsumexp of the raw (penalised) logits
    float ck;       // top-k cutoff (or -inf)
    int n_surv;     // survivors after top-k
    int mode;       // 0 greedy done, 1 candidates, 2 full sort
    uint32_t prefix;  // radix select: key bits fixed so far
    int need;         // radix select: rank still to find below the prefix
};

struct SampWork {
    float *xw = nullptr;      // [V] penalised raw logits
    float *sw = nullptr;      // [V] scaled + top-k masked
    float *cand_v = nullptr;  // [CAND]
    int *cand_i = nullptr;
    float *sorted_v = nullptr;  // [V] (full-sort path)
    int *sorted_i = nullptr;
    uint32_t *rs_k = nullptr;       // [V] radix sort: keys and indices between passes
    int *rs_i = nullptr;
    unsigned *rs_off = nullptr;     // [256 * ceil(V / 1024)] per (digit, tile) counts, then offsets
    SampMeta *meta = nullptr;
    // per-CTA partials of the parallel passes ([ceil(V / SAMP_CH)])
    float *p_max = nullptr, *p_sum = nullptr, *p_smax = nullptr;
    unsigned long long *p_key = nullptr;
    unsigned int *hist = nullptr;   // [256] radix histogram (zero between passes)
    unsigned int *ctr = nullptr;    // [2] arrivals, survivors (zero between launches)
    float *ev = nullptr;            // exp(v - m) of the ascending survivors, block-transposed:
                                    // position b*bs + j at ev[j*1024 + b] (bs = ceil(V/1024))
    float *pv = nullptr;            // exp(v - m) / z, same layout (top_p)
    int V = 0;
};

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

// reductions over the SAMP_PT threads of a CTA (result in every thread)
MLXD_DEV float cta_max(float v, float *sh) {
    v = warp_max(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = -INFINITY;
#pragma unroll
    for (int i = 0; i < SAMP_PT / 32; i++) r = fmaxf(r, sh[i]);
    return r;
}
MLXD_DEV float cta_sum(float v, float *sh) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int i = 0; i < SAMP_PT / 32; i++) r += sh[i];
    return r;
}
MLXD_DEV unsigned long long cta_max_u64(unsigned long long v, unsigned long long *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
        v = other > v ? other : v;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long r = 0ull;
#pragma unroll
    for (int i = 0; i < SAMP_PT / 32; i++) r = sh[i] > r ? sh[i] : r;
    return r;
}
// count one value in bin b of a shared-memory histogram: the lanes of a warp
// that share a bin add once (logits crowd a few bins of the top key bytes)
MLXD_DEV void hist_add(unsigned int *hist, unsigned b, bool on) {
    const unsigned act = __ballot_sync(0xffffffffu, on);
    if (!on) return;
    const unsigned peers = __match_any_sync(act, b);
    if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[b], (unsigned)__popc(peers));
}
// true in every thread of the CTA that arrived last at ctr (after its
// writes); that CTA then sees every other CTA's writes
MLXD_DEV bool last_arrival(unsigned int *ctr, bool *s_last) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_last = atomicAdd(ctr, 1u) == gridDim.x - 1;
    __syncthreads();
    if (*s_last) __threadfence();
    return *s_last;
}
// next radix digit (bits shift..shift+7 below the prefix) from the summed
// histogram hs (256 bins, shared memory): the bin holding the need-th largest
// key, i.e. the first bin from the top whose running count reaches need. All
// SAMP_PT (= 256) threads take part: thread t holds bin 255 - t and the
// running counts come from a block scan; *prefix and *need (shared, read by
// every thread beforehand) are updated by the thread that finds the bin.
MLXD_DEV void radix_step(const unsigned int *hs, int shift, uint32_t *prefix, int *need, unsigned *s_wsum) {
    const int t = threadIdx.x, lane = t & 31, wp = t >> 5;
    const unsigned c = hs[255 - t];
    unsigned incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[wp] = incl;
    const int nd = *need;
    const uint32_t pf = *prefix;
    __syncthreads();
    unsigned before = 0;
    for (int k = 0; k < wp; k++) before += s_wsum[k];
    incl += before;
    const unsigned excl = incl - c;
    __syncthreads();
    // the first bin (from the top) whose running count reaches need
    if ((int)incl >= nd && (int)excl < nd) {
        *prefix = pf | ((uint32_t)(255 - t) << shift);
        *need = nd - (int)excl;
    }
    __syncthreads();
}

// Pass 1 over chunk blockIdx.x: logits (repetition penalty applied), their
// max / first-index argmax / exp-sum partials, the scaled values and the
// histogram of their top key byte. The last CTA reduces: greedy token and
// logprob, or the max of the scaled values, the logsumexp and radix digit 0.
template <typename T>
__global__ void __launch_bounds__(SAMP_PT) samp_stats_kernel(
    const void *logits, int V, mlxd_sampling sp, const int32_t *ctx, int n_ctx, SampWork w,
    int32_t *tok, float *lp, int topk, const int32_t *d_nctx) {
    __shared__ float xs[SAMP_CH];
    __shared__ int first[SAMP_CH];
    __shared__ unsigned int hist[256];
    __shared__ float sh[SAMP_PT / 32];
    __shared__ unsigned long long shk[SAMP_PT / 32];
    __shared__ bool s_last;
    const int tid = threadIdx.x;
    const int c0 = blockIdx.x * SAMP_CH, n = min(V - c0, SAMP_CH);
    const bool greedy = sp.temperature < 0.01f;
    if (d_nctx) n_ctx = *d_nctx;
    const bool pen = sp.repetition_penalty > 0.f && sp.repetition_penalty != 1.0f && n_ctx > 0;
    for (int i = tid; i < n; i += SAMP_PT) {
        xs[i] = load_logit<T>(logits, c0 + i);
        first[i] = 0x7fffffff;
    }
    hist[tid] = 0u;
    __syncthreads();
    if (pen) {
        // each distinct id of the last R context tokens once (its first
        // occurrence in the window)
        const int R = sp.repetition_context > 0 ? sp.repetition_context : n_ctx;
        const int start = n_ctx > R ? n_ctx - R : 0;
        for (int j = start + tid; j < n_ctx; j += SAMP_PT) {
            const int id = ctx[j];
            if (id >= c0 && id < c0 + n) atomicMin(&first[id - c0], j);
        }
        __syncthreads();
        for (int i = tid; i < n; i += SAMP_PT)
            if (first[i] != 0x7fffffff) {
                const float x = xs[i];
                xs[i] = x > 0.f ? __fdiv_rn(x, sp.repetition_penalty) : __fmul_rn(x, sp.repetition_penalty);
            }
    }
    float mx = -INFINITY;
    unsigned long long best = 0ull;
    for (int i = tid; i < n; i += SAMP_PT) {
        const float x = xs[i];
        w.xw[c0 + i] = x;
        mx = fmaxf(mx, x);
        const unsigned long long k = ((unsigned long long)ord_key(x) << 32) | (0xFFFFFFFFu - (uint32_t)(c0 + i));
        best = k > best ? k : best;
    }
    mx = cta_max(mx, sh);
    best = cta_max_u64(best, shk);
    float se = 0.f;
    if (mx > -INFINITY)
        for (int i = tid; i < n; i += SAMP_PT) se += expf(xs[i] - mx);
    se = cta_sum(se, sh);
    float smx = -INFINITY;
    if (!greedy) {
        for (int it = 0; it < SAMP_CH / SAMP_PT; it++) {
            const int i = tid + it * SAMP_PT;
            float v = -INFINITY;
            if (i < n) {
                v = sp.temperature != 1.0f ? __fdiv_rn(xs[i], sp.temperature) : xs[i];
                w.sw[c0 + i] = v;
                smx = fmaxf(smx, v);
            }
            if (topk) hist_add(hist, ord_key(v) >> 24, i < n);
        }
        smx = cta_max(smx, sh);
        if (topk && hist[tid]) atomicAdd(&w.hist[tid], hist[tid]);
    }
    if (tid == 0) {
        w.p_max[blockIdx.x] = mx;
        w.p_sum[blockIdx.x] = se;
        w.p_key[blockIdx.x] = best;
        w.p_smax[blockIdx.x] = smx;
    }
    if (!last_arrival(&w.ctr[0], &s_last)) return;
    const int G = gridDim.x;
    float M = -INFINITY, m = -INFINITY;
    unsigned long long key = 0ull;
    for (int g = tid; g < G; g += SAMP_PT) {
        M = fmaxf(M, __ldcg(&w.p_max[g]));
        m = fmaxf(m, __ldcg(&w.p_smax[g]));
        const unsigned long long kg = __ldcg(&w.p_key[g]);
        key = kg > key ? kg : key;
    }
    M = cta_max(M, sh);
    m = cta_max(m, sh);
    key = cta_max_u64(key, shk);
    float S = 0.f;
    for (int g = tid; g < G; g += SAMP_PT) {
        const float pm = __ldcg(&w.p_max[g]);
        if (pm > -INFINITY) S += __ldcg(&w.p_sum[g]) * expf(pm - M);
    }
    S = cta_sum(S, sh);
    __shared__ uint32_t s_prefix;
    __shared__ int s_need;
    __shared__ unsigned s_wsum[SAMP_PT / 32];
    if (topk) {
        hist[tid] = __ldcg(&w.hist[tid]);
        w.hist[tid] = 0u;
        if (tid == 0) {
            s_prefix = 0u;
            s_need = sp.top_k;
        }
        __syncthreads();
        radix_step(hist, 24, &s_prefix, &s_need, s_wsum);
    }
    if (tid == 0) {
        const float lse = M + logf(S);
        if (greedy) {
            const int t = (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
            *tok = t;
            if (lp) *lp = __ldcg(&w.xw[t]) - lse;
            w.meta->mode = 0;
        } else {
            w.meta->m = m;
            w.meta->lse = lse;
            w.meta->ck = -INFINITY;
            if (topk) {
                w.meta->prefix = s_prefix;
                w.meta->need = s_need;
            }
        }
        w.ctr[0] = 0u;
    }
}

// radix passes 1..3 of the top_k select over the scaled values; the last
// CTA fixes the next key byte (and after pass 3 the cutoff)
__global__ void __launch_bounds__(SAMP_PT) samp_radix_kernel(int V, int pass, SampWork w) {
    __shared__ unsigned int hist[256];
    __shared__ bool s_last;
    const int tid = threadIdx.x;
    const int c0 = blockIdx.x * SAMP_CH, n = min(V - c0, SAMP_CH);
    const int shift = 24 - 8 * pass;
    const uint32_t pmask = 0xFFFFFFFFu << (32 - 8 * pass);
    const uint32_t prefix = w.meta->prefix;
    const int need = w.meta->need;
    __shared__ uint32_t s_prefix;
    __shared__ int s_need;
    __shared__ unsigned s_wsum[SAMP_PT / 32];
    hist[tid] = 0u;
    __syncthreads();
    for (int it = 0; it < SAMP_CH / SAMP_PT; it++) {
        const int i = tid + it * SAMP_PT;
        const uint32_t k = i < n ? ord_key(w.sw[c0 + i]) : 0u;
        hist_add(hist, (k >> shift) & 0xFFu, i < n && (k & pmask) == prefix);
    }
    __syncthreads();
    if (hist[tid]) atomicAdd(&w.hist[tid], hist[tid]);
    if (!last_arrival(&w.ctr[0], &s_last)) return;
    hist[tid] = __ldcg(&w.hist[tid]);
    w.hist[tid] = 0u;
    if (tid == 0) {
        s_prefix = prefix;
        s_need = need;
    }
    __syncthreads();
    radix_step(hist, shift, &s_prefix, &s_need, s_wsum);
    if (tid == 0) {
        w.meta->prefix = s_prefix;
        w.meta->need = s_need;
        if (pass == 3) w.meta->ck = key_val(s_prefix);
        w.ctr[0] = 0u;
    }
}

// values below the top_k cutoff masked to -inf; survivors appended to the
// candidate list (one slot reservation per CTA); the last CTA records the
// survivor count and the path (candidates or full sort)
__global__ void __launch_bounds__(SAMP_PT) samp_mask_kernel(int V, SampWork w, int topk) {
    __shared__ float lv[SAMP_CH];
    __shared__ int li[SAMP_CH];
    __shared__ int s_cnt, s_base;
    __shared__ bool s_last;
    const int tid = threadIdx.x, lane = tid & 31;
    const int c0 = blockIdx.x * SAMP_CH, n = min(V - c0, SAMP_CH);
    const float ck = topk ? w.meta->ck : -INFINITY;
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    for (int it = 0; it < SAMP_CH / SAMP_PT; it++) {
        const int i = tid + it * SAMP_PT;
        float v = -INFINITY;
        if (i < n) {
            v = w.sw[c0 + i];
            if (topk && !(v >= ck)) {
                v = -INFINITY;
                w.sw[c0 + i] = v;
            }
        }
        const bool sv = i < n && v > -INFINITY;
        const unsigned bal = __ballot_sync(0xffffffffu, sv);
        int base = 0;
        if (lane == 0 && bal) base = atomicAdd(&s_cnt, __popc(bal));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (sv) {
            const int slot = base + __popc(bal & ((1u << lane) - 1u));
            lv[slot] = v;
            li[slot] = c0 + i;
        }
    }
    __syncthreads();
    if (tid == 0) s_base = s_cnt ? (int)atomicAdd(&w.ctr[1], (unsigned)s_cnt) : 0;
    __syncthreads();
    for (int j = tid; j < s_cnt && s_base + j < SAMP_CAND; j += SAMP_PT) {
        w.cand_v[s_base + j] = lv[j];
        w.cand_i[s_base + j] = li[j];
    }
    if (!last_arrival(&w.ctr[0], &s_last)) return;
    if (tid == 0) {
        const int tot = (int)__ldcg(&w.ctr[1]);
        w.meta->n_surv = tot;
        w.meta->mode = tot <= SAMP_CAND ? 1 : 2;
        w.ctr[1] = 0u;
        w.ctr[0] = 0u;
    }
}

__global__ void samp_keep_token_kernel(int V, const int32_t *tok, uint8_t *keep) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < V) keep[i] = i == *tok ? 1 : 0;
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

// Candidate path: the survivors sorted ascending by (value, index) in shared
// memory and written to the tail of the sorted arrays, where the full-sort
// path leaves its survivors too.
__device__ void finish_stage(int V, const mlxd_sampling &sp, float log_mp, uint64_t step, const SampWork &w,
                             int32_t *tok, float *lp, uint8_t *keep, const unsigned long long *d_step);

// finish_here (no full sort scheduled): the exp values and the final stage
// follow in the same CTA
__global__ void __launch_bounds__(SAMP_THREADS) samp_cand_kernel(
    int V, SampWork w, int32_t *tok, int full_scheduled, mlxd_sampling sp, float log_mp, uint64_t step,
    float *lp, uint8_t *keep, const unsigned long long *d_step, int finish_here) {
    __shared__ float sv[SAMP_CAND];
    __shared__ int si[SAMP_CAND];
    __shared__ int s_gt, s_tie, s_tot, s_wsum[SAMP_THREADS / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int mode = w.meta->mode;
    const int n = w.meta->n_surv;
    if (mode == 0 || (mode == 2 && full_scheduled)) return;
    if (mode == 2) {
        // more survivors than the candidate list holds under a top-k bound:
        // ties at the cutoff ck (the values above it are fewer than
        // k <= 1024). Ascending (value, index) is the ties in index order,
        // then the values above the cutoff: one ordered pass over the row
        // places the ties, the others are sorted here.
        const float ck = w.meta->ck;
        if (tid == 0) s_gt = s_tie = 0;
        __syncthreads();
        for (int c0 = 0; c0 < V; c0 += SAMP_THREADS) {
            const int i = c0 + tid;
            const float v = i < V ? w.sw[i] : -INFINITY;
            if (v > ck) {
                const int slot = atomicAdd(&s_gt, 1);
                if (slot < SAMP_NB) {
                    sv[slot] = v;
                    si[slot] = i;
                }
            }
            const bool tie = i < V && v == ck;
            const unsigned bal = __ballot_sync(0xffffffffu, tie);
            if (lane == 0) s_wsum[warp] = __popc(bal);
            __syncthreads();
            if (warp == 0) {   // exclusive prefix of the warps' tie counts
                const int x = s_wsum[lane];
                int inc = x;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, inc, o);
                    if (lane >= o) inc += y;
                }
                s_wsum[lane] = inc - x;
                if (lane == 31) s_tot = inc;
            }
            __syncthreads();
            if (tie) {
                const int p = V - n + s_tie + s_wsum[warp] + __popc(bal & ((1u << lane) - 1u));
                if (p >= V - n && p < V) {
                    w.sorted_v[p] = v;
                    w.sorted_i[p] = i;
                }
            }
            __syncthreads();
            if (tid == 0) s_tie += s_tot;
            __syncthreads();
        }
        const int ngt = s_gt;
        if (ngt > SAMP_NB || s_tie + ngt != n) {
            // not a top-k cut with ties: report an invalid token, never a wrong one
            if (tid == 0) *tok = -1;
            return;
        }
        int np2 = 1;
        while (np2 < ngt) np2 <<= 1;
        for (int i = ngt + tid; i < np2; i += blockDim.x) {
            sv[i] = __int_as_float(0x7f800000);
            si[i] = 0x7fffffff;
        }
        __syncthreads();
        bitonic_sort_asc(sv, si, np2);
        for (int i = tid; i < ngt; i += blockDim.x) {
            w.sorted_v[V - ngt + i] = sv[i];
            w.sorted_i[V - ngt + i] = si[i];
        }
    } else {
        int np2 = 1;
        while (np2 < n) np2 <<= 1;
        for (int i = threadIdx.x; i < np2; i += blockDim.x) {
            sv[i] = i < n ? w.cand_v[i] : __int_as_float(0x7f800000);
            si[i] = i < n ? w.cand_i[i] : 0x7fffffff;
        }
        __syncthreads();
        bitonic_sort_asc(sv, si, np2);
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            w.sorted_v[V - n + i] = sv[i];
            w.sorted_i[V - n + i] = si[i];
        }
    }
    if (!finish_here) return;
    __syncthreads();   // the sorted survivors (global), seen by every thread
    // exp(v - m) in the final stage's block-transposed layout
    const float m = w.meta->m;
    const int bs = max(1, (V + SAMP_NB - 1) / SAMP_NB);
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const int i = V - n + j;
        w.ev[(i % bs) * SAMP_NB + i / bs] = own_expf(__fsub_rn(w.sorted_v[i], m));
    }
    __syncthreads();   // the CTA's global writes above, seen by every thread
    finish_stage(V, sp, log_mp, step, w, tok, lp, keep, d_step);
}

// exp(v - m) of the n ascending survivors at sorted positions V-n..V-1, in
// the block-transposed layout the final stage reads (thread b of a warp
// walking block b reads 32 consecutive floats per step)
__global__ void samp_exp_kernel(int V, SampWork w, int full_scheduled) {
    const int mode = w.meta->mode;
    if (mode == 0 || (mode == 2 && !full_scheduled)) return;
    const int n = w.meta->n_surv;
    const float m = w.meta->m;
    const int bs = max(1, (V + SAMP_NB - 1) / SAMP_NB);
    for (int i = V - n + blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x)
        w.ev[(i % bs) * SAMP_NB + i / bs] = own_expf(__fsub_rn(w.sorted_v[i], m));
}

// Final stage over the ascending survivors v[V-n..V-1] (sorted position p is
// the p-th smallest of V virtual positions). Every sum below uses the blocked
// association: positions form blocks of bs = ceil(V/1024); a block's values
// are summed in order starting from zero, the block totals are folded in
// block order, and a running sum enters each block at the fold of the
// previous blocks' totals. Thread b owns block b, so the per-block parts run
// in parallel and only the fold over at most 1024 totals is sequential; the
// first position where a running sum crosses its target is the smallest such
// position over all blocks. The result equals the sequential walk bit for bit.
//   top_p: z = sum exp(v - m); cutoff = the value where the running sum of
//          exp(v - m) / z first exceeds 1 - top_p (clamped to the max);
//   min_p: cutoff >= max + log(min_p);
//   draw:  inverse CDF of exp(v - m) over the kept suffix v >= cutoff, at
//          u * (its blocked total), u from SplitMix64 on (seed, step).
// (run by all SAMP_THREADS threads of one CTA)
__device__ void finish_stage(int V, const mlxd_sampling &sp, float log_mp, uint64_t step, const SampWork &w,
                             int32_t *tok, float *lp, uint8_t *keep, const unsigned long long *d_step) {
    __shared__ __align__(16) float sbt[SAMP_NB];
    __shared__ __align__(16) float spre[SAMP_NB];
    __shared__ float s_z, s_thr;
    __shared__ int s_at, s_first;
    MLXD_TRACE_START
    const int tid = threadIdx.x;
    const int n = w.meta->n_surv;
    const float m = w.meta->m;
    const int base = V - n;
    const int bs = max(1, (V + SAMP_NB - 1) / SAMP_NB);
    const int b_lo = base / bs, b_hi = (V - 1) / bs;   // blocks holding survivors
    const float *v = w.sorted_v;
    const int b = tid;
    // exp(v[i] - m) for a position i of this thread's block
    auto ev = [&](int i) { return w.ev[(i - b * bs) * SAMP_NB + b]; };
    // this thread's block clipped to [from, V)
    auto range = [&](int from, int &lo, int &hi) {
        lo = max(from, b * bs);
        hi = min(V, (b + 1) * bs);
    };
    // block totals of f over [from, V) into sbt, then (thread 0) the running
    // prefixes into spre and the total into *total
    auto blocked = [&](int from, auto f, float *total) {
        int lo, hi;
        range(from, lo, hi);
        if (b < SAMP_NB) {
            // 16 values in flight, then added in order
            float bt = 0.f;
            for (int i0 = lo; i0 < hi; i0 += 16) {
                float x[16];
#pragma unroll
                for (int j = 0; j < 16; j++) x[j] = i0 + j < hi ? f(i0 + j) : 0.f;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (i0 + j < hi) bt = __fadd_rn(bt, x[j]);
            }
            sbt[b] = bt;
        }
        __syncthreads();
        if (tid == 0) {
            // the fold over the block totals of blocks b_lo..b_hi, in groups of
            // 8 (blocks without positions in range hold +0, which leaves the
            // non-negative prefix as it is); only the additions are serial
            float prefix = 0.f;
            for (int k0 = b_lo & ~7; k0 <= b_hi; k0 += 8) {
                const float4 q0 = *reinterpret_cast<const float4 *>(sbt + k0);
                const float4 q1 = *reinterpret_cast<const float4 *>(sbt + k0 + 4);
                const float in[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                float out[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    out[j] = prefix;
                    prefix = __fadd_rn(prefix, in[j]);
                }
                *reinterpret_cast<float4 *>(spre + k0) = make_float4(out[0], out[1], out[2], out[3]);
                *reinterpret_cast<float4 *>(spre + k0 + 4) = make_float4(out[4], out[5], out[6], out[7]);
            }
            *total = prefix;
        }
        __syncthreads();
    };
    // smallest position in [from, V) where the running sum of f first
    // exceeds target (and ok(i) holds), or INT_MAX
    auto crossing = [&](int from, auto f, float target, auto ok) {
        if (tid == 0) s_at = 0x7fffffff;
        __syncthreads();
        int lo, hi;
        range(from, lo, hi);
        if (b >= b_lo && b <= b_hi && lo < hi) {
            float run = spre[b];
            bool found = false;
            for (int i0 = lo; i0 < hi && !found; i0 += 16) {
                float x[16];
#pragma unroll
                for (int j = 0; j < 16; j++) x[j] = i0 + j < hi ? f(i0 + j) : 0.f;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (!found && i0 + j < hi) {
                        run = __fadd_rn(run, x[j]);
                        if (run > target && ok(x[j])) {
                            atomicMin(&s_at, i0 + j);
                            found = true;
                        }
                    }
            }
        }
        __syncthreads();
        return s_at;
    };
    float thr = -INFINITY;
    if (sp.top_p < 1.0f) {
        if (sp.top_p <= 0.0f) {
            thr = m;
        } else {
            blocked(base, ev, &s_z);
            MLXD_TRACE_T(tr_z_)
            const float z = s_z;
            // p = exp(v - m) / z, kept for the crossing pass (each thread
            // reads back only its own block)
            auto pf = [&](int i) {
                const float pi = __fdiv_rn(ev(i), z);
                w.pv[(i - b * bs) * SAMP_NB + b] = pi;
                return pi;
            };
            auto pc = [&](int i) { return w.pv[(i - b * bs) * SAMP_NB + b]; };
            blocked(base, pf, &s_thr);   // block totals and prefixes of p
            MLXD_TRACE_T(tr_p_)
            const int at = crossing(base, pc, __fsub_rn(1.0f, sp.top_p), [](float) { return true; });
            MLXD_TRACE_T(tr_c_)
            MLXD_TRACE_REC(tid == 0, 0x90, tr_z_, tr_p_, tr_c_)
            const float cut = at != 0x7fffffff ? v[at] : __int_as_float(0x7f800000);
            thr = fminf(cut, m);
        }
    }
    if (sp.min_p > 0.0f) thr = fmaxf(thr, __fadd_rn(m, log_mp));
    // kept = the suffix with v >= thr: the smallest such position, 16
    // positions (a warp's 16 coalesced rows) in flight per step
    if (tid == 0) s_first = V;
    __syncthreads();
    for (int i0 = base + tid; i0 < V; i0 += 16 * SAMP_THREADS) {
        bool hit[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int i = i0 + j * SAMP_THREADS;
            hit[j] = i < V && v[i] >= thr;
        }
        int f = 0x7fffffff;
#pragma unroll
        for (int j = 15; j >= 0; j--)
            if (hit[j]) f = i0 + j * SAMP_THREADS;
        if (f != 0x7fffffff) {
            atomicMin(&s_first, f);
            break;
        }
    }
    __syncthreads();
    const int first = s_first;
    MLXD_TRACE_T(tr_f_)
    blocked(first, ev, &s_z);
    MLXD_TRACE_T(tr_z2_)
    const float z2 = s_z;
    const float u = draw_uniform(sp.seed < 0 ? 0 : sp.seed, d_step ? *d_step : step);
    const int at = crossing(first, ev, __fmul_rn(u, z2),
                            [](float e) { return e > 0.f; });
    const int pick = at != 0x7fffffff ? at : V - 1;
    MLXD_TRACE_T(tr_d_)
    MLXD_TRACE_REC(tid == 0, 0x91, tr_f_, tr_z2_, tr_d_)
    if (tid == 0) {
        const int t = w.sorted_i[pick];
        *tok = t;
        if (lp) *lp = w.xw[t] - w.meta->lse;
    }
    if (keep)
#pragma unroll 8
        for (int i = tid; i < V; i += blockDim.x) {
            const float x = w.sw[i];
            keep[i] = (x > -INFINITY && x >= thr) ? 1 : 0;
        }
    MLXD_TRACE_WAITED
    MLXD_TRACE_END(0x92)
}

// the final stage after the full-vocabulary sort
__global__ void __launch_bounds__(SAMP_THREADS) samp_finish_kernel(
    int V, mlxd_sampling sp, float log_mp, uint64_t step, SampWork w, int32_t *tok, float *lp,
    uint8_t *keep, int full_scheduled, const unsigned long long *d_step) {
    const int mode = w.meta->mode;
    if (mode == 0 || (mode == 2 && !full_scheduled)) return;
    finish_stage(V, sp, log_mp, step, w, tok, lp, keep, d_step);
}

// ------------------------------------------------ full-row sort (no top-k)
//
// Stable LSD radix sort of the masked row by its order key (ord_key, the
// float order with -inf first; equal values keep index order), 8 bits per
// pass: per pass a histogram of each 1024-entry tile, one CTA's exclusive
// scan over (digit, tile), and a stable scatter. Pass 0 reads the row
// itself, pass 3 writes the values back as floats; the passes ping-pong
// between the sorted arrays and a second key/index pair. Every kernel is a
// no-op unless the row took the full path (mode 2).
constexpr int RS_TILE = 1024, RS_T = 256;

__global__ void __launch_bounds__(RS_T) rs_hist_kernel(int V, SampWork w, int pass, const uint32_t *keys) {
    if (w.meta->mode != 2) return;
    __shared__ unsigned h[256];
    const int tid = threadIdx.x, c0 = blockIdx.x * RS_TILE, G = gridDim.x;
    h[tid] = 0u;
    __syncthreads();
    for (int r = 0; r < RS_TILE / RS_T; r++) {
        const int i = c0 + r * RS_T + tid;
        if (i < V) {
            const uint32_t k = pass == 0 ? ord_key(w.sw[i]) : keys[i];
            atomicAdd(&h[(k >> (8 * pass)) & 255u], 1u);
        }
    }
    __syncthreads();
    w.rs_off[tid * G + blockIdx.x] = h[tid];
}

// exclusive prefix over the (digit, tile) counts in digit-major order: warp w
// owns a contiguous segment (a multiple of 32 counts); it sums its segment,
// the 32 segment totals are scanned once, then each warp walks its segment
// 32 counts at a time (coalesced), a warp scan per step plus the carry
__global__ void __launch_bounds__(1024) rs_scan_kernel(SampWork w, int G) {
    if (w.meta->mode != 2) return;
    __shared__ unsigned wtot[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, n = 256 * G;
    const int seg = ((n + 32 * 32 - 1) / (32 * 32)) * 32;
    const int s0 = warp * seg, s1 = min(n, s0 + seg);
    unsigned t = 0u;
#pragma unroll 8
    for (int i = s0 + lane; i < s1; i += 32) t += w.rs_off[i];
    t = __reduce_add_sync(0xffffffffu, t);
    if (lane == 0) wtot[warp] = t;
    __syncthreads();
    if (warp == 0) {
        const unsigned own = wtot[lane];
        unsigned x = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        wtot[lane] = x - own;
    }
    __syncthreads();
    unsigned carry = wtot[warp];
#pragma unroll 4
    for (int b0 = s0; b0 < s1; b0 += 32) {
        const int i = b0 + lane;
        const unsigned v = i < s1 ? w.rs_off[i] : 0u;
        unsigned x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (i < s1) w.rs_off[i] = carry + x - v;
        carry += __shfl_sync(0xffffffffu, x, 31);
    }
}

// stable scatter of one tile: rounds of 256 consecutive entries; in a round
// an entry's place among equal digits is its lane rank in the warp plus the
// counts of the earlier warps and of the earlier rounds
__global__ void __launch_bounds__(RS_T) rs_scatter_kernel(int V, SampWork w, int pass, const uint32_t *kin,
                                                          const int *iin, uint32_t *kout, int *iout) {
    if (w.meta->mode != 2) return;
    __shared__ unsigned base[256];
    __shared__ unsigned wc[RS_T / 32][256];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, G = gridDim.x;
    const int c0 = blockIdx.x * RS_TILE;
    base[tid] = w.rs_off[tid * G + blockIdx.x];
    for (int r = 0; r < RS_TILE / RS_T; r++) {
        for (int x = 0; x < RS_T / 32; x++) wc[x][tid] = 0u;
        __syncthreads();
        const int i = c0 + r * RS_T + tid;
        const bool valid = i < V;
        uint32_t k = 0u;
        int ix = 0;
        if (valid) {
            k = pass == 0 ? ord_key(w.sw[i]) : kin[i];
            ix = pass == 0 ? i : iin[i];
        }
        const unsigned d = valid ? (k >> (8 * pass)) & 255u : 256u;
        const unsigned peers = __match_any_sync(0xffffffffu, d);
        const unsigned rank = __popc(peers & ((1u << lane) - 1u));
        if (valid && rank == 0) wc[warp][d] = __popc(peers);
        __syncthreads();
        // per digit (thread = digit): the earlier warps' counts, and the total
        unsigned run = 0u;
#pragma unroll
        for (int x = 0; x < RS_T / 32; x++) {
            const unsigned c = wc[x][tid];
            wc[x][tid] = run;
            run += c;
        }
        __syncthreads();
        if (valid) {
            const unsigned dst = base[d] + wc[warp][d] + rank;
            if (pass == 3) {
                w.sorted_v[dst] = key_val(k);
                w.sorted_i[dst] = ix;
            } else {
                kout[dst] = k;
                iout[dst] = ix;
            }
        }
        __syncthreads();
        base[tid] += run;
    }
}

// the four passes: sw -> (rs_k, rs_i) -> (sorted as keys) -> (rs_k, rs_i) -> sorted
static void rs_sort(int V, const SampWork &w, cudaStream_t st) {
    const int G = (V + RS_TILE - 1) / RS_TILE;
    uint32_t *ka = w.rs_k, *kb = reinterpret_cast<uint32_t *>(w.sorted_v);
    int *ia = w.rs_i, *ib = w.sorted_i;
    const uint32_t *kin = nullptr;
    const int *iin = nullptr;
    for (int pass = 0; pass < 4; pass++) {
        uint32_t *ko = pass % 2 == 0 ? ka : kb;
        int *io = pass % 2 == 0 ? ia : ib;
        rs_hist_kernel<<<G, RS_T, 0, st>>>(V, w, pass, kin);
        rs_scan_kernel<<<1, 1024, 0, st>>>(w, G);
        rs_scatter_kernel<<<G, RS_T, 0, st>>>(V, w, pass, kin, iin, ko, io);
        kin = ko;
        iin = io;
    }
}

void samp_work_destroy(SampWork *w) {
    if (!w) return;
    dev_free(w->xw); dev_free(w->sw); dev_free(w->cand_v); dev_free(w->cand_i);
    dev_free(w->sorted_v); dev_free(w->sorted_i); dev_free(w->rs_k); dev_free(w->rs_i); dev_free(w->rs_off);
    dev_free(w->meta);
    dev_free(w->p_max); dev_free(w->p_sum); dev_free(w->p_smax); dev_free(w->p_key);
    dev_free(w->hist); dev_free(w->ctr); dev_free(w->ev); dev_free(w->pv);
    delete w;
}

int samp_work_capacity(const SampWork *w) { return w ? w->V : 0; }

// scratch for rows of up to V logits on the current device (its caller owns
// it: one per model, so that a captured decode graph keeps valid pointers)
SampWork *samp_work_create(int V) {
    if (V <= 0) {
        set_error("sample: bad vocabulary size %d", V);
        return nullptr;
    }
    SampWork *pw = new SampWork();
    SampWork &w = *pw;
    w.xw = (float *)dev_alloc(sizeof(float) * V);
    w.sw = (float *)dev_alloc(sizeof(float) * V);
    w.cand_v = (float *)dev_alloc(sizeof(float) * SAMP_CAND);
    w.cand_i = (int *)dev_alloc(sizeof(int) * SAMP_CAND);
    w.sorted_v = (float *)dev_alloc(sizeof(float) * V);
    w.sorted_i = (int *)dev_alloc(sizeof(int) * V);
    w.rs_k = (uint32_t *)dev_alloc(sizeof(uint32_t) * V);
    w.rs_i = (int *)dev_alloc(sizeof(int) * V);
    w.rs_off = (unsigned *)dev_alloc(sizeof(unsigned) * 256 * (size_t)((V + RS_TILE - 1) / RS_TILE));
    w.meta = (SampMeta *)dev_alloc(sizeof(SampMeta));
    const int G = (V + SAMP_CH - 1) / SAMP_CH;
    w.p_max = (float *)dev_alloc(sizeof(float) * G);
    w.p_sum = (float *)dev_alloc(sizeof(float) * G);
    w.p_smax = (float *)dev_alloc(sizeof(float) * G);
    w.p_key = (unsigned long long *)dev_alloc(sizeof(unsigned long long) * G);
    w.hist = (unsigned int *)dev_alloc(sizeof(unsigned int) * 256);
    w.ctr = (unsigned int *)dev_alloc(sizeof(unsigned int) * 2);
    w.ev = (float *)dev_alloc(sizeof(float) * ((V + SAMP_NB - 1) / SAMP_NB) * SAMP_NB);
    w.pv = (float *)dev_alloc(sizeof(float) * ((V + SAMP_NB - 1) / SAMP_NB) * SAMP_NB);
    if (!w.xw || !w.sw || !w.cand_v || !w.cand_i || !w.sorted_v || !w.sorted_i || !w.rs_k || !w.rs_i ||
        !w.rs_off || !w.meta || !w.p_max || !w.p_sum || !w.p_smax || !w.p_key || !w.hist || !w.ctr || !w.ev ||
        !w.pv) {
        samp_work_destroy(pw);
        return nullptr;
    }
    if (cudaMemset(w.hist, 0, sizeof(unsigned int) * 256) != cudaSuccess ||
        cudaMemset(w.ctr, 0, sizeof(unsigned int) * 2) != cudaSuccess) {
        set_error("sample: clearing the sampler's counters failed");
        samp_work_destroy(pw);
        return nullptr;
    }
    w.V = V;
    return pw;
}

int sample(SampWork *pw, const void *logits, int dtype, int V, const mlxd_sampling &sp, const int32_t *ctx,
           int n_ctx, uint64_t step, int32_t *tok, float *lp, uint8_t *keep, cudaStream_t st,
           const int32_t *d_nctx, const unsigned long long *d_step) {
    if (V <= 0 || !tok || !pw) {
        set_error("sample: bad arguments");
        return -1;
    }
    if (pw->V < V) {
        set_error("sample: scratch for %d logits, row of %d", pw->V, V);
        return -1;
    }
    const SampWork &w = *pw;
    const int G = (V + SAMP_CH - 1) / SAMP_CH;
    const bool greedy = sp.temperature < 0.01f;
    const int topk = !greedy && sp.top_k > 0 && sp.top_k < V;
    if (dtype == MLXD_BF16)
        samp_stats_kernel<uint16_t><<<G, SAMP_PT, 0, st>>>(logits, V, sp, ctx, n_ctx, w, tok, lp, topk, d_nctx);
    else if (dtype == MLXD_F32)
        samp_stats_kernel<float><<<G, SAMP_PT, 0, st>>>(logits, V, sp, ctx, n_ctx, w, tok, lp, topk, d_nctx);
    else {
        set_error("sample: logits dtype must be bf16 or f32");
        return -1;
    }
    MLXD_CHECK(cudaGetLastError());
    if (greedy) {
        if (keep) samp_keep_token_kernel<<<(V + 255) / 256, 256, 0, st>>>(V, tok, keep);
        MLXD_CHECK(cudaGetLastError());
        return 0;
    }
    if (topk)
        for (int pass = 1; pass < 4; pass++) samp_radix_kernel<<<G, SAMP_PT, 0, st>>>(V, pass, w);
    samp_mask_kernel<<<G, SAMP_PT, 0, st>>>(V, w, topk);
    MLXD_CHECK(cudaGetLastError());
    float log_mp = sp.min_p > 0.0f ? logf(sp.min_p) : 0.0f;
    // With top_k <= 1024 the survivors fit the candidate list unless more than
    // 3072 values tie at the cutoff; otherwise the whole vocabulary is sorted.
    bool need_full = !(sp.top_k > 0 && sp.top_k <= 1024);
    samp_cand_kernel<<<1, SAMP_THREADS, 0, st>>>(V, w, tok, need_full, sp, log_mp, step, lp, keep, d_step,
                                                 !need_full);
    MLXD_CHECK(cudaGetLastError());
    if (!need_full) return 0;   // the candidate kernel finished the draw
    // ascending (value, index) over the whole row: the stable radix sort
    rs_sort(V, w, st);
    MLXD_CHECK(cudaGetLastError());
    samp_exp_kernel<<<(V + 1023) / 1024, 256, 0, st>>>(V, w, need_full);
    samp_finish_kernel<<<1, SAMP_THREADS, 0, st>>>(V, sp, log_mp, step, w, tok, lp, keep, need_full, d_step);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace mlxd
