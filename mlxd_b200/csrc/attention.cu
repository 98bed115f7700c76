// Attention for the decoder step (mlx_fast_scaled_dot_product_attention,
// src/engine/forward.c:713-731, with the KV update of kvcache.c:98-180).
//
// * attention_decode: one new token. Split-KV flash-decode, grid (kv head,
//   split). Each CTA also does the token's q/k RMSNorm + RoPE (fwd_attention
//   :591-697) for its GQA group and the KV append (split 0 writes the slot;
//   the split that covers the new position reads it from shared memory, so no
//   CTA waits on another). Partial (max, sum, o) per split go to a scratch
//   buffer; the last CTA of a kv head (atomic counter) merges them.
// * attention_prefill: S queries over the cache, FA2-style mma.sync tiles,
//   causal (bottom-right aligned) plus the sliding-window rule
//   0 <= (pos_q - pos_k) < window (fwd_sliding_window_mask, forward.c:241-292).
// * attention_small: head dims outside {64, 128} take mlx's composed
//   fallback (q*scale in bf16, bf16 scores, precise softmax rounded to bf16,
//   bf16 matmul with v), reproduced operation for operation.
// Sliding-window caches are rings: position p lives in slot p % cap.
#include <cooperative_groups.h>
#include <stdlib.h>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace mlxd {

// ------------------------------------------------------------------ decode

MLXD_TRACE_BINDER(attention)

constexpr int DEC_THREADS = 256;
constexpr int DEC_MAX_SPLIT = 64;

template <int D, int REP>
__global__ void __launch_bounds__(DEC_THREADS, 2) attn_decode_kernel(AttnDecodeArgs a) {
    MLXD_TRACE_START
    constexpr int DL = D / 32;   // dims per lane
    constexpr int NW = DEC_THREADS / 32;
    constexpr int DEC_U = D == 128 ? 4 : 8;   // positions per warp per pass, loads in flight
    using RowT = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    __shared__ float s_vec[NW][D];
    __shared__ float s_q[REP][D];
    __shared__ __align__(16) uint16_t s_knew[D];
    __shared__ __align__(16) uint16_t s_vnew[D];
    __shared__ float s_m[NW][REP], s_l[NW][REP];
    __shared__ float s_o[NW][REP][D];
    __shared__ int s_last;

    const int kh = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The position counter and the cache rows of earlier positions were
    // written by earlier decode steps, so they are read before waiting on the
    // q/k/v projection of this step: the cache stream overlaps its tail.
    const int pos = *a.d_pos;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int span = T - lo;
    const int s0 = lo + (int)(((long long)span * split) / a.nsplit);
    const int s1 = lo + (int)(((long long)span * (split + 1)) / a.nsplit);
    const int per_warp = (s1 - s0 + NW - 1) / NW;
    const int w0 = s0 + warp * per_warp;
    const int w1 = min(s1, w0 + per_warp);
    const int slot_new = pos % a.cap;
    uint16_t *kc = a.kc + (size_t)kh * a.cap * D;
    uint16_t *vc = a.vc + (size_t)kh * a.cap * D;

    RowT kraw[DEC_U], vraw[DEC_U];
    auto fetch = [&](int j0) {
#pragma unroll
        for (int u = 0; u < DEC_U; u++) {
            int j = j0 + u;
            if (j < w1 && j != pos) {
                const size_t off = (size_t)(j % a.cap) * D + lane * DL;
                kraw[u] = *reinterpret_cast<const RowT *>(kc + off);
                vraw[u] = *reinterpret_cast<const RowT *>(vc + off);
            }
        }
    };
    fetch(w0);
    // the next kernel (the o projection) may start streaming its weights now
    pdl_trigger();

    pdl_wait();
    MLXD_TRACE_WAITED
    const uint16_t *qkv = a.qkv;
    const int qstride = D * (a.gate ? 2 : 1);
    // q heads of this GQA group, the new k (norm + rope) and the new v: one warp each
    for (int vi = warp; vi <= REP + 1; vi += NW) {
        if (vi == REP + 1) {
            for (int d = lane; d < D; d += 32) s_vnew[d] = qkv[a.qdim + (size_t)(a.hkv + kh) * D + d];
            continue;
        }
        float *v = s_vec[warp];
        const uint16_t *src = vi < REP ? qkv + (size_t)(kh * REP + vi) * qstride
                                       : qkv + a.qdim + (size_t)kh * D;
        for (int d = lane; d < D; d += 32) v[d] = bf2f(src[d]);
        __syncwarp();
        head_norm_rope(v, D, vi < REP ? a.qn : a.kn, a.eps, a.rope.cs, a.rope.rope_dims, pos);
        if (vi < REP) {
            for (int d = lane; d < D; d += 32) s_q[vi][d] = v[d];
        } else {
            for (int d = lane; d < D; d += 32) s_knew[d] = f2bf(v[d]);
        }
        __syncwarp();
    }
    __syncthreads();
    if (split == 0) {
        for (int d = threadIdx.x; d < D; d += DEC_THREADS) {
            kc[(size_t)slot_new * D + d] = s_knew[d];
            vc[(size_t)slot_new * D + d] = s_vnew[d];
        }
    }

    // q in registers, pre-scaled by 1/sqrt(D) * log2(e) for exp2
    const float qscale = rsqrtf((float)D) * 1.4426950408889634f;
    float q[REP][DL];
#pragma unroll
    for (int r = 0; r < REP; r++)
#pragma unroll
        for (int i = 0; i < DL; i++) q[r][i] = s_q[r][lane * DL + i] * qscale;

    float m[REP], l[REP], o[REP][DL];
#pragma unroll
    for (int r = 0; r < REP; r++) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; i++) o[r][i] = 0.f;
    }

    auto unpack = [&](const RowT &raw, float (&dst)[DL]) {
        if constexpr (DL == 4) {
            dst[0] = lo_bf(raw.x); dst[1] = hi_bf(raw.x); dst[2] = lo_bf(raw.y); dst[3] = hi_bf(raw.y);
        } else {
            dst[0] = lo_bf(raw); dst[1] = hi_bf(raw);
        }
    };
    const RowT *knew_row = reinterpret_cast<const RowT *>(s_knew + lane * DL);
    const RowT *vnew_row = reinterpret_cast<const RowT *>(s_vnew + lane * DL);

    for (int j0 = w0; j0 < w1; j0 += DEC_U) {
        if (j0 != w0) fetch(j0);
        float kr[DEC_U][DL], vr[DEC_U][DL];
#pragma unroll
        for (int u = 0; u < DEC_U; u++) {
            int j = j0 + u;
            RowT kk = kraw[u], vv = vraw[u];
            if (j == pos) {
                kk = *knew_row;
                vv = *vnew_row;
            }
            if (j < w1) {
                unpack(kk, kr[u]);
                unpack(vv, vr[u]);
            } else {
#pragma unroll
                for (int i = 0; i < DL; i++) kr[u][i] = vr[u][i] = 0.f;
            }
        }
        // U independent scores per head, then one online-softmax update
#pragma unroll
        for (int r = 0; r < REP; r++) {
            float sc[DEC_U];
#pragma unroll
            for (int u = 0; u < DEC_U; u++) {
                float x = 0.f;
#pragma unroll
                for (int i = 0; i < DL; i++) x = fmaf(q[r][i], kr[u][i], x);
                sc[u] = x;
            }
#pragma unroll
            for (int sh = 16; sh > 0; sh >>= 1)
#pragma unroll
                for (int u = 0; u < DEC_U; u++) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], sh);
            float mn = m[r];
#pragma unroll
            for (int u = 0; u < DEC_U; u++)
                if (j0 + u < w1) mn = fmaxf(mn, sc[u]);
            float alpha = exp2f(m[r] - mn);
            float ps = 0.f;
            float pu[DEC_U];
#pragma unroll
            for (int u = 0; u < DEC_U; u++) {
                pu[u] = (j0 + u < w1) ? exp2f(sc[u] - mn) : 0.f;
                ps += pu[u];
            }
            l[r] = l[r] * alpha + ps;
#pragma unroll
            for (int i = 0; i < DL; i++) {
                float acc = o[r][i] * alpha;
#pragma unroll
                for (int u = 0; u < DEC_U; u++) acc = fmaf(pu[u], vr[u][i], acc);
                o[r][i] = acc;
            }
            m[r] = mn;
        }
    }
    // merge the warps of this CTA
#pragma unroll
    for (int r = 0; r < REP; r++) {
        if (lane == 0) {
            s_m[warp][r] = m[r];
            s_l[warp][r] = l[r];
        }
#pragma unroll
        for (int i = 0; i < DL; i++) s_o[warp][r][lane * DL + i] = o[r][i];
    }
    __syncthreads();
    float *part = a.part;
    for (int idx = threadIdx.x; idx < REP * D; idx += DEC_THREADS) {
        int r = idx / D, d = idx % D;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) mx = fmaxf(mx, s_m[w][r]);
        float ls = 0.f, os = 0.f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            float e = (s_m[w][r] == -INFINITY) ? 0.f : exp2f(s_m[w][r] - mx);
            ls += s_l[w][r] * e;
            os += s_o[w][r][d] * e;
        }
        int h = kh * REP + r;
        float *rec = part + ((size_t)h * a.nsplit + split) * (D + 2);
        rec[2 + d] = os;
        if (d == 0) {
            rec[0] = mx;
            rec[1] = ls;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int old = atomicAdd(&a.count[kh], 1);
        s_last = (old == a.nsplit - 1);
    }
    __syncthreads();
    if (!s_last) {
        MLXD_TRACE_END(0x30)
        return;
    }

    __threadfence();
    // last split of this kv head: merge all splits. The (max, sum) pairs of
    // every split are loaded in parallel, one warp per q head turns them
    // into weights 2^(m_s - m) / L, then each output element is a dot
    // product over the splits with 32 independent loads in flight.
    __shared__ float s_w[REP][DEC_MAX_SPLIT];
    __shared__ float s_lw[REP][DEC_MAX_SPLIT];
    const int ns = a.nsplit;
    for (int idx = threadIdx.x; idx < REP * ns; idx += DEC_THREADS) {
        int r = idx / ns, sp = idx % ns;
        const float *rec = part + ((size_t)(kh * REP + r) * ns + sp) * (D + 2);
        s_w[r][sp] = __ldcg(rec);
        s_lw[r][sp] = __ldcg(rec + 1);
    }
    __syncthreads();
    for (int r = warp; r < REP; r += NW) {
        const float m0 = lane < ns ? s_w[r][lane] : -INFINITY;
        const float m1 = lane + 32 < ns ? s_w[r][lane + 32] : -INFINITY;
        const float mx = warp_max(fmaxf(m0, m1));
        const float w0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mx);
        const float w1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mx);
        const float L = warp_sum(fmaf(w0, lane < ns ? s_lw[r][lane] : 0.f,
                                      w1 * (lane + 32 < ns ? s_lw[r][lane + 32] : 0.f)));
        const float invL = 1.f / L;
        if (lane < ns) s_w[r][lane] = w0 * invL;
        if (lane + 32 < ns) s_w[r][lane + 32] = w1 * invL;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < REP * D; idx += DEC_THREADS) {
        int r = idx / D, d = idx % D;
        int h = kh * REP + r;
        const float *base = part + (size_t)h * ns * (D + 2) + 2 + d;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int sp0 = 0; sp0 < ns; sp0 += 32) {
            float v[32];
#pragma unroll
            for (int u = 0; u < 32; u++) v[u] = sp0 + u < ns ? __ldcg(base + (size_t)(sp0 + u) * (D + 2)) : 0.f;
#pragma unroll
            for (int u = 0; u < 32; u++)
                if (sp0 + u < ns) acc[u & 3] = fmaf(s_w[r][sp0 + u], v[u], acc[u & 3]);
        }
        float val = rbf((acc[0] + acc[1]) + (acc[2] + acc[3]));
        if (a.gate) {
            float gv = bf2f(qkv[(size_t)h * qstride + D + d]);
            val = rbf(__fmul_rn(val, sigmoid_bf16(gv)));
        }
        a.out[(size_t)h * D + d] = f2bf(val);
    }
    MLXD_TRACE_END(0x31)
    if (threadIdx.x == 0) a.count[kh] = 0;
}

template <int D>
static int launch_decode(const AttnDecodeArgs &a, int rep, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.hkv, a.nsplit);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (rep) {
    case 1: MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, 1>, a)); return 0;
    case 2: MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, 2>, a)); return 0;
    case 4: MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, 4>, a)); return 0;
    case 8: MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, 8>, a)); return 0;
    default: set_error("attention_decode: GQA ratio %d not supported", rep); return -1;
    }
}

// ------------------------------------------------- decode, cluster merge
//
// The same step with the splits of one kv head forming one thread-block
// cluster (CL CTAs of 16 warps): each CTA attends over its contiguous share
// of the positions, merges its warps in shared memory, and after a cluster
// barrier every CTA merges a slice of the head group's outputs from all CL
// CTAs' shared memory (distributed shared memory), so no partial sums go
// through global memory and no CTA waits for a last arriver.
constexpr int CL_THREADS = 512, CL_WARPS = 16, CL_PB = 4;
// opt-in (MLXD_ATTN_CLUSTER=1, read at each launch): on Qwen3-8B it runs as
// fast as the split-merge kernel, which stays the default
static bool attn_cluster_on() {
    const char *e = getenv("MLXD_ATTN_CLUSTER");
    return e && atoi(e) != 0;
}

template <int D, int REP>
__global__ void __launch_bounds__(CL_THREADS, 1) attn_decode_cluster_kernel(AttnDecodeArgs a) {
    MLXD_TRACE_START
    namespace cg = cooperative_groups;
    constexpr int DL = D / 32;
    using RowT = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    cg::cluster_group cluster = cg::this_cluster();
    const int CL = (int)cluster.num_blocks();
    const int split = (int)cluster.block_rank();
    const int kh = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float s_q[REP][D];
    __shared__ __align__(16) uint16_t s_knew[D];
    __shared__ __align__(16) uint16_t s_vnew[D];
    __shared__ float s_wml[8][REP][2];
    // the per-warp staging of the q/k vectors and, later, the warps' partial
    // outputs share one buffer
    constexpr int WO = 8 * REP * D > CL_WARPS * D ? 8 * REP * D : CL_WARPS * D;
    __shared__ __align__(16) float s_buf[WO];
    float (*s_vec)[D] = reinterpret_cast<float (*)[D]>(s_buf);
    float (*s_wo)[REP][D] = reinterpret_cast<float (*)[REP][D]>(s_buf);
    __shared__ float s_pm[REP], s_pl[REP];    // this CTA's merged partial
    __shared__ __align__(16) float s_po[REP][D];

    const int pos = *a.d_pos;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int span = T - lo;
    const int s0 = lo + (int)(((long long)span * split) / CL);
    const int s1 = lo + (int)(((long long)span * (split + 1)) / CL);
    const int nc = max(0, min(s1, pos) - s0);          // cached rows of this split
    const int per = (nc + CL_WARPS - 1) / CL_WARPS;
    const int w0 = s0 + warp * per, w1 = min(s0 + nc, w0 + per);
    const uint16_t *kc = a.kc + (size_t)kh * a.cap * D;
    const uint16_t *vc = a.vc + (size_t)kh * a.cap * D;

    // two batches of cached rows stream before the projection is waited for
    RowT kb[2][CL_PB], vb[2][CL_PB];
    auto fetch = [&](const int b, int j0) {
#pragma unroll
        for (int u = 0; u < CL_PB; u++) {
            const int j = min(j0 + u, w1 - 1);
            if (j >= w0) {
                const size_t off = (size_t)(j % a.cap) * D + lane * DL;
                if (b == 0) {
                    kb[0][u] = *reinterpret_cast<const RowT *>(kc + off);
                    vb[0][u] = *reinterpret_cast<const RowT *>(vc + off);
                } else {
                    kb[1][u] = *reinterpret_cast<const RowT *>(kc + off);
                    vb[1][u] = *reinterpret_cast<const RowT *>(vc + off);
                }
            }
        }
    };
    fetch(0, w0);
    fetch(1, w0 + CL_PB);
    pdl_trigger();
    pdl_wait();
    MLXD_TRACE_WAITED

    const uint16_t *qkv = a.qkv;
    const int qstride = D * (a.gate ? 2 : 1);
    for (int vi = warp; vi < REP + 2; vi += CL_WARPS) {
        if (vi == REP + 1) {
            for (int d = lane; d < D; d += 32) s_vnew[d] = qkv[a.qdim + (size_t)(a.hkv + kh) * D + d];
            continue;
        }
        float *v = s_vec[warp];
        const uint16_t *src = vi < REP ? qkv + (size_t)(kh * REP + vi) * qstride : qkv + a.qdim + (size_t)kh * D;
        for (int d = lane; d < D; d += 32) v[d] = bf2f(src[d]);
        __syncwarp();
        head_norm_rope(v, D, vi < REP ? a.qn : a.kn, a.eps, a.rope.cs, a.rope.rope_dims, pos);
        if (vi < REP) {
            for (int d = lane; d < D; d += 32) s_q[vi][d] = v[d];
        } else {
            for (int d = lane; d < D; d += 32) s_knew[d] = f2bf(v[d]);
        }
        __syncwarp();
    }
    __syncthreads();
    if (split == 0) {
        for (int d = tid; d < D; d += CL_THREADS) {
            const size_t off = (size_t)(pos % a.cap) * D + d;
            const_cast<uint16_t *>(kc)[off] = s_knew[d];
            const_cast<uint16_t *>(vc)[off] = s_vnew[d];
        }
    }

    const float qscale = rsqrtf((float)D) * 1.4426950408889634f;
    float q[REP][DL], m[REP], lsum[REP], o[REP][DL];
#pragma unroll
    for (int r = 0; r < REP; r++) {
        m[r] = -INFINITY;
        lsum[r] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; i++) {
            q[r][i] = s_q[r][lane * DL + i] * qscale;
            o[r][i] = 0.f;
        }
    }
    auto unpack = [&](const RowT &raw, float (&dst)[DL]) {
        if constexpr (DL == 4) {
            dst[0] = lo_bf(raw.x); dst[1] = hi_bf(raw.x); dst[2] = lo_bf(raw.y); dst[3] = hi_bf(raw.y);
        } else {
            dst[0] = lo_bf(raw); dst[1] = hi_bf(raw);
        }
    };
    // nv (<= CL_PB) positions: independent scores, one reduction pass, one
    // online-softmax update per head
    auto visit = [&](const RowT (&kr)[CL_PB], const RowT (&vr)[CL_PB], int nv) {
        float sc[REP][CL_PB];
#pragma unroll
        for (int u = 0; u < CL_PB; u++) {
            float kf[DL];
            unpack(kr[u], kf);
#pragma unroll
            for (int r = 0; r < REP; r++) {
                float x = 0.f;
#pragma unroll
                for (int i = 0; i < DL; i++) x = fmaf(q[r][i], kf[i], x);
                sc[r][u] = x;
            }
        }
#pragma unroll
        for (int sh = 16; sh > 0; sh >>= 1)
#pragma unroll
            for (int r = 0; r < REP; r++)
#pragma unroll
                for (int u = 0; u < CL_PB; u++) sc[r][u] += __shfl_xor_sync(0xffffffffu, sc[r][u], sh);
#pragma unroll
        for (int r = 0; r < REP; r++) {
            float mn = m[r];
#pragma unroll
            for (int u = 0; u < CL_PB; u++)
                if (u < nv) mn = fmaxf(mn, sc[r][u]);
            const float al = exp2f(m[r] - mn);
            float ps = 0.f;
#pragma unroll
            for (int u = 0; u < CL_PB; u++) {
                sc[r][u] = u < nv ? exp2f(sc[r][u] - mn) : 0.f;
                ps += sc[r][u];
            }
            lsum[r] = lsum[r] * al + ps;
#pragma unroll
            for (int i = 0; i < DL; i++) o[r][i] *= al;
            m[r] = mn;
        }
#pragma unroll
        for (int u = 0; u < CL_PB; u++) {
            float vf[DL];
            unpack(vr[u], vf);
#pragma unroll
            for (int r = 0; r < REP; r++)
#pragma unroll
                for (int i = 0; i < DL; i++) o[r][i] = fmaf(sc[r][u], vf[i], o[r][i]);
        }
    };
    // the batch index stays a compile-time constant (registers, not local memory)
    auto step = [&](auto bc, int j0) {
        constexpr int B = decltype(bc)::value;
        RowT kr[CL_PB], vr[CL_PB];
#pragma unroll
        for (int u = 0; u < CL_PB; u++) {
            kr[u] = kb[B][u];
            vr[u] = vb[B][u];
        }
        if (j0 + 2 * CL_PB < w1) fetch(B, j0 + 2 * CL_PB);
        visit(kr, vr, min(CL_PB, w1 - j0));
    };
    for (int j0 = w0; j0 < w1; j0 += 2 * CL_PB) {
        step(std::integral_constant<int, 0>(), j0);
        if (j0 + CL_PB < w1) step(std::integral_constant<int, 1>(), j0 + CL_PB);
    }
    // the new position (its row came from this step's projection)
    if (warp == CL_WARPS - 1 && pos >= s0 && pos < s1) {
        RowT kr[CL_PB], vr[CL_PB];
#pragma unroll
        for (int u = 0; u < CL_PB; u++) {
            kr[u] = *reinterpret_cast<const RowT *>(s_knew + lane * DL);
            vr[u] = *reinterpret_cast<const RowT *>(s_vnew + lane * DL);
        }
        visit(kr, vr, 1);
    }
    // warps 8..15 hand their state to warps 0..7, which write theirs
    auto put = [&](int w) {
#pragma unroll
        for (int r = 0; r < REP; r++) {
            if (lane == 0) {
                s_wml[w][r][0] = m[r];
                s_wml[w][r][1] = lsum[r];
            }
#pragma unroll
            for (int i = 0; i < DL; i++) s_wo[w][r][lane * DL + i] = o[r][i];
        }
    };
    if (warp >= 8) put(warp - 8);
    __syncthreads();
    if (warp < 8) {
#pragma unroll
        for (int r = 0; r < REP; r++) {
            const float m2 = s_wml[warp][r][0], l2 = s_wml[warp][r][1];
            const float mx = fmaxf(m[r], m2);
            if (mx != -INFINITY) {
                const float wa = m[r] == -INFINITY ? 0.f : exp2f(m[r] - mx);
                const float wb = m2 == -INFINITY ? 0.f : exp2f(m2 - mx);
#pragma unroll
                for (int i = 0; i < DL; i++) o[r][i] = o[r][i] * wa + s_wo[warp][r][lane * DL + i] * wb;
                lsum[r] = lsum[r] * wa + l2 * wb;
                m[r] = mx;
            }
        }
    }
    __syncthreads();
    if (warp < 8) put(warp);
    __syncthreads();
    for (int idx = tid; idx < REP * D; idx += CL_THREADS) {
        const int r = idx / D, d = idx % D;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; w++) mx = fmaxf(mx, s_wml[w][r][0]);
        float ls = 0.f, os = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const float e = s_wml[w][r][0] == -INFINITY ? 0.f : exp2f(s_wml[w][r][0] - mx);
            ls += s_wml[w][r][1] * e;
            os += s_wo[w][r][d] * e;
        }
        s_po[r][d] = os;
        if (d == 0) {
            s_pm[r] = mx;
            s_pl[r] = ls;
        }
    }
    cluster.sync();
    // this CTA's slice of the head group's outputs, from every CTA's partial
    const int n_out = REP * D;
    const int o0 = (int)(((long long)n_out * split) / CL), o1 = (int)(((long long)n_out * (split + 1)) / CL);
    const int lanes_per = 16;                       // splits handled per output, one per lane
    for (int base_o = o0; base_o < o1; base_o += CL_THREADS / lanes_per) {
        const int oi = base_o + tid / lanes_per, sub = tid % lanes_per;
        float mm = -INFINITY, ll = 0.f, oo = 0.f;
        if (oi < o1) {
            const int r = oi / D, d = oi % D;
            for (int sp = sub; sp < CL; sp += lanes_per) {
                const float pm = *cluster.map_shared_rank(&s_pm[r], sp);
                const float pl = *cluster.map_shared_rank(&s_pl[r], sp);
                const float po = *cluster.map_shared_rank(&s_po[r][d], sp);
                const float mx = fmaxf(mm, pm);
                if (mx != -INFINITY) {
                    const float wa = mm == -INFINITY ? 0.f : exp2f(mm - mx);
                    const float wb = pm == -INFINITY ? 0.f : exp2f(pm - mx);
                    ll = ll * wa + pl * wb;
                    oo = oo * wa + po * wb;
                    mm = mx;
                }
            }
        }
#pragma unroll
        for (int sh = 1; sh < lanes_per; sh <<= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, mm, sh);
            const float l2 = __shfl_xor_sync(0xffffffffu, ll, sh);
            const float o2 = __shfl_xor_sync(0xffffffffu, oo, sh);
            const float mx = fmaxf(mm, m2);
            if (mx != -INFINITY) {
                const float wa = mm == -INFINITY ? 0.f : exp2f(mm - mx);
                const float wb = m2 == -INFINITY ? 0.f : exp2f(m2 - mx);
                ll = ll * wa + l2 * wb;
                oo = oo * wa + o2 * wb;
                mm = mx;
            }
        }
        if (oi < o1 && sub == 0) {
            const int r = oi / D, d = oi % D;
            const int h = kh * REP + r;
            float val = rbf(oo / ll);
            if (a.gate) {
                const float gv = bf2f(qkv[(size_t)h * qstride + D + d]);
                val = rbf(__fmul_rn(val, sigmoid_bf16(gv)));
            }
            a.out[(size_t)h * D + d] = f2bf(val);
        }
    }
    // every CTA's shared memory stays until all slices are read
    cluster.sync();
    MLXD_TRACE_END(0x32)
}

template <int D, int REP>
static int launch_decode_cluster(const AttnDecodeArgs &a, int cl, cudaStream_t st, bool pdl) {
    auto kern = attn_decode_cluster_kernel<D, REP>;
    static bool configured = false;
    if (!configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, a.hkv);
    cfg.blockDim = dim3(CL_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
    return 0;
}

// cluster size for a head group: 16 CTAs when the device schedules eight of
// those clusters at once, else 8; 0 when no cluster fits (split-merge runs)
template <int D, int REP>
static int cluster_size(int hkv) {
    static int cached = -1;
    if (cached < 0) {
        cached = 0;
        auto kern = attn_decode_cluster_kernel<D, REP>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        for (int cl : {16, 8}) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(cl, 8);
            cfg.blockDim = dim3(CL_THREADS);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = cl;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n >= 8) {
                cached = cl;
                break;
            }
        }
        cudaGetLastError();
    }
    (void)hkv;
    return cached;
}

template <int D>
static int decode_cluster_any(const AttnDecodeArgs &a, int rep, cudaStream_t st, bool pdl) {
    int cl = 0;
    switch (rep) {
    case 1: cl = cluster_size<D, 1>(a.hkv); return cl ? launch_decode_cluster<D, 1>(a, cl, st, pdl) : 1;
    case 2: cl = cluster_size<D, 2>(a.hkv); return cl ? launch_decode_cluster<D, 2>(a, cl, st, pdl) : 1;
    case 4: cl = cluster_size<D, 4>(a.hkv); return cl ? launch_decode_cluster<D, 4>(a, cl, st, pdl) : 1;
    case 8: cl = cluster_size<D, 8>(a.hkv); return cl ? launch_decode_cluster<D, 8>(a, cl, st, pdl) : 1;
    default: return 1;
    }
}

int attention_decode(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    int rep = a.hq / a.hkv;
    int D = a.rope.D;
    if (attn_cluster_on()) {
        // 1: no cluster configuration fits; the split-merge kernel runs
        int rc = D == 128 ? decode_cluster_any<128>(a, rep, st, pdl)
                          : D == 64 ? decode_cluster_any<64>(a, rep, st, pdl) : 1;
        if (rc <= 0) return rc;
    }
    if (D == 128) return launch_decode<128>(a, rep, st, pdl);
    if (D == 64) return launch_decode<64>(a, rep, st, pdl);
    set_error("attention_decode: head_dim %d not supported", D);
    return -1;
}

// ------------------------------------------------------------------ prefill

constexpr int PF_BR = 64, PF_BC = 64, PF_THREADS = 128;

template <int D>
__global__ void __launch_bounds__(PF_THREADS) attn_prefill_kernel(
    const uint16_t *__restrict__ q, int S, int pos0, const uint16_t *__restrict__ kc,
    const uint16_t *__restrict__ vc, int cap, int window, int hq, int hkv,
    const uint16_t *__restrict__ gate_src, int qdim, int row_stride, uint16_t *__restrict__ out) {
    constexpr int LD = D + 8;   // padded row (bank-conflict-free ldmatrix)
    extern __shared__ __align__(16) uint16_t sm[];
    uint16_t *sQ = sm;
    uint16_t *sK = sQ + PF_BR * LD;
    uint16_t *sV = sK + PF_BC * LD;
    const int qt = blockIdx.x, h = blockIdx.y, kh = h / (hq / hkv);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int q0 = qt * PF_BR;
    const int nq = min(PF_BR, S - q0);
    const uint16_t *kbase = kc + (size_t)kh * cap * D;
    const uint16_t *vbase = vc + (size_t)kh * cap * D;

    // Q tile
    for (int c = tid; c < PF_BR * (D / 8); c += PF_THREADS) {
        int r = c / (D / 8), cc = c % (D / 8);
        bool ok = r < nq;
        const uint16_t *src = q + ((size_t)(q0 + (ok ? r : 0)) * hq + h) * D + cc * 8;
        cp_async16_zfill(sQ + r * LD + cc * 8, src, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    uint32_t qf[D / 16][4];
#pragma unroll
    for (int kk = 0; kk < D / 16; kk++) {
        int r = warp * 16 + (lane & 15);
        int c = kk * 16 + (lane >> 4) * 8;
        ldmatrix_x4(qf[kk], sQ + r * LD + c);
    }

    const float sl2 = rsqrtf((float)D) * 1.4426950408889634f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    float oacc[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; n++) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;

    const int qp_lo = pos0 + q0, qp_hi = pos0 + q0 + nq - 1;   // absolute positions
    int klo = 0;
    if (window > 0) klo = max(0, qp_lo - window + 1);
    const int khi = qp_hi + 1;
    const int my_r0 = q0 + warp * 16 + g, my_r1 = my_r0 + 8;
    const int my_p0 = pos0 + my_r0, my_p1 = pos0 + my_r1;

    for (int kb = klo; kb < khi; kb += PF_BC) {
        int nk = min(PF_BC, khi - kb);
        __syncthreads();
        for (int c = tid; c < PF_BC * (D / 8); c += PF_THREADS) {
            int r = c / (D / 8), cc = c % (D / 8);
            bool ok = r < nk;
            size_t slot = (size_t)((kb + (ok ? r : 0)) % cap);
            cp_async16_zfill(sK + r * LD + cc * 8, kbase + slot * D + cc * 8, ok);
            cp_async16_zfill(sV + r * LD + cc * 8, vbase + slot * D + cc * 8, ok);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        // S = Q K^T (16 x 64 per warp)
        float sacc[PF_BC / 8][4];
#pragma unroll
        for (int n = 0; n < PF_BC / 8; n++) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < D / 16; kk++) {
#pragma unroll
            for (int n = 0; n < PF_BC / 8; n += 2) {
                uint32_t b[4];
                int r = n * 8 + (lane & 7) + ((lane >> 4) << 3);
                int c = kk * 16 + ((lane >> 3) & 1) * 8;
                ldmatrix_x4(b, sK + r * LD + c);
                mma_bf16_16816(sacc[n], qf[kk], b[0], b[1]);
                mma_bf16_16816(sacc[n + 1], qf[kk], b[2], b[3]);
            }
        }
        // mask + online softmax
        float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int n = 0; n < PF_BC / 8; n++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                int kp = kb + n * 8 + 2 * t + (e & 1);
                int qp = (e < 2) ? my_p0 : my_p1;
                int qr = (e < 2) ? my_r0 : my_r1;
                bool ok = (kp - kb) < nk && kp <= qp && qr < S && (window <= 0 || qp - kp < window);
                float v = ok ? sacc[n][e] * sl2 : -INFINITY;
                sacc[n][e] = v;
                mnew[e >> 1] = fmaxf(mnew[e >> 1], v);
            }
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            mnew[i] = fmaxf(mnew[i], __shfl_xor_sync(0xffffffffu, mnew[i], 1));
            mnew[i] = fmaxf(mnew[i], __shfl_xor_sync(0xffffffffu, mnew[i], 2));
        }
        float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 2; i++) alpha[i] = (mnew[i] == -INFINITY) ? 1.f : exp2f(mrow[i] - mnew[i]);
        // P split as bf16 hi + bf16 lo so P.V keeps ~16 mantissa bits of the
        // f32 probabilities (mlx keeps P in f32 for the product)
        uint32_t pf[PF_BC / 16][4], pl[PF_BC / 16][4];
#pragma unroll
        for (int n = 0; n < PF_BC / 8; n++) {
            float p[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float mm = mnew[e >> 1];
                p[e] = (mm == -INFINITY) ? 0.f : exp2f(sacc[n][e] - mm);
                rs[e >> 1] += p[e];
                lo[e] = p[e] - rbf(p[e]);
            }
            int kk = n >> 1;
            int o = (n & 1) * 2;
            pf[kk][o] = pack_bf2(p[0], p[1]);
            pf[kk][o + 1] = pack_bf2(p[2], p[3]);
            pl[kk][o] = pack_bf2(lo[0], lo[1]);
            pl[kk][o + 1] = pack_bf2(lo[2], lo[3]);
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
            rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
            lrow[i] = lrow[i] * alpha[i] + rs[i];
            mrow[i] = mnew[i];
        }
#pragma unroll
        for (int n = 0; n < D / 8; n++) {
            oacc[n][0] *= alpha[0];
            oacc[n][1] *= alpha[0];
            oacc[n][2] *= alpha[1];
            oacc[n][3] *= alpha[1];
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < PF_BC / 16; kk++) {
#pragma unroll
            for (int n = 0; n < D / 8; n += 2) {
                uint32_t b[4];
                int r = kk * 16 + (lane & 15);
                int c = n * 8 + (lane >> 4) * 8;
                ldmatrix_x4_trans(b, sV + r * LD + c);
                mma_bf16_16816(oacc[n], pf[kk], b[0], b[1]);
                mma_bf16_16816(oacc[n + 1], pf[kk], b[2], b[3]);
                mma_bf16_16816(oacc[n], pl[kk], b[0], b[1]);
                mma_bf16_16816(oacc[n + 1], pl[kk], b[2], b[3]);
            }
        }
    }
    // epilogue: O / l, optional qwen3_5 gate, bf16 out [S][hq][D]
#pragma unroll
    for (int i = 0; i < 2; i++) {
        int qr = (i == 0) ? my_r0 : my_r1;
        if (qr >= S) continue;
        float inv = lrow[i] > 0.f ? 1.f / lrow[i] : 0.f;
        uint16_t *dst = out + ((size_t)qr * hq + h) * D;
        const uint16_t *gp = gate_src ? gate_src + (size_t)qr * row_stride + (size_t)h * 2 * D + D : nullptr;
#pragma unroll
        for (int n = 0; n < D / 8; n++) {
            int c = n * 8 + 2 * t;
            float v0 = rbf(oacc[n][2 * i] * inv), v1 = rbf(oacc[n][2 * i + 1] * inv);
            if (gp) {
                v0 = rbf(__fmul_rn(v0, sigmoid_bf16(bf2f(gp[c]))));
                v1 = rbf(__fmul_rn(v1, sigmoid_bf16(bf2f(gp[c + 1]))));
            }
            *reinterpret_cast<uint32_t *>(dst + c) = pack_bf2(v0, v1);
        }
    }
}

// ------------------------------------------------------------ small head dims
// mlx composed fallback, exact order: one warp per (query, head).
__global__ void attn_small_kernel(const uint16_t *__restrict__ q, int S, int pos0,
                                  const uint16_t *__restrict__ kc, const uint16_t *__restrict__ vc,
                                  int cap, int window, int hq, int hkv, int D,
                                  const uint16_t *__restrict__ gate_src, int row_stride,
                                  uint16_t *__restrict__ out, float *scratch, int tmax) {
    int i = blockIdx.x, h = blockIdx.y, kh = h / (hq / hkv), lane = threadIdx.x;
    float *sc = scratch + ((size_t)i * hq + h) * tmax;
    int qp = pos0 + i;
    int T = qp + 1;
    int j0 = 0;
    if (window > 0) {
        if (S == 1) j0 = max(0, T - window);
        else j0 = max(0, qp - window + 1);
    }
    const uint16_t *qv = q + ((size_t)i * hq + h) * D;
    const uint16_t *K = kc + (size_t)kh * cap * D;
    const uint16_t *V = vc + (size_t)kh * cap * D;
    float sbf = rbf(rsqrtf((float)D));
    for (int j = j0 + lane; j < T; j += 32) {
        float a = 0.f;
        for (int d = 0; d < D; d++) {
            float qs = rbf(__fmul_rn(sbf, bf2f(qv[d])));
            a = __fadd_rn(a, __fmul_rn(qs, bf2f(K[(size_t)(j % cap) * D + d])));
        }
        sc[j - j0] = rbf(a);
    }
    __syncwarp();
    float mx = -INFINITY;
    for (int j = lane; j < T - j0; j += 32) mx = fmaxf(mx, sc[j]);
    mx = warp_max(mx);
    for (int j = lane; j < T - j0; j += 32) sc[j] = own_expf(__fsub_rn(sc[j], mx));
    __syncwarp();
    float l = 0.f;
    for (int j = 0; j < T - j0; j++) l = __fadd_rn(l, sc[j]);
    for (int d = lane; d < D; d += 32) {
        float o = 0.f;
        for (int j = 0; j < T - j0; j++) {
            float p = rbf(__fdiv_rn(sc[j], l));
            o = __fadd_rn(o, __fmul_rn(p, bf2f(V[(size_t)((j0 + j) % cap) * D + d])));
        }
        float val = rbf(o);
        if (gate_src) {
            float g = bf2f(gate_src[(size_t)i * row_stride + (size_t)h * 2 * D + D + d]);
            val = rbf(__fmul_rn(val, sigmoid_bf16(g)));
        }
        out[((size_t)i * hq + h) * D + d] = f2bf(val);
    }
}

int attention_prefill(const uint16_t *q, int S, int pos0, const uint16_t *kc, const uint16_t *vc,
                      int cap, int window, int hq, int hkv, int D, const uint16_t *gate_src,
                      int qdim, uint16_t *out, cudaStream_t st) {
    int row_stride = qdim + 2 * hkv * D;
    if (D == 64 || D == 128) {
        size_t smem = (size_t)(PF_BR + 2 * PF_BC) * (D + 8) * 2;
        dim3 grid((S + PF_BR - 1) / PF_BR, hq);
        if (D == 128) {
            static bool set = false;
            if (!set) {
                MLXD_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<128>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                set = true;
            }
            attn_prefill_kernel<128><<<grid, PF_THREADS, smem, st>>>(
                q, S, pos0, kc, vc, cap, window, hq, hkv, gate_src, qdim, row_stride, out);
        } else {
            attn_prefill_kernel<64><<<grid, PF_THREADS, smem, st>>>(
                q, S, pos0, kc, vc, cap, window, hq, hkv, gate_src, qdim, row_stride, out);
        }
        MLXD_CHECK(cudaGetLastError());
        return 0;
    }
    // composed path: scratch for the scores of every (query, head)
    int tmax = pos0 + S;
    if (window > 0 && tmax > window + S) tmax = window + S;
    size_t need = (size_t)S * hq * tmax * sizeof(float);
    static float *scr = nullptr;
    static size_t scr_bytes = 0;
    if (need > scr_bytes) {
        if (scr) dev_free(scr);
        scr = (float *)dev_alloc(need);
        if (!scr) return -1;
        scr_bytes = need;
    }
    dim3 grid(S, hq);
    attn_small_kernel<<<grid, 32, 0, st>>>(q, S, pos0, kc, vc, cap, window, hq, hkv, D, gate_src,
                                           row_stride, out, scr, tmax);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace mlxd
