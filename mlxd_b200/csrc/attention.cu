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
constexpr int DEC_CH = 32;     // cached positions per shared-memory chunk
constexpr int DEC_PB = 4;      // positions scored together by one warp

template <int D>
static constexpr size_t dec_smem_bytes() { return (size_t)2 * 2 * DEC_CH * D * 2; }

// One new token, split-KV over (kv head, split) CTAs of 8 warps. Before
// griddepcontrol.wait, i.e. while the q|k|v projection still runs, each CTA
// requests its first two chunks of cached K/V rows into shared memory
// (cp.async; the rows of earlier positions do not depend on this step) and
// loads the q/k norm weights and the position's cos/sin row. After the wait
// it normalises and rotates q and k (fwd_attention :591-697), split 0 appends
// the new K/V row, and the warps score the chunk rows from shared memory (4
// positions per warp per pass, one online-softmax update per pass). The CTA's
// warps are merged in shared memory, the split's (max, sum, o) goes to a
// scratch buffer and the last CTA of a kv head (atomic counter) merges all
// splits with every load of a pass in flight at once.
template <int D, int REP>
__global__ void __launch_bounds__(DEC_THREADS, 2) attn_decode_kernel(AttnDecodeArgs a) {
    MLXD_TRACE_START
    constexpr int DL = D / 32;   // dims per lane
    constexpr int NW = DEC_THREADS / 32;
    using RowT = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    extern __shared__ __align__(16) unsigned char dec_smem[];   // [2 chunks][K|V][DEC_CH][D] bf16
    __shared__ float s_vec[NW][D];
    __shared__ float s_q[REP][D];
    __shared__ float s_nw[2][D];          // q and k norm weights
    __shared__ float s_cs[D];             // cos/sin of the position (rope_dims/2 pairs)
    __shared__ __align__(16) uint16_t s_knew[D];
    __shared__ __align__(16) uint16_t s_vnew[D];
    __shared__ float s_m[NW][REP], s_l[NW][REP];
    __shared__ float s_o[NW][REP][D];
    __shared__ float s_w[REP][DEC_MAX_SPLIT];
    __shared__ float s_lw[REP][DEC_MAX_SPLIT];
    __shared__ int s_last;

    const int kh = blockIdx.x, split = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = *a.d_pos;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int span = T - lo;
    const int s0 = lo + (int)(((long long)span * split) / a.nsplit);
    const int s1 = lo + (int)(((long long)span * (split + 1)) / a.nsplit);
    const int nc = max(0, min(s1, pos) - s0);    // cached rows of this split
    const int nchunks = (nc + DEC_CH - 1) / DEC_CH;
    const int slot_new = pos % a.cap;
    uint16_t *kc = a.kc + (size_t)kh * a.cap * D;
    uint16_t *vc = a.vc + (size_t)kh * a.cap * D;

    // chunk c of the split's cached rows into buffer c & 1 (16 bytes per copy)
    constexpr int RV = D / 8;                  // 16-byte vectors per row
    auto issue = [&](int c) {
        uint16_t *buf = reinterpret_cast<uint16_t *>(dec_smem) + (size_t)(c & 1) * 2 * DEC_CH * D;
        const int j0 = s0 + c * DEC_CH;
        const int n = min(DEC_CH, nc - c * DEC_CH);
        for (int i = tid; i < 2 * n * RV; i += DEC_THREADS) {
            const int kv = i / (n * RV), rem = i - kv * n * RV, r = rem / RV, v = rem - r * RV;
            const uint16_t *src = (kv ? vc : kc) + (size_t)((j0 + r) % a.cap) * D + v * 8;
            cp_async16(buf + ((size_t)kv * DEC_CH + r) * D + v * 8, src);
        }
        cp_async_commit();
    };
    issue(0);
    issue(1);
    l2_prefetch_share(a.pf);
    // norm weights and the rotation row are fixed for this step
    {
        const int half = a.rope.rope_dims / 2;
        const float *cs = a.rope.cs + (size_t)pos * half * 2;
        for (int i = tid; i < D; i += DEC_THREADS) {
            s_nw[0][i] = a.qn ? bf2f(a.qn[i]) : 1.f;
            s_nw[1][i] = a.kn ? bf2f(a.kn[i]) : 1.f;
            if (i < 2 * half) s_cs[i] = cs[i];
        }
    }
    pdl_trigger();
    pdl_wait();
    MLXD_TRACE_WAITED
    const uint16_t *qkv = a.qkv;
    const int qstride = D * (a.gate ? 2 : 1);
    const bool norm = a.qn != nullptr;
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
        // head_norm_rope with the staged weights and row: same arithmetic
        if (norm) {
            float acc = 0.f;
            for (int d = lane; d < D; d += 32) acc = fmaf(v[d], v[d], acc);
            acc = warp_sum(acc);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), a.eps)));
            __syncwarp();
            const float *nw = s_nw[vi < REP ? 0 : 1];
            for (int d = lane; d < D; d += 32) v[d] = rbf(__fmul_rn(nw[d], rbf(__fmul_rn(v[d], inv))));
            __syncwarp();
        }
        {
            const int half = a.rope.rope_dims / 2;
            float ra[4], rb[4];
            int cnt = 0;
            for (int i = lane; i < half; i += 32, cnt++) {
                const float x1 = v[i], x2 = v[i + half];
                const float co = s_cs[2 * i], si = s_cs[2 * i + 1];
                ra[cnt] = rbf(__fsub_rn(__fmul_rn(x1, co), __fmul_rn(x2, si)));
                rb[cnt] = rbf(__fadd_rn(__fmul_rn(x1, si), __fmul_rn(x2, co)));
            }
            __syncwarp();
            cnt = 0;
            for (int i = lane; i < half; i += 32, cnt++) {
                v[i] = ra[cnt];
                v[i + half] = rb[cnt];
            }
            __syncwarp();
        }
        if (vi < REP) {
            for (int d = lane; d < D; d += 32) s_q[vi][d] = v[d];
        } else {
            for (int d = lane; d < D; d += 32) s_knew[d] = f2bf(v[d]);
        }
        __syncwarp();
    }
    __syncthreads();
#ifdef MLXD_TRACE
    const unsigned long long tr_prep_ = gtime();
#endif
    if (split == 0) {
        for (int d = tid; d < D; d += DEC_THREADS) {
            kc[(size_t)slot_new * D + d] = s_knew[d];
            vc[(size_t)slot_new * D + d] = s_vnew[d];
        }
    }

    // q in registers, pre-scaled by 1/sqrt(D) * log2(e) for exp2
    const float qscale = rsqrtf((float)D) * 1.4426950408889634f;
    float q[REP][DL], m[REP], l[REP], o[REP][DL];
#pragma unroll
    for (int r = 0; r < REP; r++) {
        m[r] = -INFINITY;
        l[r] = 0.f;
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
    // nv (<= DEC_PB) rows: independent scores, one reduction pass, one
    // online-softmax update per head
    auto visit = [&](const RowT (&kr)[DEC_PB], const RowT (&vr)[DEC_PB], int nv) {
        float sc[REP][DEC_PB];
#pragma unroll
        for (int u = 0; u < DEC_PB; u++) {
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
                for (int u = 0; u < DEC_PB; u++) sc[r][u] += __shfl_xor_sync(0xffffffffu, sc[r][u], sh);
#pragma unroll
        for (int r = 0; r < REP; r++) {
            float mn = m[r];
#pragma unroll
            for (int u = 0; u < DEC_PB; u++)
                if (u < nv) mn = fmaxf(mn, sc[r][u]);
            const float al = exp2f(m[r] - mn);
            float ps = 0.f;
#pragma unroll
            for (int u = 0; u < DEC_PB; u++) {
                sc[r][u] = u < nv ? exp2f(sc[r][u] - mn) : 0.f;
                ps += sc[r][u];
            }
            l[r] = l[r] * al + ps;
#pragma unroll
            for (int i = 0; i < DL; i++) o[r][i] *= al;
            m[r] = mn;
        }
#pragma unroll
        for (int u = 0; u < DEC_PB; u++) {
            float vf[DL];
            unpack(vr[u], vf);
#pragma unroll
            for (int r = 0; r < REP; r++)
#pragma unroll
                for (int i = 0; i < DL; i++) o[r][i] = fmaf(sc[r][u], vf[i], o[r][i]);
        }
    };
    for (int c = 0; c < nchunks; c++) {
        cp_async_wait<1>();
        __syncthreads();
        const uint16_t *buf = reinterpret_cast<const uint16_t *>(dec_smem) + (size_t)(c & 1) * 2 * DEC_CH * D;
        const int n = min(DEC_CH, nc - c * DEC_CH);
        const int r0 = warp * DEC_PB;
        if (r0 < n) {
            RowT kr[DEC_PB], vr[DEC_PB];
#pragma unroll
            for (int u = 0; u < DEC_PB; u++) {
                const int r = min(r0 + u, n - 1);
                kr[u] = *reinterpret_cast<const RowT *>(buf + (size_t)r * D + lane * DL);
                vr[u] = *reinterpret_cast<const RowT *>(buf + (size_t)(DEC_CH + r) * D + lane * DL);
            }
            visit(kr, vr, min(DEC_PB, n - r0));
        }
        __syncthreads();
        if (c + 2 < nchunks) issue(c + 2);
        else cp_async_commit();
    }
    // the new position (its row came from this step's projection)
    if (warp == 0 && pos >= s0 && pos < s1) {
        RowT kr[DEC_PB], vr[DEC_PB];
#pragma unroll
        for (int u = 0; u < DEC_PB; u++) {
            kr[u] = *reinterpret_cast<const RowT *>(s_knew + lane * DL);
            vr[u] = *reinterpret_cast<const RowT *>(s_vnew + lane * DL);
        }
        visit(kr, vr, 1);
    }
#ifdef MLXD_TRACE
    const unsigned long long tr_loop_ = gtime();
#endif
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
    for (int idx = tid; idx < REP * D; idx += DEC_THREADS) {
        const int r = idx / D, d = idx % D;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) mx = fmaxf(mx, s_m[w][r]);
        float ls = 0.f, os = 0.f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float e = (s_m[w][r] == -INFINITY) ? 0.f : exp2f(s_m[w][r] - mx);
            ls += s_l[w][r] * e;
            os += s_o[w][r][d] * e;
        }
        const int h = kh * REP + r;
        float *rec = part + ((size_t)h * a.nsplit + split) * (D + 2);
        rec[2 + d] = os;
        if (d == 0) {
            rec[0] = mx;
            rec[1] = ls;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const int old = atomicAdd(&a.count[kh], 1);
        s_last = (old == a.nsplit - 1);
    }
    __syncthreads();
    MLXD_TRACE_REC(tid == 0, 0x38 + s_last, tr_prep_, tr_loop_, gtime())
    if (!s_last) {
        MLXD_TRACE_END(0x30)
        return;
    }
    __threadfence();
    // last split of this kv head: merge all splits. The (max, sum) pairs of
    // every split are loaded in parallel, one warp per q head turns them
    // into weights 2^(m_s - m) / L, then each output element is a dot
    // product over the splits with all of its loads in flight at once.
    const int ns = a.nsplit;
    for (int idx = tid; idx < REP * ns; idx += DEC_THREADS) {
        const int r = idx / ns, sp = idx % ns;
        const float *rec = part + ((size_t)(kh * REP + r) * ns + sp) * (D + 2);
        s_w[r][sp] = __ldcg(rec);
        s_lw[r][sp] = __ldcg(rec + 1);
    }
    __syncthreads();
    for (int r = warp; r < REP; r += NW) {
        const float *sl = s_lw[r];
        const float m0 = lane < ns ? s_w[r][lane] : -INFINITY;
        const float m1 = lane + 32 < ns ? s_w[r][lane + 32] : -INFINITY;
        const float mx = warp_max(fmaxf(m0, m1));
        const float w0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mx);
        const float w1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mx);
        const float L = warp_sum(fmaf(w0, lane < ns ? sl[lane] : 0.f, w1 * (lane + 32 < ns ? sl[lane + 32] : 0.f)));
        const float invL = 1.f / L;
        __syncwarp();
        if (lane < ns) s_w[r][lane] = w0 * invL;
        if (lane + 32 < ns) s_w[r][lane + 32] = w1 * invL;
    }
    __syncthreads();
    // REP*D outputs x ns splits: each thread takes its outputs in pairs and
    // the splits 16 at a time, with all 32 loads of a round in flight
    for (int ob = tid; ob < REP * D; ob += 2 * DEC_THREADS) {
        const int oi[2] = {ob, ob + DEC_THREADS};
        float acc[2] = {0.f, 0.f};
        for (int sp0 = 0; sp0 < ns; sp0 += 16) {
            float v[2][16];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int r = oi[e] / D, d = oi[e] % D;
                const float *base = part + (size_t)(kh * REP + r) * ns * (D + 2) + 2 + d;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    v[e][j] = oi[e] < REP * D && sp0 + j < ns ? __ldcg(base + (size_t)(sp0 + j) * (D + 2)) : 0.f;
            }
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int r = min(oi[e], REP * D - 1) / D;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (sp0 + j < ns) acc[e] = fmaf(s_w[r][sp0 + j], v[e][j], acc[e]);
            }
        }
#pragma unroll
        for (int e = 0; e < 2; e++) {
            if (oi[e] >= REP * D) continue;
            const int r = oi[e] / D, d = oi[e] % D;
            const int h = kh * REP + r;
            float val = rbf(acc[e]);
            if (a.gate) {
                const float gv = bf2f(qkv[(size_t)h * qstride + D + d]);
                val = rbf(__fmul_rn(val, sigmoid_bf16(gv)));
            }
            a.out[(size_t)h * D + d] = f2bf(val);
        }
    }
    if (tid == 0) a.count[kh] = 0;
    MLXD_TRACE_END(0x31)
}

template <int D, int REP>
static int launch_decode_rep(cudaLaunchConfig_t &cfg, const AttnDecodeArgs &a) {
    auto kern = attn_decode_kernel<D, REP>;
    static bool configured = false;
    if (!configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)dec_smem_bytes<D>()));
        configured = true;
    }
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
    return 0;
}

template <int D>
static int launch_decode(const AttnDecodeArgs &a, int rep, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.hkv, a.nsplit);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = dec_smem_bytes<D>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (rep) {
    case 1: return launch_decode_rep<D, 1>(cfg, a);
    case 2: return launch_decode_rep<D, 2>(cfg, a);
    case 4: return launch_decode_rep<D, 4>(cfg, a);
    case 8: return launch_decode_rep<D, 8>(cfg, a);
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
    {
        // tensor-core kernel with a cluster per kv head (attention_tc.cu);
        // 1: it does not serve this shape
        const int rc = attention_decode_tc(a, st, pdl);
        if (rc <= 0) return rc;
    }
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
