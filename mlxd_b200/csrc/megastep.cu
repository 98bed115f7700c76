// One greedy/logits decode step as a single persistent kernel.
//
// model_forward for one token (src/engine/emodel.c:221-337 with the layer of
// forward.c:1288-1380) runs as one cooperative launch of one CTA (16 warps)
// per SM. The step is a fixed sequence of phases: embed, then per layer
//   qkv  = W_qkv . rmsnorm(h)                        (fwd_attention :497-549)
//   attn = SDPA(norm+rope(q), cache + norm+rope(k))  (:591-731)
//   h1   = h + W_o . attn
//   act  = swiglu(W_gate|up . rmsnorm(h1))           (fwd_swiglu :900-958)
//   h    = h1 + W_down . act
// and finally logits = W_lm . rmsnorm(h) with the fused greedy key.
//
// Every CTA owns a static share of every phase: whole row blocks (gate|up
// pairs for SwiGLU) of each projection, one (kv head, split) of the
// attention. Warp w of a CTA takes items w, w+16, ... of its share (an item
// is one block of 8 groups of one row block: 4 KB of packed weights in the
// integer-MMA layout + 512 B of scale/bias records, as qgemv_i8_kernel). A warp's items of all projection phases, in order, form
// its weight stream, which it keeps two items ahead with cp.async into two
// private shared-memory buffers: the copy of the item after next is issued as
// soon as an item is consumed, across phase boundaries (and over the
// attention phase, which reads the cache with its own register prefetch).
// Weights and cached rows do not depend on the activations, so they stream
// while the grid waits at the phase boundary. Phases are separated by a grid-wide arrival counter;
// each CTA then stages the phase input (with RMSNorm) in shared memory.
// Partial sums of each item are kept per item and added in item order by the
// warp that completes a row block (deterministic). Attention partials of the
// splits of a kv head are merged by all CTAs of that head after a per-head
// arrival counter.
//
// All waits are bounded; on a timeout the kernel records an error flag and
// stops waiting, so the launch ends and the host reports the step as failed.
#include <stdlib.h>
#include <string.h>
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(megastep)

constexpr int MS_WARPS = 16;
constexpr int MS_CT = MS_WARPS * 32;
constexpr int MS_ITEM = 4608;                       // 8 tiles + 512 B of scale/bias records
constexpr int MS_KB = 4;                            // cached positions per warp batch
#ifndef MS_AHEAD
#define MS_AHEAD 2                                  // stream items in flight per warp (1 or 2)
#endif
constexpr unsigned long long MS_WAIT_NS = 500000000ull;   // give up on a wait after 0.5 s

struct MsMat {
    const uint8_t *tiles, *sbr;   // integer-MMA tiles and scale/bias records
    int rows, cols;
};
struct MsLayer {
    MsMat qkv, o, gu, down;
    const uint16_t *ln1, *ln2, *qn, *kn;
};
struct MsArgs {
    int L;
    MsMat lm;
    const uint16_t *fnorm;
    const uint32_t *emb_w;
    const uint16_t *emb_s, *emb_b;
    int emb_g;
    int H, hq, hkv, qdim, vocab;
    float eps;
    const float *rope_cs;
    int rope_dims;
    int32_t *token;
    uint16_t *h, *h1, *qkv, *att, *act;
    float *part;                // [hq][nspl][D + 4]
    int *sync;                  // [0] grid arrivals, [1 + kh] attention arrivals
    int nspl;
    int *err;
};

// What changes from call to call (the cache, the position counter, the input
// and output slots) is a kernel parameter passed on by value.
struct MsCall {
    uint16_t *kc, *vc;
    size_t layer_elems;
    int cap, window;
    int32_t *d_pos;
    const int32_t *ids;
    unsigned long long *amax;   // null: no greedy key
    uint16_t *logits;           // null: logits not kept
};

// The model's arguments and layer table live in constant memory (copied from
// the model's fixed pinned block before each launch), so every warp reads
// them through the constant cache and nothing goes to the phase functions by
// address.
constexpr int MS_MAX_LAYERS = 128;
struct MsConst {
    MsArgs a;
    MsLayer layers[MS_MAX_LAYERS];
};
static __constant__ MsConst c_ms;
#define MA (c_ms.a)

struct MsSmem {
    size_t wbuf, xb, xsum, zero, u, cnt, actx, total;
};
// The phase input staged as integer-MMA B fragments (xb, xsum, zero, as
// gemv_i8.cuh); u holds the raw x while it is staged and the item partials
// of the CTA's share afterwards; the attention working set (q, new k/v,
// per-warp partials) reuses the space from xb on.
static __host__ __device__ inline MsSmem ms_layout(int max_cols, int H, int D, int rep, int pool_items,
                                                   int pool_units) {
    MsSmem L;
    const int ng = max_cols / 64;
    const size_t att = (size_t)rep * D * 4 + (size_t)D * 4 + (size_t)MS_WARPS * D * 4 + (size_t)8 * rep * 8 +
                       (size_t)8 * rep * D * 4;
    const size_t xraw = (((size_t)(max_cols > H ? max_cols : H) * 2 + 15) / 16) * 16;
    const size_t pool = (size_t)pool_items * 64;
    L.wbuf = 0;
    L.xb = (size_t)MS_WARPS * 2 * MS_ITEM;
    L.xsum = L.xb + (size_t)ng * I8_ENT * 16;
    L.zero = L.xsum + (size_t)(ng / 8) * 64 + 64;
    L.u = L.zero + 16;
    size_t end = L.u + (xraw > pool ? xraw : pool);
    if (L.xb + att > end) end = L.xb + att;
    L.cnt = ((end + 15) / 16) * 16;
    L.actx = L.cnt + (((size_t)pool_units * 4 + 15) / 16) * 16;
    L.total = L.actx + (size_t)3 * D * 4;
    return L;
}

MLXD_DEV int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
MLXD_DEV int ld_relaxed(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// one thread: wait until *p >= target (false after MS_WAIT_NS). The polls are
// relaxed; one acquiring load once the count is reached orders the reads
// that follow (an acquire per poll would keep invalidating this SM's L1).
MLXD_DEV bool ms_spin(const int *p, int target) {
    if (ld_relaxed(p) < target) {
        const unsigned long long t0 = global_ns();
        for (;;) {
            __nanosleep(32);
            if (ld_relaxed(p) >= target) break;
            if (global_ns() - t0 > MS_WAIT_NS) return false;
        }
    }
    return ld_acquire(p) >= target;
}
// A CTA that gave up on one wait (flag `dead` in shared memory, error word
// set) stops waiting from then on and runs through the remaining phases, so
// the launch ends within about one wait limit per CTA.
MLXD_DEV void ms_fail(volatile int *dead, int *err) {
    *dead = 1;
    *err = 1;
}
MLXD_DEV void cbar() { __syncthreads(); }

// the CTA's share of n units for phase ph (rotated so that no CTA takes the
// larger share in every phase)
MLXD_DEV void ms_units(int n, int ph, int &u0, int &u1) {
    const int G = gridDim.x;
    const int c = (int)((blockIdx.x + (unsigned)ph * 37u) % (unsigned)G);
    u0 = (int)((long long)n * c / G);
    u1 = (int)((long long)n * (c + 1) / G);
}
// items of the CTA's share of a projection phase; u0 = its first unit
MLXD_DEV int ms_share(const MsMat &M, int unit_rb, int ph, int &u0) {
    int u1;
    ms_units(M.rows / 16 / unit_rb, ph, u0, u1);
    return (u1 - u0) * unit_rb * (M.cols / 512);
}

struct MsAttnShare {
    int kh, sp;            // kh < 0: no attention work for this CTA
    int s0, s1, nc;        // positions [s0, s1) of the split; nc = cached rows in it
};
MLXD_DEV MsAttnShare ms_attn_share(int ph, int pos, int window) {
    MsAttnShare s;
    const int G = gridDim.x;
    const int c = (int)((blockIdx.x + (unsigned)ph * 37u) % (unsigned)G);
    s.kh = -1;
    s.sp = 0;
    s.s0 = s.s1 = s.nc = 0;
    if (c >= MA.hkv * MA.nspl) return s;
    s.kh = c / MA.nspl;
    s.sp = c % MA.nspl;
    const int T = pos + 1;
    const int lo = window > 0 ? max(0, T - window) : 0;
    const int span = T - lo;
    s.s0 = lo + (int)((long long)span * s.sp / MA.nspl);
    s.s1 = lo + (int)((long long)span * (s.sp + 1) / MA.nspl);
    s.nc = max(0, min(s.s1, pos) - s.s0);
    return s;
}

// The warp's weight stream: its items of every projection phase in order
// (projection phase g: 4 per layer, q|k|v, o, gate|up, down, then lm_head).
struct MsStream {
    int g;               // projection phase of the issue cursor; -1 when done
    int j, m;            // next item of the warp's share in it, share size
    long long i0;        // first item of the CTA's share in the matrix
    const uint8_t *tiles, *sbr;
    long long issued, consumed;
};
MLXD_DEV MsMat ms_proj(int g, int &unit_rb, int &ph) {
    if (g >= 4 * MA.L) {
        unit_rb = 1;
        ph = 1 + 5 * MA.L;
        return MA.lm;
    }
    const int l = g >> 2, r = g & 3;
    ph = 1 + 5 * l + (r == 0 ? 0 : r + 1);   // q|k|v 1, o 3, gate|up 4, down 5
    unit_rb = r == 2 ? 2 : 1;
    return r == 0 ? c_ms.layers[l].qkv : r == 1 ? c_ms.layers[l].o : r == 2 ? c_ms.layers[l].gu
                                                                           : c_ms.layers[l].down;
}
// move the cursor to the next phase in which the warp has items
MLXD_DEV void ms_seek(MsStream &st, int warp) {
    while (st.g >= 0) {
        if (st.g > 4 * MA.L) {
            st.g = -1;
            return;
        }
        int urb, ph, u0;
        const MsMat M = ms_proj(st.g, urb, ph);
        const int n = ms_share(M, urb, ph, u0);
        st.m = n > warp ? (n - warp + MS_WARPS - 1) / MS_WARPS : 0;
        st.i0 = (long long)u0 * urb * (M.cols / 512);
        st.tiles = M.tiles;
        st.sbr = M.sbr;
        if (st.j < st.m) return;
        st.g++;
        st.j = 0;
    }
}
// request the stream's next item into the buffer the warp consumed last (one
// commit group per stream position, empty past the end)
MLXD_DEV void ms_issue(MsStream &st, unsigned char *wbuf, int warp, int lane) {
    if (st.g >= 0) {
        unsigned char *dst = wbuf + (st.issued & 1) * MS_ITEM + lane * 16;
        const long long item = st.i0 + warp + (long long)st.j * MS_WARPS;
        const uint8_t *t = st.tiles + item * 4096 + lane * 16;
#pragma unroll
        for (int p = 0; p < 8; p++) cp_async16(dst + p * 512, t + p * 512);
        cp_async16(dst + 4096, st.sbr + item * 512 + lane * 16);
        st.j++;
        ms_seek(st, warp);
    }
    cp_async_commit();
    st.issued++;
}

// phase input as integer-MMA B fragments (one copy of the code for every
// phase, instruction-cache friendly; the norm is on when nw is given)
__device__ __noinline__ float ms_stage_x(const uint16_t *x, const uint16_t *nw, int cols, float eps,
                                         unsigned char *smem, const MsSmem &Lo, float *s_red, unsigned *s_max) {
    I8Pre<MS_CT> pre;
    i8_stage_pre<MS_CT>(pre, nw, cols);
    return i8_stage<MS_CT>(x, nw, cols, eps, reinterpret_cast<uint16_t *>(smem + Lo.u),
                           reinterpret_cast<uint32_t *>(smem + Lo.xb), reinterpret_cast<float *>(smem + Lo.xsum),
                           reinterpret_cast<uint32_t *>(smem + Lo.zero), s_red, s_max, pre);
}

enum { MS_EPI_STORE = 0, MS_EPI_RESIDUAL = 1, MS_EPI_SWIGLU = 2, MS_EPI_LOGITS = 3 };

struct MsGemvOut {
    uint16_t *y;
    const uint16_t *residual;
    unsigned long long *amax;
    int row_offset;
};

// one unit's rows once all its items are in: the items' partial sums added in
// item order, then the epilogue (lanes 0..15, one row each)
MLXD_DEV void ms_unit_epilogue(int EPI, const MsGemvOut &o, const float *ps, int nbk, int unit, int lane) {
    const int UNIT_RB = EPI == MS_EPI_SWIGLU ? 2 : 1;
    unsigned long long key = 0ull;
    if (lane < 16) {
        float acc[2] = {0.f, 0.f};
        for (int u = 0; u < UNIT_RB; u++) {
            float sum = 0.f;
            for (int i = u * nbk; i < (u + 1) * nbk; i++) sum += ps[i * 16 + lane];
            acc[u] = sum;
        }
        const int row = unit * 16 + lane;
        if (EPI == MS_EPI_STORE) {
            o.y[row] = f2bf(acc[0]);
        } else if (EPI == MS_EPI_RESIDUAL) {
            o.y[row] = f2bf(__fadd_rn(bf2f(o.residual[row]), rbf(acc[0])));
        } else if (EPI == MS_EPI_SWIGLU) {
            o.y[row] = f2bf(swiglu_bf16(rbf(acc[0]), rbf(acc[1])));
        } else {
            if (o.y) o.y[row] = f2bf(acc[0]);
            key = argmax_key(rbf(acc[0]), o.row_offset + row);
        }
    }
    if (EPI == MS_EPI_LOGITS) {
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, key, s);
            key = other > key ? other : key;
        }
        if (lane == 0 && o.amax) atomicMax(o.amax, key);
    }
}

// The warp's share of one projection phase, consumed from its weight stream
// (the item now consumed has landed once at most one newer copy group is
// pending); each consumed buffer is refilled with the stream's item after
// next at once.
MLXD_DEV void ms_gemv(int EPI, const MsMat M, int u0, int n, const MsGemvOut o, MsStream &st,
                      unsigned char *wbuf, const I8Lane &IL, int *s_cnt, float *pool) {
    const int UNIT_RB = EPI == MS_EPI_SWIGLU ? 2 : 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = lane & 3, gq = lane >> 2;
    const int nbk = M.cols / 512;
    const int ipu = nbk * UNIT_RB;
    for (int k = warp; k < n; k += MS_WARPS) {
#if MS_AHEAD == 1
        ms_issue(st, wbuf, warp, lane);
#endif
        cp_async_wait<1>();
        __syncwarp();   // the lanes' copies of the item, seen by every lane

        const unsigned char *buf = wbuf + (st.consumed & 1) * MS_ITEM;
        const int unit = k / ipu;
        const int iu = k - unit * ipu;
        const int bk = iu % nbk;
        uint4 w[8];
#pragma unroll
        for (int p = 0; p < 8; p++) w[p] = *reinterpret_cast<const uint4 *>(buf + p * 512 + lane * 16);
        const unsigned char *rec = buf + 4096 + (gq * 2 + (t >> 1)) * 32;
        const uint4 sA = *reinterpret_cast<const uint4 *>(rec);
        const uint4 sB = *reinterpret_cast<const uint4 *>(rec + 16);
        // every lane's reads of the buffer are done: refill it
        __syncwarp();
        st.consumed++;
#if MS_AHEAD == 2
        ms_issue(st, wbuf, warp, lane);
#endif
        float y0, y1;
        i8_item(w, sA, sB, IL, bk, y0, y1, I8NoRefill{});
        float *ps = pool + (size_t)unit * ipu * 16;
        if (t == 0) {
            ps[iu * 16 + gq] = y0;
            ps[iu * 16 + gq + 8] = y1;
        }
        __syncwarp();
        int done = 0;
        if (lane == 0) {
            __threadfence_block();
            const int old = atomicAdd(&s_cnt[unit], 1);
            done = old + 1 == ipu;
            if (done) s_cnt[unit] = 0;
        }
        done = __shfl_sync(0xffffffffu, done, 0);

        if (done) {
            __threadfence_block();
            ms_unit_epilogue(EPI, o, ps, nbk, u0 + unit, lane);
        }
    }
}

// online-softmax pair merge (log2 domain); m = -inf means empty
MLXD_DEV void sm_merge(float &m, float &l, float &o, float m2, float l2, float o2) {
    const float mx = fmaxf(m, m2);
    if (mx == -INFINITY) return;
    const float a = m == -INFINITY ? 0.f : exp2f(m - mx);
    const float b = m2 == -INFINITY ? 0.f : exp2f(m2 - mx);
    l = l * a + l2 * b;
    o = o * a + o2 * b;
    m = mx;
}

// Attention constants that do not depend on this step's projection (the q/k
// norm weights and the cos/sin row of the position), loaded into shared
// memory while the q|k|v phase still runs. actx: [D] qn, [D] kn, [rope_dims]
// cos/sin pairs, as f32.
template <int D>
MLXD_DEV void ms_attn_preload(const MsLayer &Ly, int pos, float *actx) {
    const int tid = threadIdx.x;
    const int half = MA.rope_dims / 2;
    const float *cs = MA.rope_cs + (size_t)pos * half * 2;
    for (int i = tid; i < 2 * D + 2 * half; i += MS_CT) {
        float v;
        if (i < D) v = Ly.qn ? bf2f(Ly.qn[i]) : 1.f;
        else if (i < 2 * D) v = Ly.kn ? bf2f(Ly.kn[i - D]) : 1.f;
        else v = cs[i - 2 * D];
        actx[i] = v;
    }
}

// head_norm_rope (common.cuh) with the norm weights and the cos/sin row in
// shared memory: same arithmetic, same association
MLXD_DEV void ms_norm_rope(float *v, int D, const float *nwf, bool norm, float eps, const float *csrow,
                           int rope_dims) {
    const int lane = threadIdx.x & 31;
    if (norm) {
        float acc = 0.f;
        for (int d = lane; d < D; d += 32) acc = fmaf(v[d], v[d], acc);
        acc = warp_sum(acc);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), eps)));
        __syncwarp();
        for (int d = lane; d < D; d += 32) v[d] = rbf(__fmul_rn(nwf[d], rbf(__fmul_rn(v[d], inv))));
        __syncwarp();
    }
    const int half = rope_dims / 2;
    float ra[4], rb[4];
    int cnt = 0;
    for (int i = lane; i < half; i += 32, cnt++) {
        const float x1 = v[i], x2 = v[i + half];
        const float co = csrow[2 * i], si = csrow[2 * i + 1];
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

// cached rows of positions [j0, j0 + MS_KB) (clamped to j1) of one kv head
template <int D>
MLXD_DEV void ms_load_kv(typename std::conditional<D == 128, uint2, uint32_t>::type (&kb)[MS_KB],
                         typename std::conditional<D == 128, uint2, uint32_t>::type (&vb)[MS_KB],
                         const uint16_t *kc, const uint16_t *vc, int j0, int j1, int cap, int lane) {
    using RowT = typename std::conditional<D == 128, uint2, uint32_t>::type;
    constexpr int DL = D / 32;
#pragma unroll
    for (int u = 0; u < MS_KB; u++) {
        const int j = min(j0 + u, j1 - 1);
        if (j >= 0) {
            const size_t off = (size_t)(j % cap) * D + lane * DL;
            kb[u] = *reinterpret_cast<const RowT *>(kc + off);
            vb[u] = *reinterpret_cast<const RowT *>(vc + off);
        }
    }
}

// the CTA's attention share; kb/vb hold the warp's first MS_KB cached rows on
// entry; afterwards `it` gets the warp's first item of the o projection
template <int D, int REP>
__device__ __noinline__ void ms_attention(const MsCall kv, int l, int ph, int pos, const MsAttnShare s,
                           typename std::conditional<D == 128, uint2, uint32_t>::type (&kb)[MS_KB],
                           typename std::conditional<D == 128, uint2, uint32_t>::type (&vb)[MS_KB],
                           unsigned char *scratch, const float *actx, bool qk_norm, volatile int *dead) {
    constexpr int DL = D / 32;
    constexpr int PB = MS_KB;                  // positions scored together
    using RowT = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (s.kh < 0) return;
    const int kh = s.kh;
    const uint16_t *kc = kv.kc + (size_t)l * kv.layer_elems + (size_t)kh * kv.cap * D;
    const uint16_t *vc = kv.vc + (size_t)l * kv.layer_elems + (size_t)kh * kv.cap * D;
    const int per = (s.nc + MS_WARPS - 1) / MS_WARPS;
    const int w0 = s.s0 + warp * per, w1 = min(s.s0 + s.nc, w0 + per);

    float *s_q = reinterpret_cast<float *>(scratch);                 // [REP][D]
    uint16_t *s_knew = reinterpret_cast<uint16_t *>(s_q + REP * D);  // [D]
    uint16_t *s_vnew = s_knew + D;                                   // [D]
    float *s_v = reinterpret_cast<float *>(s_vnew + D);              // [16][D] staging
    float *s_ml = s_v + MS_WARPS * D;                                // [8][REP][2]
    float *s_o = s_ml + 8 * REP * 2;                                 // [8][REP][D]

    // q heads of the group, the new k (norm + rope) and the new v
    const uint16_t *qkv = MA.qkv;
    for (int vi = warp; vi < REP + 2; vi += MS_WARPS) {
        if (vi == REP + 1) {
            for (int d = lane; d < D; d += 32) s_vnew[d] = qkv[MA.qdim + (size_t)(MA.hkv + kh) * D + d];
            continue;
        }
        float *v = s_v + warp * D;
        const uint16_t *src = vi < REP ? qkv + (size_t)(kh * REP + vi) * D : qkv + MA.qdim + (size_t)kh * D;
        for (int d = lane; d < D; d += 32) v[d] = bf2f(src[d]);
        __syncwarp();
        ms_norm_rope(v, D, vi < REP ? actx : actx + D, qk_norm, MA.eps, actx + 2 * D, MA.rope_dims);
        if (vi < REP) {
            for (int d = lane; d < D; d += 32) s_q[vi * D + d] = v[d];
        } else {
            for (int d = lane; d < D; d += 32) s_knew[d] = f2bf(v[d]);
        }
        __syncwarp();
    }
    __syncthreads();
    if (s.sp == 0) {
        for (int d = tid; d < D; d += MS_CT) {
            const size_t off = (size_t)(pos % kv.cap) * D + d;
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
            q[r][i] = s_q[r * D + lane * DL + i] * qscale;
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
    // nv (<= PB) positions at once: independent scores, one reduction pass,
    // one online-softmax update per head
    auto visit = [&](const RowT (&kr)[PB], const RowT (&vr)[PB], int nv) {
        float sc[REP][PB];
#pragma unroll
        for (int u = 0; u < PB; u++) {
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
                for (int u = 0; u < PB; u++) sc[r][u] += __shfl_xor_sync(0xffffffffu, sc[r][u], sh);
#pragma unroll
        for (int r = 0; r < REP; r++) {
            float mn = m[r];
#pragma unroll
            for (int u = 0; u < PB; u++)
                if (u < nv) mn = fmaxf(mn, sc[r][u]);
            const float al = exp2f(m[r] - mn);
            float ps = 0.f;
#pragma unroll
            for (int u = 0; u < PB; u++) {
                sc[r][u] = u < nv ? exp2f(sc[r][u] - mn) : 0.f;
                ps += sc[r][u];
            }
            lsum[r] = lsum[r] * al + ps;
#pragma unroll
            for (int i = 0; i < DL; i++) o[r][i] *= al;
            m[r] = mn;
        }
#pragma unroll
        for (int u = 0; u < PB; u++) {
            float vf[DL];
            unpack(vr[u], vf);
#pragma unroll
            for (int r = 0; r < REP; r++)
#pragma unroll
                for (int i = 0; i < DL; i++) o[r][i] = fmaf(sc[r][u], vf[i], o[r][i]);
        }
    };
    for (int j0 = w0; j0 < w1; j0 += PB) {
        RowT kr[PB], vr[PB];
#pragma unroll
        for (int u = 0; u < PB; u++) {
            kr[u] = kb[u];
            vr[u] = vb[u];
        }
        if (j0 + PB < w1) ms_load_kv<D>(kb, vb, kc, vc, j0 + PB, w1, kv.cap, lane);
        visit(kr, vr, min(PB, w1 - j0));
    }
    // the new position (its row came from this step's projection)
    if (warp == MS_WARPS - 1 && pos >= s.s0 && pos < s.s1) {
        RowT kr[PB], vr[PB];
#pragma unroll
        for (int u = 0; u < PB; u++) {
            kr[u] = *reinterpret_cast<const RowT *>(s_knew + lane * DL);
            vr[u] = *reinterpret_cast<const RowT *>(s_vnew + lane * DL);
        }
        visit(kr, vr, 1);
    }
    // merge the warps of this CTA into the split's partial: warps 8..15 hand
    // their state to warps 0..7, which then write theirs for the final sum
    static_assert(MS_WARPS == 16, "two-round warp merge");
    auto put = [&](int slotw) {
#pragma unroll
        for (int r = 0; r < REP; r++) {
            if (lane == 0) {
                s_ml[(slotw * REP + r) * 2] = m[r];
                s_ml[(slotw * REP + r) * 2 + 1] = lsum[r];
            }
            if constexpr (DL == 4)
                *reinterpret_cast<float4 *>(s_o + (slotw * REP + r) * D + lane * 4) =
                    make_float4(o[r][0], o[r][1], o[r][2], o[r][3]);
            else
                *reinterpret_cast<float2 *>(s_o + (slotw * REP + r) * D + lane * 2) = make_float2(o[r][0], o[r][1]);
        }
    };
    if (warp >= 8) put(warp - 8);
    __syncthreads();
    if (warp < 8) {
#pragma unroll
        for (int r = 0; r < REP; r++) {
            const float m2 = s_ml[(warp * REP + r) * 2], l2 = s_ml[(warp * REP + r) * 2 + 1];
            const float mx = fmaxf(m[r], m2);
            if (mx != -INFINITY) {
                const float wa = m[r] == -INFINITY ? 0.f : exp2f(m[r] - mx);
                const float wb = m2 == -INFINITY ? 0.f : exp2f(m2 - mx);
#pragma unroll
                for (int i = 0; i < DL; i++)
                    o[r][i] = o[r][i] * wa + s_o[(warp * REP + r) * D + lane * DL + i] * wb;
                lsum[r] = lsum[r] * wa + l2 * wb;
                m[r] = mx;
            }
        }
    }
    __syncthreads();
    if (warp < 8) put(warp);
    __syncthreads();
    for (int idx = tid; idx < REP * D; idx += MS_CT) {
        const int r = idx / D, d = idx % D;
        float mm = -INFINITY, ll = 0.f, oo = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++)
            sm_merge(mm, ll, oo, s_ml[(w * REP + r) * 2], s_ml[(w * REP + r) * 2 + 1],
                     s_o[(w * REP + r) * D + d]);
        float *rec = MA.part + ((size_t)(kh * REP + r) * MA.nspl + s.sp) * (D + 4);
        rec[d] = oo;
        if (d == 0) {
            rec[D] = mm;
            rec[D + 1] = ll;
        }
    }
    // wait for every split of this kv head, then merge a slice of its outputs
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&MA.sync[1 + kh], 1);
        if (!*dead && !ms_spin(&MA.sync[1 + kh], MA.nspl * (l + 1))) ms_fail(dead, MA.err);
    }
    __syncthreads();
    const int n_out = REP * D;
    const int o0 = (int)((long long)n_out * s.sp / MA.nspl);
    const int o1 = (int)((long long)n_out * (s.sp + 1) / MA.nspl);
    constexpr int MSPL = 4;   // splits per thread loaded together
    for (int base_o = o0; base_o < o1; base_o += MS_CT / 8) {
        const int oi = base_o + tid / 8, sub = tid % 8;
        float mm = -INFINITY, ll = 0.f, oo = 0.f;
        if (oi < o1) {
            const int r = oi / D, d = oi % D;
            const float *rec = MA.part + (size_t)(kh * REP + r) * MA.nspl * (D + 4);
            for (int sp0 = sub; sp0 < MA.nspl; sp0 += 8 * MSPL) {
                float pm[MSPL], pl[MSPL], po[MSPL];
#pragma unroll
                for (int j = 0; j < MSPL; j++) {
                    const int sp = sp0 + 8 * j;
                    pm[j] = -INFINITY;
                    pl[j] = po[j] = 0.f;
                    if (sp < MA.nspl) {
                        const float *rr = rec + (size_t)sp * (D + 4);
                        pm[j] = __ldcg(rr + D);
                        pl[j] = __ldcg(rr + D + 1);
                        po[j] = __ldcg(rr + d);
                    }
                }
#pragma unroll
                for (int j = 0; j < MSPL; j++) sm_merge(mm, ll, oo, pm[j], pl[j], po[j]);
            }
        }
#pragma unroll
        for (int sh = 1; sh < 8; sh <<= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, mm, sh);
            const float l2 = __shfl_xor_sync(0xffffffffu, ll, sh);
            const float o2 = __shfl_xor_sync(0xffffffffu, oo, sh);
            sm_merge(mm, ll, oo, m2, l2, o2);
        }
        if (oi < o1 && sub == 0) {
            const int r = oi / D, d = oi % D;
            MA.att[(size_t)(kh * REP + r) * D + d] = f2bf(oo / ll);
        }
    }
}

template <int D, int REP>
__global__ void __launch_bounds__(MS_CT, 1) megastep_kernel(const MsCall kv, int max_cols, int pool_items,
                                                            int pool_units) {
    using RowT = typename std::conditional<D == 128, uint2, uint32_t>::type;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(16) float s_red[MS_WARPS];
    __shared__ __align__(16) unsigned s_max[MS_WARPS];
    __shared__ volatile int s_dead;
    const MsSmem Lo = ms_layout(max_cols, MA.H, D, REP, pool_items, pool_units);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned char *wbuf = smem + Lo.wbuf + (size_t)warp * 2 * MS_ITEM;
    unsigned char *scratch = smem + Lo.xb;
    float *pool = reinterpret_cast<float *>(smem + Lo.u);
    int *s_cnt = reinterpret_cast<int *>(smem + Lo.cnt);
    float *actx = reinterpret_cast<float *>(smem + Lo.actx);
    const int pos = *kv.d_pos;
    const int G = gridDim.x;
    const uint32_t *xbw = reinterpret_cast<const uint32_t *>(smem + Lo.xb);
    const float *xsum4 = reinterpret_cast<const float *>(smem + Lo.xsum);
    const uint32_t *zero16 = reinterpret_cast<const uint32_t *>(smem + Lo.zero);
    float lsc;

    for (int i = tid; i < pool_units; i += MS_CT) s_cnt[i] = 0;
    if (tid == 0) s_dead = 0;

    int ph = 0;
    MLXD_TRACE_START
    auto phase_done = [&]() {
        // every thread's global writes of this phase (ordered before thread 0
        // by the CTA barrier, made visible by its fence), then one arrival
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicAdd(&MA.sync[0], 1);
        }
        MLXD_TRACE_END(0x1000 + ph)
        ph++;
    };
    auto phase_wait = [&]() {
        MLXD_TRACE_RESTART
        if (tid == 0 && !s_dead && !ms_spin(&MA.sync[0], ph * G)) ms_fail(&s_dead, MA.err);
        __syncthreads();
        MLXD_TRACE_WAITED
    };

    // the weight stream starts two items ahead, during the embedding phase
    MsStream st;
    st.g = 0;
    st.j = 0;
    st.issued = st.consumed = 0;
    ms_seek(st, warp);
    for (int i = 0; i < MS_AHEAD; i++) ms_issue(st, wbuf, warp, lane);
    __syncthreads();

    // embed (fwd_embed, forward.c:65-147): this CTA's slice of the token's row
    {
        int id = kv.ids[0];
        if (id < 0 || id >= MA.vocab) id = 0;   // a failed draw; the host rejects the step
        const int nv = MA.H / 8;
        const int v0 = (int)((long long)nv * blockIdx.x / G), v1 = (int)((long long)nv * (blockIdx.x + 1) / G);
        const int ng = MA.H / MA.emb_g;
        for (int i = v0 + tid; i < v1; i += MS_CT) {
            const uint32_t w = MA.emb_w[(size_t)id * nv + i];
            const int g = (i * 8) / MA.emb_g;
            const float sc = bf2f(MA.emb_s[(size_t)id * ng + g]), bi = bf2f(MA.emb_b[(size_t)id * ng + g]);
            uint32_t o4[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                o4[j] = pack_bf2(__fmaf_rn(sc, (float)((w >> (8 * j)) & 0xF), bi),
                                 __fmaf_rn(sc, (float)((w >> (8 * j + 4)) & 0xF), bi));
            *reinterpret_cast<uint4 *>(MA.h + (size_t)i * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
        }
        phase_done();
    }
    int u0, n;
    for (int l = 0; l < MA.L; l++) {
        const MsLayer &Ly = c_ms.layers[l];
        // q|k|v; then the warp fetches its first cached rows of the attention
        phase_wait();
        lsc = ms_stage_x(MA.h, Ly.ln1, Ly.qkv.cols, MA.eps, smem, Lo, s_red, s_max);
        MLXD_TRACE_T(tr_st0_)
        n = ms_share(Ly.qkv, 1, ph, u0);
        ms_gemv(MS_EPI_STORE, Ly.qkv, u0, n, MsGemvOut{MA.qkv, nullptr, nullptr, 0}, st, wbuf,
                i8_lane(xbw, xsum4, zero16, lsc), s_cnt, pool);
                MLXD_TRACE_REC(tid == 0, 0x2000 + ph, tr_t1_, tr_st0_, gtime())

        const MsAttnShare ash = ms_attn_share(ph + 1, pos, kv.window);
        RowT kb[MS_KB], vb[MS_KB];
        if (ash.kh >= 0) {
            const int per = (ash.nc + MS_WARPS - 1) / MS_WARPS;
            const int w0 = ash.s0 + warp * per, w1 = min(ash.s0 + ash.nc, w0 + per);
            ms_load_kv<D>(kb, vb, kv.kc + (size_t)l * kv.layer_elems + (size_t)ash.kh * kv.cap * D,
                          kv.vc + (size_t)l * kv.layer_elems + (size_t)ash.kh * kv.cap * D, w0, w1, kv.cap, lane);
        }
        ms_attn_preload<D>(Ly, pos, actx);
        phase_done();
        // attention
        phase_wait();
        ms_attention<D, REP>(kv, l, ph, pos, ash, kb, vb, scratch, actx, Ly.qn != nullptr, &s_dead);
        phase_done();
        // o projection + residual
        phase_wait();
        lsc = ms_stage_x(MA.att, nullptr, Ly.o.cols, MA.eps, smem, Lo, s_red, s_max);
        MLXD_TRACE_T(tr_st1_)
        n = ms_share(Ly.o, 1, ph, u0);
        ms_gemv(MS_EPI_RESIDUAL, Ly.o, u0, n, MsGemvOut{MA.h1, MA.h, nullptr, 0}, st, wbuf,
                i8_lane(xbw, xsum4, zero16, lsc), s_cnt, pool);
                MLXD_TRACE_REC(tid == 0, 0x2000 + ph, tr_t1_, tr_st1_, gtime())
        phase_done();
        // gate|up + SwiGLU
        phase_wait();
        lsc = ms_stage_x(MA.h1, Ly.ln2, Ly.gu.cols, MA.eps, smem, Lo, s_red, s_max);
        MLXD_TRACE_T(tr_st2_)
        n = ms_share(Ly.gu, 2, ph, u0);
        ms_gemv(MS_EPI_SWIGLU, Ly.gu, u0, n, MsGemvOut{MA.act, nullptr, nullptr, 0}, st, wbuf,
                i8_lane(xbw, xsum4, zero16, lsc), s_cnt, pool);
                MLXD_TRACE_REC(tid == 0, 0x2000 + ph, tr_t1_, tr_st2_, gtime())
        phase_done();
        // down + residual
        phase_wait();
        lsc = ms_stage_x(MA.act, nullptr, Ly.down.cols, MA.eps, smem, Lo, s_red, s_max);
        MLXD_TRACE_T(tr_st3_)
        n = ms_share(Ly.down, 1, ph, u0);
        ms_gemv(MS_EPI_RESIDUAL, Ly.down, u0, n, MsGemvOut{MA.h, MA.h1, nullptr, 0}, st, wbuf,
                i8_lane(xbw, xsum4, zero16, lsc), s_cnt, pool);
                MLXD_TRACE_REC(tid == 0, 0x2000 + ph, tr_t1_, tr_st3_, gtime())
        phase_done();
    }
    // final norm + lm_head (+ greedy key)
    phase_wait();
    lsc = ms_stage_x(MA.h, MA.fnorm, MA.lm.cols, MA.eps, smem, Lo, s_red, s_max);
    MLXD_TRACE_T(tr_st4_)
    n = ms_share(MA.lm, 1, ph, u0);
    ms_gemv(MS_EPI_LOGITS, MA.lm, u0, n, MsGemvOut{kv.logits, nullptr, kv.amax, 0}, st, wbuf,
            i8_lane(xbw, xsum4, zero16, lsc), s_cnt, pool);
            MLXD_TRACE_REC(tid == 0, 0x2000 + ph, tr_t1_, tr_st4_, gtime())
    cp_async_wait<0>();
    phase_done();
    // step end (step_finish_kernel): token from the key, next position
    if (blockIdx.x == 0) {
        phase_wait();
        if (tid == 0) {
            if (kv.amax) {
                const unsigned long long key = *kv.amax;
                *MA.token = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
                *kv.amax = 0ull;
            }
            *kv.d_pos = pos + 1;
        }
    }
}

}  // namespace mlxd

namespace mlxd {

// ------------------------------------------------------------------ host

struct MegaState {
    MsConst *hc = nullptr;  // pinned host copy of the constant block
    int *sync = nullptr;   // [1 + hkv]
    int *err = nullptr;
    float *part = nullptr;
    int nspl = 0, grid = 0, max_cols = 0, D = 0, rep = 0, pool_items = 0, pool_units = 0;
    size_t smem = 0;
};

template <int D, int REP>
static int ms_prepare(size_t smem, int *blocks) {
    auto k = megastep_kernel<D, REP>;
    MLXD_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    MLXD_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, k, MS_CT, smem));
    return 0;
}
template <int D, int REP>
static int ms_launch(const MsCall &kv, const MegaState &S, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S.grid);
    cfg.blockDim = dim3(MS_CT);
    cfg.dynamicSmemBytes = S.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, megastep_kernel<D, REP>, kv, S.max_cols, S.pool_items, S.pool_units));
    return 0;
}
#define MLXD_MS_DISPATCH(FN, ...)                                        \
    switch (D * 16 + rep) {                                              \
    case 128 * 16 + 1: return FN<128, 1>(__VA_ARGS__);                   \
    case 128 * 16 + 2: return FN<128, 2>(__VA_ARGS__);                   \
    case 128 * 16 + 4: return FN<128, 4>(__VA_ARGS__);                   \
    case 128 * 16 + 8: return FN<128, 8>(__VA_ARGS__);                   \
    case 64 * 16 + 1: return FN<64, 1>(__VA_ARGS__);                     \
    case 64 * 16 + 2: return FN<64, 2>(__VA_ARGS__);                     \
    case 64 * 16 + 4: return FN<64, 4>(__VA_ARGS__);                     \
    case 64 * 16 + 8: return FN<64, 8>(__VA_ARGS__);                     \
    default: set_error("megastep: head_dim %d / GQA %d not supported", D, rep); return -1; \
    }

static int ms_prepare_any(int D, int rep, size_t smem, int *blocks) {
    MLXD_MS_DISPATCH(ms_prepare, smem, blocks)
}
static int ms_launch_any(int D, int rep, const MsCall &kv, const MegaState &S, cudaStream_t st) {
    MLXD_MS_DISPATCH(ms_launch, kv, S, st)
}

static MsMat ms_mat(const QMat &q) { return MsMat{q.ti8, q.sbi, q.rows, q.cols}; }

static bool ms_eligible(const mlxd_model *m) {
    // opt-in (MLXD_MEGASTEP=1 when the model is created): on Qwen3-8B the
    // per-op kernels with programmatic dependent launch are still faster
    const char *e = getenv("MLXD_MEGASTEP");
    if (!e || atoi(e) == 0) return false;
    const mlxd_model_config &c = m->c;
    if (c.tp_size > 1 || c.attn_gate || c.qbits != 4 || c.layers > MS_MAX_LAYERS) return false;
    if (!m->embed.quant || m->embed.sdtype != MLXD_BF16 || c.hidden % c.qgroup) return false;
    const int rep = m->hq / m->hkv;
    if (!(c.head_dim == 128 || c.head_dim == 64) || !(rep == 1 || rep == 2 || rep == 4 || rep == 8))
        return false;
    auto ok = [](const QMat &q) { return q.quant && q.fast8() && q.ti8 && q.sbi && q.rows % 16 == 0; };
    for (const Layer &L : m->L)
        if (!ok(L.qkv) || !ok(L.o) || !ok(L.gateup) || !ok(L.down) || L.gateup.rows % 32) return false;
    return ok(m->lm);
}

void megastep_free(mlxd_model *m) {
    MegaState *S = static_cast<MegaState *>(m->mega);
    if (!S) return;
    if (S->hc) cudaFreeHost(S->hc);
    dev_free(S->sync);
    dev_free(S->err);
    dev_free(S->part);
    delete S;
    m->mega = nullptr;
}

int megastep_setup(mlxd_model *m) {
    if (!ms_eligible(m)) return 0;
    const mlxd_model_config &c = m->c;
    MegaState *S = new MegaState();
    S->D = c.head_dim;
    S->rep = m->hq / m->hkv;
    S->grid = num_sms();
    S->nspl = S->grid / m->hkv;
    S->max_cols = std::max(std::max(c.hidden, m->hq * c.head_dim), m->inter_local);
    // the largest per-CTA share over the projection phases, in units and items
    auto share = [&](const QMat &q, int unit_rb) {
        const int units = q.rows / 16 / unit_rb;
        const int per = (units + S->grid - 1) / S->grid;
        S->pool_units = std::max(S->pool_units, per);
        S->pool_items = std::max(S->pool_items, per * unit_rb * (q.cols / 512));
    };
    for (const Layer &L : m->L) {
        share(L.qkv, 1);
        share(L.o, 1);
        share(L.gateup, 2);
        share(L.down, 1);
    }
    share(m->lm, 1);
    S->smem = ms_layout(S->max_cols, c.hidden, S->D, S->rep, S->pool_items, S->pool_units).total;
    int blocks = 0;
    if (S->nspl < 1 || S->smem > 227 * 1024 || ms_prepare_any(S->D, S->rep, S->smem, &blocks) || blocks < 1) {
        delete S;   // the layer-by-layer kernels serve this model
        return 0;
    }
    MsConst *hc = nullptr;
    if (!cuda_ok(cudaMallocHost(&hc, sizeof(MsConst)), "megastep constants")) {
        delete S;
        return -1;
    }
    memset(hc, 0, sizeof(MsConst));
    S->hc = hc;
    for (int l = 0; l < c.layers; l++) {
        const Layer &L = m->L[l];
        hc->layers[l] = MsLayer{ms_mat(L.qkv), ms_mat(L.o), ms_mat(L.gateup), ms_mat(L.down),
                                L.ln1, L.ln2, c.qk_norm ? L.qn : nullptr, c.qk_norm ? L.kn : nullptr};
    }
    S->sync = (int *)dev_alloc((size_t)(1 + m->hkv) * sizeof(int));
    S->err = (int *)dev_alloc(sizeof(int));
    S->part = (float *)dev_alloc((size_t)m->hq * S->nspl * (S->D + 4) * sizeof(float));
    m->mega = S;
    if (!S->sync || !S->err || !S->part || !cuda_ok(cudaMemset(S->err, 0, sizeof(int)), "megastep err")) {
        megastep_free(m);
        return -1;
    }
    MsArgs &a = hc->a;
    a.L = c.layers;
    a.lm = ms_mat(m->lm);
    a.fnorm = m->norm;
    a.emb_w = m->embed.w;
    a.emb_s = (const uint16_t *)m->embed.s;
    a.emb_b = (const uint16_t *)m->embed.b;
    a.emb_g = c.qgroup;
    a.H = c.hidden;
    a.hq = m->hq;
    a.hkv = m->hkv;
    a.qdim = m->qdim;
    a.vocab = c.vocab;
    a.eps = c.eps;
    a.rope_cs = m->rope_cs;
    a.rope_dims = c.rope_dims;
    a.token = m->token;
    a.h = m->h;
    a.h1 = m->h1;
    a.qkv = m->qkv;
    a.att = m->att;
    a.act = m->act;
    a.part = S->part;
    a.sync = S->sync;
    a.nspl = S->nspl;
    a.err = S->err;
    return 0;
}

bool megastep_ready(const mlxd_model *m, const mlxd_kv *kv) {
    const MegaState *S = static_cast<const MegaState *>(m->mega);
    return S && kv->d == S->D && kv->hkv == m->hkv;
}

int megastep_launch(mlxd_model *m, mlxd_kv *kv, const int32_t *ids_dev, uint16_t *logits, bool argmax,
                    cudaStream_t st) {
    const MegaState &S = *static_cast<const MegaState *>(m->mega);
    const mlxd_model_config &c = m->c;
    MsCall kvc = {};
    kvc.kc = kv->k;
    kvc.vc = kv->v;
    kvc.layer_elems = (size_t)kv->hkv * kv->cap * kv->d;
    kvc.cap = kv->cap;
    kvc.window = kv->window;
    kvc.d_pos = kv->d_pos;
    kvc.ids = ids_dev;
    kvc.amax = argmax ? m->amax : nullptr;
    kvc.logits = logits;
    // the model's fixed block (never rewritten after set-up) into constant memory
    MLXD_CHECK(cudaMemcpyToSymbolAsync(c_ms, S.hc, sizeof(MsArgs) + (size_t)c.layers * sizeof(MsLayer), 0,
                                       cudaMemcpyHostToDevice, st));
    MLXD_CHECK(cudaMemsetAsync(S.sync, 0, (size_t)(1 + m->hkv) * sizeof(int), st));
    return ms_launch_any(S.D, S.rep, kvc, S, st);
}

// nonzero once a megastep launch gave up on a wait (read and cleared)
int megastep_timeouts(mlxd_model *m) {
    MegaState *S = static_cast<MegaState *>(m->mega);
    if (!S) return 0;
    int v = 0, z = 0;
    if (cudaMemcpy(&v, S->err, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v) cudaMemcpy(S->err, &z, sizeof z, cudaMemcpyHostToDevice);
    return v;
}

}  // namespace mlxd
