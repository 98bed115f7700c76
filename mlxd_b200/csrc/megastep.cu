// One greedy/logits decode step as a single persistent kernel.
//
// model_forward for one token (src/engine/emodel.c:221-337 with the layer of
// forward.c:1288-1380) runs as one cooperative launch of one CTA per SM. The
// step is a fixed sequence of phases: embed, then per layer
//   qkv  = W_qkv . rmsnorm(h)                        (fwd_attention :497-549)
//   attn = SDPA(norm+rope(q), cache + norm+rope(k))  (:591-731)
//   h1   = h + W_o . attn
//   act  = swiglu(W_gate|up . rmsnorm(h1))           (fwd_swiglu :900-958)
//   h    = h1 + W_down . act
// and finally logits = W_lm . rmsnorm(h) with the fused greedy key.
//
// Every CTA owns a static share of every phase: whole row blocks (gate|up
// pairs for SwiGLU) of each projection, one (kv head, split) of the
// attention. One producer warp streams the CTA's packed weights and cached
// K/V rows, phase after phase, into a ring of MS_NS shared-memory chunks
// with cp.async.bulk (one mbarrier per chunk, no multicast); it waits only for
// free slots, never for activations, so the HBM stream runs on across phase
// boundaries while the consumer warps wait for the grid. Eight consumer warps
// wait for the previous phase (a grid-wide arrival counter), stage the phase
// input in shared memory, and consume the ring. Row-block partial sums are
// added in warp order by the warp that completes the block (deterministic).
// Attention partials of the splits of a kv head are merged by all CTAs of
// that head after a per-head arrival counter.
//
// All waits are bounded; on a timeout the kernel records an error flag,
// keeps going to the end and the host reports the step as failed.
#include <stdlib.h>
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(megastep)

constexpr int MS_CONSUMERS = 16;
constexpr int MS_CT = MS_CONSUMERS * 32;            // consumer threads
constexpr int MS_THREADS = MS_CT + 32;              // + producer warp
constexpr int MS_SLOT = 4608;                       // one item: 8 tiles + 512 B of scale/bias records
constexpr int MS_IPC = 4;                           // items per ring chunk (one copy per chunk)
constexpr int MS_CHUNK = MS_IPC * MS_SLOT;          // [4 x 4096 tiles | 4 x 512 records]
constexpr int MS_NS = 7;                            // ring chunks
constexpr int MS_POOL_ITEMS = 256;                  // item partial records (16 floats each)
constexpr unsigned long long MS_WAIT_NS = 500000000ull;   // give up on a wait after 0.5 s

struct MsMat {
    const uint8_t *tiles, *sb8;
    int rows, cols;
};
struct MsLayer {
    MsMat qkv, o, gu, down;
    const uint16_t *ln1, *ln2, *qn, *kn;
};
struct MsArgs {
    const MsLayer *layers;
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
    uint16_t *kc, *vc;
    size_t layer_elems;
    int cap, window;
    int32_t *d_pos;
    const int32_t *ids;
    unsigned long long *amax;   // null: no greedy key
    int32_t *token;
    uint16_t *logits;           // null: logits not kept
    uint16_t *h, *h1, *qkv, *att, *act;
    float *part;                // [hq][nspl][D + 4]
    int *sync;                  // [0] grid arrivals, [1 + kh] attention arrivals
    int nspl;
    int *err;
};

struct MsSmem {
    size_t ring, full, empty, cnt, red, scratch, actx, total;
};
// scratch is shared by the phase input (xp, xs, raw x) and the attention
// working set (q, new k/v, per-warp partials)
static __host__ __device__ inline MsSmem ms_layout(int max_cols, int H, int D, int rep) {
    MsSmem L;
    L.ring = 0;
    L.full = L.ring + (size_t)MS_NS * MS_CHUNK;
    L.empty = L.full + MS_NS * 8;
    L.cnt = L.empty + MS_NS * 8;
    L.red = L.cnt + (size_t)MS_POOL_ITEMS * 4;
    L.scratch = L.red + (size_t)MS_POOL_ITEMS * 16 * 4;
    const int ng = max_cols / 64;
    size_t gem = (size_t)ng * 128 + (((size_t)ng * 4 + 15) / 16) * 16 + (size_t)H * 2;
    size_t att = (size_t)rep * D * 4 + (size_t)D * 4 + (size_t)MS_CONSUMERS * D * 4 +
                 (size_t)8 * rep * 8 + (size_t)8 * rep * D * 4;
    L.actx = L.scratch + (((gem > att ? gem : att) + 15) / 16) * 16;
    L.total = L.actx + (size_t)3 * D * 4;
    return L;
}

MLXD_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(MS_CT) : "memory"); }
MLXD_DEV int ld_acquire(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
MLXD_DEV void mbar_arrive(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// arrivals item k of a phase with n items owes its chunk's empty barrier:
// the last item of a short final chunk also covers the missing items
MLXD_DEV uint32_t ms_release_count(int k, int n) {
    const int c0 = k & ~(MS_IPC - 1);
    const int len = min(MS_IPC, n - c0);
    return k == n - 1 ? (uint32_t)(MS_IPC - len + 1) : 1u;
}
// the ring chunk of chunk number g (a running count over the step)
MLXD_DEV int ms_slot(long long g) { return (int)(g % MS_NS); }
MLXD_DEV uint32_t ms_parity(long long g) { return (uint32_t)(g / MS_NS) & 1u; }
// one thread: wait until *p >= target; false after MS_WAIT_NS
MLXD_DEV bool ms_spin(const int *p, int target) {
    if (ld_acquire(p) >= target) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        __nanosleep(32);
        if (ld_acquire(p) >= target) return true;
        if (global_ns() - t0 > MS_WAIT_NS) return false;
    }
}
// A CTA that gave up on one wait (flag `dead` in shared memory, error word
// set) stops waiting from then on: the producer stops issuing copies and the
// consumers run through the remaining phases without waiting, so the launch
// ends within about one wait limit per CTA.
MLXD_DEV void ms_fail(volatile int *dead, int *err) {
    *dead = 1;
    *err = 1;
}

// the CTA's share of n units for phase ph (rotated so that no CTA takes the
// larger share in every phase)
MLXD_DEV void ms_units(int n, int ph, int &u0, int &u1) {
    const int G = gridDim.x;
    const int c = (int)((blockIdx.x + (unsigned)ph * 37u) % (unsigned)G);
    u0 = (int)((long long)n * c / G);
    u1 = (int)((long long)n * (c + 1) / G);
}

struct MsAttnShare {
    int kh, sp;            // kh < 0: no attention work for this CTA
    int s0, s1, nc;        // positions [s0, s1) of the split; nc = cached rows in it
};
template <int D>
MLXD_DEV MsAttnShare ms_attn_share(const MsArgs &a, int ph, int pos) {
    MsAttnShare s;
    const int G = gridDim.x;
    const int c = (int)((blockIdx.x + (unsigned)ph * 37u) % (unsigned)G);
    s.kh = -1;
    s.sp = 0;
    s.s0 = s.s1 = s.nc = 0;
    if (c >= a.hkv * a.nspl) return s;
    s.kh = c / a.nspl;
    s.sp = c % a.nspl;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int span = T - lo;
    s.s0 = lo + (int)((long long)span * s.sp / a.nspl);
    s.s1 = lo + (int)((long long)span * (s.sp + 1) / a.nspl);
    s.nc = max(0, min(s.s1, pos) - s.s0);
    return s;
}

// ---------------------------------------------------------------- producer
template <int D>
MLXD_DEV void ms_issue_gemv(const MsMat &M, int unit_rb, int ph, uint8_t *ring, uint64_t *full,
                            uint64_t *empty, long long &seq, volatile int *dead, int *err) {
    const int nbk = M.cols / 512;
    int u0, u1;
    ms_units(M.rows / 16 / unit_rb, ph, u0, u1);
    const long long i0 = (long long)u0 * unit_rb * nbk;
    const long long n = (long long)(u1 - u0) * unit_rb * nbk;
#ifdef MLXD_TRACE
    unsigned long long tw_ = 0, t0_ = gtime();
#endif
    for (long long k = 0; k < n; k += MS_IPC, seq++) {
        const int slot = ms_slot(seq);
        if (*dead) return;
#ifdef MLXD_TRACE
        unsigned long long ta_ = gtime();
#endif
        if (seq >= MS_NS && !mbar_wait(&empty[slot], ms_parity(seq) ^ 1u)) {
            ms_fail(dead, err);
            return;
        }
#ifdef MLXD_TRACE
        tw_ += gtime() - ta_;
#endif
        const uint32_t len = (uint32_t)min((long long)MS_IPC, n - k);
        uint8_t *dst = ring + (size_t)slot * MS_CHUNK;
        mbar_expect_tx(&full[slot], len * MS_SLOT);
        bulk_g2s(dst, M.tiles + (i0 + k) * 4096, len * 4096, &full[slot]);
        bulk_g2s(dst + MS_IPC * 4096, M.sb8 + (i0 + k) * 512, len * 512, &full[slot]);
    }
    MLXD_TRACE_REC((ph % 5) == 4 && ph < 12, 0x3100, tw_, gtime() - t0_, (unsigned long long)n)
}

template <int D>
MLXD_DEV void ms_issue_attn(const MsArgs &a, int l, int ph, int pos, uint8_t *ring, uint64_t *full,
                            uint64_t *empty, long long &seq, volatile int *dead) {
    constexpr int RB = D * 2;                 // bytes of one cached row
    constexpr int CP = MS_CHUNK / (2 * RB);   // positions per ring chunk
    const MsAttnShare s = ms_attn_share<D>(a, ph, pos);
    if (s.kh < 0) return;
    const uint16_t *kc = a.kc + (size_t)l * a.layer_elems + (size_t)s.kh * a.cap * D;
    const uint16_t *vc = a.vc + (size_t)l * a.layer_elems + (size_t)s.kh * a.cap * D;
    for (int j0 = 0; j0 < s.nc; j0 += CP, seq++) {
        const int slot = ms_slot(seq);
        if (*dead) return;
        if (seq >= MS_NS && !mbar_wait(&empty[slot], ms_parity(seq) ^ 1u)) {
            ms_fail(dead, a.err);
            return;
        }
        const int cnt = min(CP, s.nc - j0);
        mbar_expect_tx(&full[slot], (uint32_t)(2 * cnt * RB));
        const int p0 = s.s0 + j0;
        const int r0 = p0 % a.cap;
        const int n1 = min(cnt, a.cap - r0);   // rows before the ring wraps
        uint8_t *dk = ring + (size_t)slot * MS_CHUNK;
        uint8_t *dv = dk + CP * RB;
        bulk_g2s(dk, kc + (size_t)r0 * D, n1 * RB, &full[slot]);
        bulk_g2s(dv, vc + (size_t)r0 * D, n1 * RB, &full[slot]);
        if (n1 < cnt) {
            bulk_g2s(dk + n1 * RB, kc, (cnt - n1) * RB, &full[slot]);
            bulk_g2s(dv + n1 * RB, vc, (cnt - n1) * RB, &full[slot]);
        }
    }
}

// ---------------------------------------------------------------- consumers
// phase input into the fragment order, consumer threads only: one 16-byte
// load of x (and of the norm weights) per thread and pass, the RMSNorm with
// the oracle's association (Ta element-strided partials, butterfly within
// each warp, warp totals in order), and the per-group sums of x from eight
// lanes' shuffles (a group of 64 is eight consecutive threads' vectors)
template <bool NORM>
MLXD_DEV void ms_stage_x(const uint16_t *x, const uint16_t *nw, int cols, float eps, uint32_t *xp,
                         float *xs, uint16_t *xraw, float *s_red) {
    constexpr int G = 64, XW = 8, MAXV = 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nv = cols / 8;
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
    const uint4 *w4 = reinterpret_cast<const uint4 *>(nw);
    float inv = 1.f;
    if (NORM) {
        // raw x for the strided sum of squares
        for (int base = 0; base < nv; base += MS_CT * MAXV) {
            uint4 v[MAXV];
#pragma unroll
            for (int j = 0; j < MAXV; j++) {
                const int i = base + tid + j * MS_CT;
                if (i < nv) v[j] = x4[i];
            }
#pragma unroll
            for (int j = 0; j < MAXV; j++) {
                const int i = base + tid + j * MS_CT;
                if (i < nv) reinterpret_cast<uint4 *>(xraw)[i] = v[j];
            }
        }
        cbar();
        const int Ta = cols >= 1024 ? 256 : (cols >= 256 ? 128 : 32);
        float acc = 0.f;
        if (tid < Ta)
            for (int i = tid; i < cols; i += Ta) {
                const float f = bf2f(xraw[i]);
                acc = fmaf(f, f, acc);
            }
        acc = warp_sum(acc);
        if (lane == 0) s_red[warp] = acc;
        cbar();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < MS_CONSUMERS; w++) tot += s_red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)cols), eps)));
    }
    for (int base = 0; base < nv; base += MS_CT * MAXV) {
        uint4 v[MAXV], wv[MAXV];
#pragma unroll
        for (int j = 0; j < MAXV; j++) {
            const int i = base + tid + j * MS_CT;
            if (i < nv) {
                v[j] = NORM ? reinterpret_cast<const uint4 *>(xraw)[i] : x4[i];
                if (NORM) wv[j] = w4[i];
            }
        }
#pragma unroll
        for (int j = 0; j < MAXV; j++) {
            const int i = base + tid + j * MS_CT;
            uint32_t e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
            float gs = 0.f;
            if (i < nv) {
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    if (NORM) {
                        const uint32_t wq = q == 0 ? wv[j].x : q == 1 ? wv[j].y : q == 2 ? wv[j].z : wv[j].w;
                        const float lo = rbf(__fmul_rn(lo_bf(wq), rbf(__fmul_rn(lo_bf(e[q]), inv))));
                        const float hi = rbf(__fmul_rn(hi_bf(wq), rbf(__fmul_rn(hi_bf(e[q]), inv))));
                        e[q] = pack_bf2(lo, hi);
                    }
                    put_pair(xp, G, XW, i * 8 + 2 * q, e[q]);
                    gs += lo_bf(e[q]) + hi_bf(e[q]);
                }
            }
            // eight consecutive threads hold one group of 64
            gs += __shfl_xor_sync(0xffffffffu, gs, 1);
            gs += __shfl_xor_sync(0xffffffffu, gs, 2);
            gs += __shfl_xor_sync(0xffffffffu, gs, 4);
            if (i < nv && (i & 7) == 0) xs[i >> 3] = gs;
        }
    }
    cbar();
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
template <int EPI>
MLXD_DEV void ms_unit_epilogue(const MsGemvOut &o, const float *ps, int nbk, int unit, int lane) {
    constexpr int UNIT_RB = EPI == MS_EPI_SWIGLU ? 2 : 1;
    unsigned long long key = 0ull;
    if (lane < 16) {
        float acc[UNIT_RB];
#pragma unroll
        for (int u = 0; u < UNIT_RB; u++) {
            float sum = 0.f;
            for (int i = u * nbk; i < (u + 1) * nbk; i++) sum += ps[i * 16 + lane];
            acc[u] = sum;
        }
        const int row = unit * 16 + lane;
        if constexpr (EPI == MS_EPI_STORE) {
            o.y[row] = f2bf(acc[0]);
        } else if constexpr (EPI == MS_EPI_RESIDUAL) {
            o.y[row] = f2bf(__fadd_rn(bf2f(o.residual[row]), rbf(acc[0])));
        } else if constexpr (EPI == MS_EPI_SWIGLU) {
            o.y[row] = f2bf(swiglu_bf16(rbf(acc[0]), rbf(acc[1])));
        } else {
            if (o.y) o.y[row] = f2bf(acc[0]);
            key = argmax_key(rbf(acc[0]), o.row_offset + row);
        }
    }
    if constexpr (EPI == MS_EPI_LOGITS) {
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, key, s);
            key = other > key ? other : key;
        }
        if (lane == 0 && o.amax) atomicMax(o.amax, key);
    }
}

// The consumer side of one projection phase. Warps take the phase's items in
// order from a shared counter; each item's 16 (row) partial sums go to its own
// place in the unit's record, and the warp whose item completes the unit adds
// the record in item order and runs the epilogue. A ring slot is released only
// after that, so a unit record is never reused while still being read:
// MS_POOL_ITEMS >= MS_NS * MS_IPC + 2 * ipu.
template <int EPI>
__device__ __noinline__ void ms_gemv(const MsMat M, int u0, int n, long long base, const MsGemvOut o,
                                     const uint8_t *ring, uint64_t *full, uint64_t *empty,
                                     const uint32_t *xp, const float *xs, const uint32_t *s_zero,
                                     int *s_cnt, float *pool, int *s_next, volatile int *dead,
                                     int *err) {
    constexpr int UNIT_RB = EPI == MS_EPI_SWIGLU ? 2 : 1;
    const int lane = threadIdx.x & 31, t = lane & 3, gq = lane >> 2;
    const int nbk = M.cols / 512;
    const int ipu = nbk * UNIT_RB;
    const int rp = MS_POOL_ITEMS / ipu;   // unit records in the pool
#ifdef MLXD_TRACE
    unsigned long long tw_ = 0, tc_ = 0, tl_ = gtime();
#endif
    for (;;) {
        int k = 0;
        if (lane == 0) k = atomicAdd(s_next, 1);
        k = __shfl_sync(0xffffffffu, k, 0);
        if (k >= n) break;
        const long long g = base + (k >> 2);
        const int slot = ms_slot(g), sub = k & (MS_IPC - 1);
        const bool live = __all_sync(0xffffffffu, !*dead);   // warp-uniform
        if (live && !__all_sync(0xffffffffu, mbar_wait(&full[slot], ms_parity(g))) && lane == 0)
            ms_fail(dead, err);
#ifdef MLXD_TRACE
        { unsigned long long t_ = gtime(); tw_ += t_ - tl_; tl_ = t_; }
#endif
        const int unit = k / ipu;
        const int iu = k - unit * ipu;
        const int bk = iu % nbk;
        const uint8_t *sl = ring + (size_t)slot * MS_CHUNK;
        const uint4 *wt = reinterpret_cast<const uint4 *>(sl + sub * 4096) + lane;
        const uint4 sv = *(reinterpret_cast<const uint4 *>(sl + MS_IPC * 4096 + sub * 512) + lane);
        const uint32_t *xb = xp + ((size_t)bk * 32 + t) * 8;
        // four independent accumulators (one per 16-column chunk of a tile)
        float dj[4][4] = {};
#pragma unroll
        for (int p = 0; p < 8; p++) {
            const uint4 wv = wt[p * 32];
            const uint4 *xq = reinterpret_cast<const uint4 *>(gq == p ? xb + p * 32 : s_zero);
            const uint4 xa = xq[0], xc = xq[1];
            const uint32_t xv[8] = {xa.x, xa.y, xa.z, xa.w, xc.x, xc.y, xc.z, xc.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint32_t af[4] = {nib_pair(wv.x, j), nib_pair(wv.z, j), nib_pair(wv.y, j),
                                  nib_pair(wv.w, j)};
                mma_bf16_16816(dj[j], af, xv[2 * j], xv[2 * j + 1]);
            }
        }
        float d[4];
#pragma unroll
        for (int i = 0; i < 4; i++) d[i] = (dj[0][i] + dj[1][i]) + (dj[2][i] + dj[3][i]);
        const float2 xsv = *reinterpret_cast<const float2 *>(xs + bk * 8 + 2 * t);
        const float s00 = lo_bf(sv.x), b00 = hi_bf(sv.x), s01 = lo_bf(sv.y), b01 = hi_bf(sv.y);
        const float s10 = lo_bf(sv.z), b10 = hi_bf(sv.z), s11 = lo_bf(sv.w), b11 = hi_bf(sv.w);
        float y0 = s00 * d[0];
        y0 = fmaf(fmaf(-128.f, s00, b00), xsv.x, y0);
        y0 = fmaf(s01, d[1], y0);
        y0 = fmaf(fmaf(-128.f, s01, b01), xsv.y, y0);
        float y1 = s10 * d[2];
        y1 = fmaf(fmaf(-128.f, s10, b10), xsv.x, y1);
        y1 = fmaf(s11, d[3], y1);
        y1 = fmaf(fmaf(-128.f, s11, b11), xsv.y, y1);
        // the quad's four lanes hold disjoint groups of rows g, g+8
        y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
        y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
        y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
        y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
        float *ps = pool + (size_t)(unit % rp) * ipu * 16;
        if (t == 0) {
            ps[iu * 16 + gq] = y0;
            ps[iu * 16 + gq + 8] = y1;
        }
        __syncwarp();
        int done = 0;
        if (lane == 0) {
            __threadfence_block();
            const int old = atomicAdd(&s_cnt[unit % rp], 1);
            done = old + 1 == ipu;
            if (done) s_cnt[unit % rp] = 0;
        }
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done) {
            __threadfence_block();
            ms_unit_epilogue<EPI>(o, ps, nbk, u0 + unit, lane);
        }
        __syncwarp();
        if (lane == 0 && live) mbar_arrive(&empty[slot], ms_release_count(k, n));
#ifdef MLXD_TRACE
        { unsigned long long t_ = gtime(); tc_ += t_ - tl_; tl_ = t_; }
#endif
    }
    MLXD_TRACE_REC(lane == 0 && EPI == MS_EPI_SWIGLU && blockIdx.x < 16, 0x3000 + (threadIdx.x >> 5), tw_,
                   tc_, (unsigned long long)n)
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
MLXD_DEV void ms_attn_preload(const MsArgs &a, const MsLayer &Ly, int pos, float *actx) {
    const int tid = threadIdx.x;
    const int half = a.rope_dims / 2;
    const float *cs = a.rope_cs + (size_t)pos * half * 2;
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

// the consumer side of one attention phase
template <int D, int REP>
__device__ __noinline__ void ms_attention(const MsArgs &a, int l, int ph, int pos, const uint8_t *ring,
                                          uint64_t *full, uint64_t *empty, long long base,
                                          unsigned char *scratch, const float *actx, bool qk_norm,
                                          volatile int *dead) {
    constexpr int DL = D / 32;
    constexpr int RB = D * 2;
    constexpr int CP = MS_SLOT / (2 * RB);     // positions per item (a quarter chunk)
    constexpr int PB = 3;                      // positions scored together
    using RowT = typename std::conditional<DL == 4, uint2, uint32_t>::type;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const MsAttnShare s = ms_attn_share<D>(a, ph, pos);
    if (s.kh < 0) return;
    const int nck = (s.nc + CP - 1) / CP;
    const int kh = s.kh;
#ifdef MLXD_TRACE
    const unsigned long long ta0 = gtime();
    unsigned long long ta1 = 0, ta2 = 0, ta3 = 0, ta4 = 0;
#endif

    float *s_q = reinterpret_cast<float *>(scratch);                 // [REP][D]
    uint16_t *s_knew = reinterpret_cast<uint16_t *>(s_q + REP * D);  // [D]
    uint16_t *s_vnew = s_knew + D;                                   // [D]
    float *s_v = reinterpret_cast<float *>(s_vnew + D);              // [16][D] staging
    float *s_ml = s_v + MS_CONSUMERS * D;                            // [8][REP][2]
    float *s_o = s_ml + 8 * REP * 2;                                 // [8][REP][D]

    // q heads of the group, the new k (norm + rope) and the new v
    const uint16_t *qkv = a.qkv;
    for (int vi = warp; vi < REP + 2; vi += MS_CONSUMERS) {
        if (vi == REP + 1) {
            for (int d = lane; d < D; d += 32) s_vnew[d] = qkv[a.qdim + (size_t)(a.hkv + kh) * D + d];
            continue;
        }
        float *v = s_v + warp * D;
        const uint16_t *src = vi < REP ? qkv + (size_t)(kh * REP + vi) * D : qkv + a.qdim + (size_t)kh * D;
        for (int d = lane; d < D; d += 32) v[d] = bf2f(src[d]);
        __syncwarp();
        ms_norm_rope(v, D, vi < REP ? actx : actx + D, qk_norm, a.eps, actx + 2 * D, a.rope_dims);
        if (vi < REP) {
            for (int d = lane; d < D; d += 32) s_q[vi * D + d] = v[d];
        } else {
            for (int d = lane; d < D; d += 32) s_knew[d] = f2bf(v[d]);
        }
        __syncwarp();
    }
    cbar();
    if (s.sp == 0) {
        uint16_t *kc = a.kc + (size_t)l * a.layer_elems + ((size_t)kh * a.cap + pos % a.cap) * D;
        uint16_t *vc = a.vc + (size_t)l * a.layer_elems + ((size_t)kh * a.cap + pos % a.cap) * D;
        for (int d = tid; d < D; d += MS_CT) {
            kc[d] = s_knew[d];
            vc[d] = s_vnew[d];
        }
    }
#ifdef MLXD_TRACE
    ta1 = gtime();
#endif
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
            float pu[PB];
            float ps = 0.f;
#pragma unroll
            for (int u = 0; u < PB; u++) {
                pu[u] = u < nv ? exp2f(sc[r][u] - mn) : 0.f;
                ps += pu[u];
            }
            lsum[r] = lsum[r] * al + ps;
#pragma unroll
            for (int i = 0; i < DL; i++) o[r][i] *= al;
            m[r] = mn;
        }
#pragma unroll
        for (int u = 0; u < PB; u++) {
            if (u >= nv) break;
            float vf[DL];
            unpack(vr[u], vf);
            // the weights were computed per head above; recompute is cheaper
            // than keeping REP x PB of them live: p = 2^(score - m)
#pragma unroll
            for (int r = 0; r < REP; r++) {
                const float p = exp2f(sc[r][u] - m[r]);
#pragma unroll
                for (int i = 0; i < DL; i++) o[r][i] = fmaf(p, vf[i], o[r][i]);
            }
        }
    };
    for (int k = warp; k < nck; k += MS_CONSUMERS) {
        const long long g = base + (k >> 2);
        const int slot = ms_slot(g), sub = k & (MS_IPC - 1);
        const bool live = __all_sync(0xffffffffu, !*dead);   // warp-uniform
        if (live && !__all_sync(0xffffffffu, mbar_wait(&full[slot], ms_parity(g))) && lane == 0)
            ms_fail(dead, a.err);
        const uint8_t *sk = ring + (size_t)slot * MS_CHUNK + sub * CP * RB;
        const uint8_t *sv = sk + MS_IPC * CP * RB;
        const int cnt = min(CP, s.nc - k * CP);
        for (int u0 = 0; u0 < cnt; u0 += PB) {
            RowT kr[PB], vr[PB];
#pragma unroll
            for (int u = 0; u < PB; u++) {
                const int uu = min(u0 + u, cnt - 1);
                kr[u] = *reinterpret_cast<const RowT *>(sk + uu * RB + lane * DL * 2);
                vr[u] = *reinterpret_cast<const RowT *>(sv + uu * RB + lane * DL * 2);
            }
            visit(kr, vr, min(PB, cnt - u0));
        }
        __syncwarp();
        if (lane == 0 && live) mbar_arrive(&empty[slot], ms_release_count(k, nck));
    }
    // the new position (its row came from this step's projection)
    if (warp == MS_CONSUMERS - 1 && pos >= s.s0 && pos < s.s1) {
        RowT kr[PB], vr[PB];
#pragma unroll
        for (int u = 0; u < PB; u++) {
            kr[u] = *reinterpret_cast<const RowT *>(s_knew + lane * DL);
            vr[u] = *reinterpret_cast<const RowT *>(s_vnew + lane * DL);
        }
        visit(kr, vr, 1);
    }
#ifdef MLXD_TRACE
    ta2 = gtime();
#endif
    // merge the warps of this CTA into the split's partial: warps 8..15 hand
    // their state to warps 0..7, which then write theirs for the final sum
    static_assert(MS_CONSUMERS == 16, "two-round warp merge");
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
    cbar();
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
    cbar();
    if (warp < 8) put(warp);
    cbar();
    for (int idx = tid; idx < REP * D; idx += MS_CT) {
        const int r = idx / D, d = idx % D;
        float mm = -INFINITY, ll = 0.f, oo = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++)
            sm_merge(mm, ll, oo, s_ml[(w * REP + r) * 2], s_ml[(w * REP + r) * 2 + 1],
                     s_o[(w * REP + r) * D + d]);
        float *rec = a.part + ((size_t)(kh * REP + r) * a.nspl + s.sp) * (D + 4);
        rec[d] = oo;
        if (d == 0) {
            rec[D] = mm;
            rec[D + 1] = ll;
        }
    }
    // wait for every split of this kv head, then merge a slice of its outputs
    cbar();
#ifdef MLXD_TRACE
    ta3 = gtime();
#endif
    if (tid == 0) {
        __threadfence();
        atomicAdd(&a.sync[1 + kh], 1);
        if (!*dead && !ms_spin(&a.sync[1 + kh], a.nspl * (l + 1))) ms_fail(dead, a.err);
    }
    cbar();
#ifdef MLXD_TRACE
    ta4 = gtime();
#endif
    const int n_out = REP * D;
    const int o0 = (int)((long long)n_out * s.sp / a.nspl);
    const int o1 = (int)((long long)n_out * (s.sp + 1) / a.nspl);
    constexpr int MSPL = 4;   // splits per thread loaded together
    for (int base_o = o0; base_o < o1; base_o += MS_CT / 8) {
        const int oi = base_o + tid / 8, sub = tid % 8;
        float mm = -INFINITY, ll = 0.f, oo = 0.f;
        if (oi < o1) {
            const int r = oi / D, d = oi % D;
            const float *rec = a.part + (size_t)(kh * REP + r) * a.nspl * (D + 4);
            for (int sp0 = sub; sp0 < a.nspl; sp0 += 8 * MSPL) {
                float pm[MSPL], pl[MSPL], po[MSPL];
#pragma unroll
                for (int j = 0; j < MSPL; j++) {
                    const int sp = sp0 + 8 * j;
                    pm[j] = -INFINITY;
                    pl[j] = po[j] = 0.f;
                    if (sp < a.nspl) {
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
            a.att[(size_t)(kh * REP + r) * D + d] = f2bf(oo / ll);
        }
    }
#ifdef MLXD_TRACE
    MLXD_TRACE_REC(tid == 0 && l == 1, 0x5000, ta1 - ta0, ta2 - ta1, ta3 - ta2)
    MLXD_TRACE_REC(tid == 0 && l == 1, 0x5001, ta4 - ta3, gtime() - ta4, (unsigned long long)nck)
#endif
}

template <int D, int REP>
__global__ void __launch_bounds__(MS_THREADS, 1) megastep_kernel(MsArgs a, int max_cols) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(16) uint32_t s_zero[8];
    __shared__ float s_red[MS_CONSUMERS];
    __shared__ volatile int s_dead;
    __shared__ int s_next;
    const MsSmem Lo = ms_layout(max_cols, a.H, D, REP);
    uint8_t *ring = smem + Lo.ring;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lo.full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + Lo.empty);
    int *s_cnt = reinterpret_cast<int *>(smem + Lo.cnt);
    float *pool = reinterpret_cast<float *>(smem + Lo.red);
    unsigned char *scratch = smem + Lo.scratch;
    float *actx = reinterpret_cast<float *>(smem + Lo.actx);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = *a.d_pos;
    const int G = gridDim.x;

    for (int i = tid; i < MS_POOL_ITEMS; i += MS_THREADS) s_cnt[i] = 0;
    if (tid < 8) s_zero[tid] = 0u;
    if (tid == 0) {
        s_dead = 0;
        s_next = 0;
    }
    if (tid == MS_CT) {
        for (int i = 0; i < MS_NS; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], MS_IPC);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == MS_CONSUMERS) {
        // ---- producer: the CTA's weight and cache stream, in phase order
        if (lane == 0) {
            long long seq = 0;
            for (int l = 0; l < a.L; l++) {
                const MsLayer &Ly = a.layers[l];
                const int ph = 1 + 5 * l;
                ms_issue_gemv<D>(Ly.qkv, 1, ph, ring, full, empty, seq, &s_dead, a.err);
                ms_issue_attn<D>(a, l, ph + 1, pos, ring, full, empty, seq, &s_dead);
                ms_issue_gemv<D>(Ly.o, 1, ph + 2, ring, full, empty, seq, &s_dead, a.err);
                ms_issue_gemv<D>(Ly.gu, 2, ph + 3, ring, full, empty, seq, &s_dead, a.err);
                ms_issue_gemv<D>(Ly.down, 1, ph + 4, ring, full, empty, seq, &s_dead, a.err);
            }
            ms_issue_gemv<D>(a.lm, 1, 1 + 5 * a.L, ring, full, empty, seq, &s_dead, a.err);
            // every issued copy has landed before the CTA (and its shared
            // memory) goes away: the last fill of each slot
            for (long long g = seq > MS_NS ? seq - MS_NS : 0; g < seq; g++)
                if (!mbar_wait(&full[ms_slot(g)], ms_parity(g))) ms_fail(&s_dead, a.err);
        }
        return;
    }

    // ---- consumers
    uint32_t *xp = reinterpret_cast<uint32_t *>(scratch);
    const int ngmax = max_cols / 64;
    float *xs = reinterpret_cast<float *>(scratch + (size_t)ngmax * 128);
    uint16_t *xraw = reinterpret_cast<uint16_t *>(scratch + (size_t)ngmax * 128 +
                                                  (((size_t)ngmax * 4 + 15) / 16) * 16);
    long long seq = 0;
    int ph = 0;
    MLXD_TRACE_START
    auto phase_done = [&]() {
        // every consumer's global writes of this phase (ordered before thread
        // 0 by the CTA barrier, made visible by its fence), then one arrival
        cbar();
        if (tid == 0) {
            __threadfence();
            atomicAdd(&a.sync[0], 1);
        }
        MLXD_TRACE_END(0x1000 + ph)
        ph++;
    };
    auto phase_wait = [&]() {
        MLXD_TRACE_RESTART
        if (tid == 0) {
            s_next = 0;
            if (!s_dead && !ms_spin(&a.sync[0], ph * G)) ms_fail(&s_dead, a.err);
        }
        cbar();
        MLXD_TRACE_WAITED
    };
    auto gemv_n = [&](const MsMat &M, int unit_rb, int &u0) {
        int u1;
        ms_units(M.rows / 16 / unit_rb, ph, u0, u1);
        return (u1 - u0) * unit_rb * (M.cols / 512);
    };

    // embed (fwd_embed, forward.c:65-147): this CTA's slice of the token's row
    {
        int id = a.ids[0];
        if (id < 0 || id >= a.vocab) id = 0;   // a failed draw; the host rejects the step
        const int nv = a.H / 8;
        const int v0 = (int)((long long)nv * blockIdx.x / G), v1 = (int)((long long)nv * (blockIdx.x + 1) / G);
        const int ng = a.H / a.emb_g;
        for (int i = v0 + tid; i < v1; i += MS_CT) {
            const uint32_t w = a.emb_w[(size_t)id * nv + i];
            const int g = (i * 8) / a.emb_g;
            const float sc = bf2f(a.emb_s[(size_t)id * ng + g]), bi = bf2f(a.emb_b[(size_t)id * ng + g]);
            uint32_t o4[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                o4[j] = pack_bf2(__fmaf_rn(sc, (float)((w >> (8 * j)) & 0xF), bi),
                                 __fmaf_rn(sc, (float)((w >> (8 * j + 4)) & 0xF), bi));
            *reinterpret_cast<uint4 *>(a.h + (size_t)i * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
        }
        phase_done();
    }
    for (int l = 0; l < a.L; l++) {
        const MsLayer &Ly = a.layers[l];
        int u0, n;
        // q|k|v
        phase_wait();
        ms_stage_x<true>(a.h, Ly.ln1, Ly.qkv.cols, a.eps, xp, xs, xraw, s_red);
        n = gemv_n(Ly.qkv, 1, u0);
        ms_gemv<MS_EPI_STORE>(Ly.qkv, u0, n, seq, MsGemvOut{a.qkv, nullptr, nullptr, 0}, ring, full, empty,
                              xp, xs, s_zero, s_cnt, pool, &s_next, &s_dead, a.err);
        seq += (n + MS_IPC - 1) / MS_IPC;
        ms_attn_preload<D>(a, Ly, pos, actx);
        phase_done();
        // attention
        phase_wait();
        {
            constexpr int CPC = MS_CHUNK / (4 * D);   // positions per ring chunk
            const MsAttnShare sh = ms_attn_share<D>(a, ph, pos);
            ms_attention<D, REP>(a, l, ph, pos, ring, full, empty, seq, scratch, actx, Ly.qn != nullptr,
                                 &s_dead);
            seq += sh.kh < 0 ? 0 : (sh.nc + CPC - 1) / CPC;
        }
        phase_done();
        // o projection + residual
        phase_wait();
        ms_stage_x<false>(a.att, nullptr, Ly.o.cols, a.eps, xp, xs, xraw, s_red);
        n = gemv_n(Ly.o, 1, u0);
        ms_gemv<MS_EPI_RESIDUAL>(Ly.o, u0, n, seq, MsGemvOut{a.h1, a.h, nullptr, 0}, ring, full, empty, xp,
                                 xs, s_zero, s_cnt, pool, &s_next, &s_dead, a.err);
        seq += (n + MS_IPC - 1) / MS_IPC;
        phase_done();
        // gate|up + SwiGLU
        phase_wait();
        ms_stage_x<true>(a.h1, Ly.ln2, Ly.gu.cols, a.eps, xp, xs, xraw, s_red);
#ifdef MLXD_TRACE
        const unsigned long long t_staged = gtime();
#endif
        n = gemv_n(Ly.gu, 2, u0);
        ms_gemv<MS_EPI_SWIGLU>(Ly.gu, u0, n, seq, MsGemvOut{a.act, nullptr, nullptr, 0}, ring, full, empty,
                               xp, xs, s_zero, s_cnt, pool, &s_next, &s_dead, a.err);
        seq += (n + MS_IPC - 1) / MS_IPC;
#ifdef MLXD_TRACE
        const unsigned long long t_gemv = gtime();
        cbar();
        MLXD_TRACE_REC(tid == 0 && blockIdx.x < 32, 0x4000, t_staged - tr_t1_, t_gemv - t_staged, gtime() - t_gemv)
#endif
        phase_done();
        // down + residual
        phase_wait();
        ms_stage_x<false>(a.act, nullptr, Ly.down.cols, a.eps, xp, xs, xraw, s_red);
        n = gemv_n(Ly.down, 1, u0);
        ms_gemv<MS_EPI_RESIDUAL>(Ly.down, u0, n, seq, MsGemvOut{a.h, a.h1, nullptr, 0}, ring, full, empty,
                                 xp, xs, s_zero, s_cnt, pool, &s_next, &s_dead, a.err);
        seq += (n + MS_IPC - 1) / MS_IPC;
        phase_done();
    }
    // final norm + lm_head (+ greedy key)
    phase_wait();
    ms_stage_x<true>(a.h, a.fnorm, a.lm.cols, a.eps, xp, xs, xraw, s_red);
    {
        int u0;
        const int n = gemv_n(a.lm, 1, u0);
        ms_gemv<MS_EPI_LOGITS>(a.lm, u0, n, seq, MsGemvOut{a.logits, nullptr, a.amax, 0}, ring, full, empty,
                               xp, xs, s_zero, s_cnt, pool, &s_next, &s_dead, a.err);
        seq += (n + MS_IPC - 1) / MS_IPC;
    }
    phase_done();
    // step end (step_finish_kernel): token from the key, next position
    if (blockIdx.x == 0) {
        phase_wait();
        if (tid == 0) {
            if (a.amax) {
                const unsigned long long key = *a.amax;
                *a.token = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
                *a.amax = 0ull;
            }
            *a.d_pos = pos + 1;
        }
    }
}

// ------------------------------------------------------------------ host

struct MegaState {
    MsLayer *d_layers = nullptr;
    int *sync = nullptr;   // [1 + hkv]
    int *err = nullptr;
    float *part = nullptr;
    int nspl = 0, grid = 0, max_cols = 0, D = 0, rep = 0;
    size_t smem = 0;
};

template <int D, int REP>
static int ms_prepare(size_t smem, int *blocks) {
    auto k = megastep_kernel<D, REP>;
    MLXD_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    MLXD_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, k, MS_THREADS, smem));
    return 0;
}
template <int D, int REP>
static int ms_launch(const MsArgs &a, const MegaState &S, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S.grid);
    cfg.blockDim = dim3(MS_THREADS);
    cfg.dynamicSmemBytes = S.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, megastep_kernel<D, REP>, a, S.max_cols));
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
static int ms_launch_any(int D, int rep, const MsArgs &a, const MegaState &S, cudaStream_t st) {
    MLXD_MS_DISPATCH(ms_launch, a, S, st)
}

static MsMat ms_mat(const QMat &q) { return MsMat{q.tiles, q.sb8, q.rows, q.cols}; }

static bool ms_eligible(const mlxd_model *m) {
    // opt-in (MLXD_MEGASTEP=1 when the model is created): on Qwen3-8B the
    // per-op kernels with programmatic dependent launch are still faster
    const char *e = getenv("MLXD_MEGASTEP");
    if (!e || atoi(e) == 0) return false;
    const mlxd_model_config &c = m->c;
    if (c.tp_size > 1 || c.attn_gate || c.qbits != 4) return false;
    if (!m->embed.quant || m->embed.sdtype != MLXD_BF16 || c.hidden % c.qgroup) return false;
    const int rep = m->hq / m->hkv;
    if (!(c.head_dim == 128 || c.head_dim == 64) || !(rep == 1 || rep == 2 || rep == 4 || rep == 8))
        return false;
    auto ok = [](const QMat &q) { return q.quant && q.fast8() && q.sb8 && q.rows % 16 == 0; };
    for (const Layer &L : m->L)
        if (!ok(L.qkv) || !ok(L.o) || !ok(L.gateup) || !ok(L.down) || L.gateup.rows % 32) return false;
    return ok(m->lm);
}

void megastep_free(mlxd_model *m) {
    MegaState *S = static_cast<MegaState *>(m->mega);
    if (!S) return;
    dev_free(S->d_layers);
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
    S->smem = ms_layout(S->max_cols, c.hidden, S->D, S->rep).total;
    int blocks = 0;
    if (S->nspl < 1 || S->smem > 227 * 1024 || ms_prepare_any(S->D, S->rep, S->smem, &blocks) || blocks < 1) {
        delete S;   // the layer-by-layer kernels serve this model
        return 0;
    }
    std::vector<MsLayer> hl(c.layers);
    for (int l = 0; l < c.layers; l++) {
        const Layer &L = m->L[l];
        hl[l] = MsLayer{ms_mat(L.qkv), ms_mat(L.o), ms_mat(L.gateup), ms_mat(L.down),
                        L.ln1, L.ln2, c.qk_norm ? L.qn : nullptr, c.qk_norm ? L.kn : nullptr};
    }
    S->d_layers = (MsLayer *)dev_alloc(hl.size() * sizeof(MsLayer));
    S->sync = (int *)dev_alloc((size_t)(1 + m->hkv) * sizeof(int));
    S->err = (int *)dev_alloc(sizeof(int));
    S->part = (float *)dev_alloc((size_t)m->hq * S->nspl * (S->D + 4) * sizeof(float));
    m->mega = S;
    if (!S->d_layers || !S->sync || !S->err || !S->part ||
        !cuda_ok(cudaMemcpy(S->d_layers, hl.data(), hl.size() * sizeof(MsLayer), cudaMemcpyHostToDevice),
                 "megastep layers") ||
        !cuda_ok(cudaMemset(S->err, 0, sizeof(int)), "megastep err")) {
        megastep_free(m);
        return -1;
    }
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
    MsArgs a = {};
    a.layers = S.d_layers;
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
    a.kc = kv->k;
    a.vc = kv->v;
    a.layer_elems = (size_t)kv->hkv * kv->cap * kv->d;
    a.cap = kv->cap;
    a.window = kv->window;
    a.d_pos = kv->d_pos;
    a.ids = ids_dev;
    a.amax = argmax ? m->amax : nullptr;
    a.token = m->token;
    a.logits = logits;
    a.h = m->h;
    a.h1 = m->h1;
    a.qkv = m->qkv;
    a.att = m->att;
    a.act = m->act;
    a.part = S.part;
    a.sync = S.sync;
    a.nspl = S.nspl;
    a.err = S.err;
    MLXD_CHECK(cudaMemsetAsync(S.sync, 0, (size_t)(1 + m->hkv) * sizeof(int), st));
    return ms_launch_any(S.D, S.rep, a, S, st);
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
