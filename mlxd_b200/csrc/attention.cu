// Attention: mlx_fast_scaled_dot_product_attention as fwd_attention calls it
// (src/engine/forward.c:713-731), with the q/k RMSNorm + RoPE of :591-697 and
// the KV append of kvcache.c:98-180 fused into the decode kernel.
//
// One arithmetic for decode and prefill (the oracle restates it): for a
// query q at position i over the keys it attends (causal, bottom-right
// aligned; with a window w, positions (i - w, i]),
//   q_d' = f32(scale * q_d), scale = 1/sqrtf(D);
//   z_j  = fmaf chain over d = 0..D-1 of q_d' * k_jd;
//   per block of 64 absolute positions [64b, 64b + 64) holding attended
//   keys: m_b = max z_j, p_j = own_expf(z_j - m_b), l_b = in-order f32 sum
//   of p_j, o_bd = fmaf chain of p_j v_jd in key order;
//   the blocks merge in key order into f64 (M, L, O_d): the first sets
//   them; a block with m_b > M first scales by s = own_expf(M - m_b):
//   L = fma(L, s, l_b), O_d = fma(O_d, s, o_bd), M = m_b; any other adds
//   with e = own_expf(m_b - M): L = fma(l_b, e, L), O_d = fma(o_bd, e, O_d);
//   out_d = bf16(O_d / L), rounded once.
// A block is finished before the merge reads it, so a decode step splits the
// blocks over CTAs with no exchange between them, a prefill tile walks the
// keys once, and both give the same bits at the same position. Head dims
// other than 64/128 take mlx's composed fallback (q scaled in bf16, bf16
// scores, precise softmax rounded to bf16, bf16 output).
#include <cooperative_groups.h>
#include <mutex>
#include <stdlib.h>
#include <vector>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(attention)

constexpr int AB = 64;            // key block of the arithmetic (absolute positions)

// byte offset of 16-byte chunk c of row r in a 64-row block of D bf16 rows,
// chunks XOR-swizzled by the row so that a warp reading one chunk of 8 rows
// (or 32 consecutive pairs of one row) hits every bank once
template <int D>
MLXD_DEV int blk_off(int r, int c) {
    return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

// ======================================================== decode (S = 1)
//
// Grid (NS, hkv): CTA (r, kh) takes a contiguous share of the attended
// blocks (lo/64 .. pos/64) of kv head kh. Its K and V blocks stream through
// rings of DR slots (cp.async); the first round is requested before waiting
// on the q|k|v projection, on which none of it depends, so the cache streams
// while the projection finishes. After the wait, warp h normalises and
// rotates q head h in registers (lane l holds features l, l + 32, ...: the
// oracle's per-head RMSNorm association, and rotation pairs i, i + D/2 in
// one lane); the CTA holding the new position also does the new k, whose
// row (and v's) replaces the not yet appended cache row in its slot. Per
// round of DR blocks: thread (position, slot) runs the REP score chains;
// per (block, head) the maximum; p in place; thread (feature pair, slot)
// runs the 2 REP o chains and one l chain of its block. Each block's
// (m_b, l_b, o_b) goes to the cache's step partials in global memory; the
// last CTA of the kv head to finish (a counter) merges the group's blocks
// in key order and writes the outputs. No CTA waits for another.
constexpr int DA_THREADS = 256;
constexpr int DR = DA_THREADS / AB;   // blocks per round (thread = position in phase A)

struct DaLayout {
    size_t kring, vring, qs, stage, newkv, sc, red, inbox, total;
};
// inbox_floats: the cluster path's inbox (block results of the CTA's output
// slice), 0 on the global path
static __host__ __device__ inline DaLayout da_layout(int D, int REP, size_t inbox_floats = 0) {
    DaLayout l;
    l.kring = 0;
    l.vring = l.kring + (size_t)DR * AB * D * 2;
    l.qs = l.vring + (size_t)DR * AB * D * 2;
    l.stage = l.qs + (size_t)REP * D * 4;
    l.newkv = l.stage + (size_t)8 * D * 4;
    l.sc = l.newkv + (size_t)2 * D * 2;
    l.red = l.sc + (size_t)DR * AB * REP * 4;
    l.inbox = l.red + (size_t)8 * REP * 4 + 16;
    l.total = l.inbox + inbox_floats * 4;
    return l;
}

// cluster path: blocks an inbox holds, and its floats (per block the CTA's
// slice of o, then m and l of the slice's head)
constexpr int DA_NBX = 128;
template <int D, int REP, int CL>
__host__ __device__ constexpr int da_es() { return CL > 0 ? REP * D / CL : 2; }
template <int D, int REP, int CL>
__host__ __device__ constexpr size_t da_inbox_floats(int nbx) { return (size_t)nbx * (da_es<D, REP, CL>() + 2); }

MLXD_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
MLXD_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

static __device__ int g_attn_err;

// One head vector (warp-wide, DS = D/32 features per lane at d = lane + 32 i):
// optional RMSNorm (fmaf partials in element order per lane, butterfly,
// precise 1/sqrt), RoPE with rotation pairs (i, i + DS/2) in the lane, every
// result rounded to bf16 as the oracle rounds it.
template <int DS>
MLXD_DEV void norm_rope_regs(float (&v)[DS], const float (&nw)[DS], bool norm, float eps, const float (&c)[DS / 2],
                             const float (&sn)[DS / 2], int D) {
    if (norm) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < DS; i++) acc = fmaf(v[i], v[i], acc);
        acc = warp_sum(acc);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), eps)));
#pragma unroll
        for (int i = 0; i < DS; i++) v[i] = rbf(__fmul_rn(nw[i], rbf(__fmul_rn(v[i], inv))));
    }
#pragma unroll
    for (int i = 0; i < DS / 2; i++) {
        const float x1 = v[i], x2 = v[i + DS / 2];
        v[i] = rbf(__fsub_rn(__fmul_rn(x1, c[i]), __fmul_rn(x2, sn[i])));
        v[i + DS / 2] = rbf(__fadd_rn(__fmul_rn(x1, sn[i]), __fmul_rn(x2, c[i])));
    }
}

// REP consecutive floats from shared memory
template <int REP>
MLXD_DEV void lds_rep(float (&o)[REP], const float *p) {
    if constexpr (REP % 4 == 0) {
#pragma unroll
        for (int i = 0; i < REP; i += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(p + i);
            o[i] = v.x;
            o[i + 1] = v.y;
            o[i + 2] = v.z;
            o[i + 3] = v.w;
        }
    } else if constexpr (REP == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        o[0] = v.x;
        o[1] = v.y;
    } else {
#pragma unroll
        for (int i = 0; i < REP; i++) o[i] = p[i];
    }
}

// CL = 0: the global path (block results in the cache's step partials, the
// last CTA of the head group merges); CL > 0: one cluster of CL CTAs per kv
// head, block results pushed into the inbox of the CTA owning each output
// slice (distributed shared memory), one cluster barrier, every CTA merges
// its slice
template <int D, int REP, int CL>
__global__ void __launch_bounds__(DA_THREADS, 1) attn_decode_kernel(AttnDecodeArgs a) {
    constexpr int NCH = D / 8;               // 16-byte chunks per row
    constexpr int NP = D / 2;                // feature pairs
    constexpr int DS = D / 32;
    constexpr int ES = CL > 0 ? da_es<D, REP, CL>() : 2;   // outputs per CTA slice (cluster path)
    static_assert(CL == 0 || (ES % 2 == 0 && D % ES == 0), "a slice holds whole feature pairs of one head");
    const int NS = gridDim.x, rank = blockIdx.x, kh = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    extern __shared__ __align__(128) unsigned char sm[];
    const DaLayout Ly = da_layout(D, REP, CL > 0 ? da_inbox_floats<D, REP, CL>(a.nbmax) : 0);
    float *inbox_o = reinterpret_cast<float *>(sm + Ly.inbox);            // [nbmax][ES]
    float *inbox_ml = inbox_o + (size_t)a.nbmax * ES;                      // [nbmax][2]
    namespace cg = cooperative_groups;
    if constexpr (CL > 0) cluster_arrive_relaxed();   // every CTA of the cluster has started
    unsigned char *kring = sm + Ly.kring, *vring = sm + Ly.vring;
    float *qs = reinterpret_cast<float *>(sm + Ly.qs);          // [D][REP], scaled
    float *stage = reinterpret_cast<float *>(sm + Ly.stage) + (size_t)warp * D;
    uint16_t *newk = reinterpret_cast<uint16_t *>(sm + Ly.newkv), *newv = newk + D;
    float *sc = reinterpret_cast<float *>(sm + Ly.sc);          // [DR][AB][REP]: z, then p
    float *red = reinterpret_cast<float *>(sm + Ly.red);        // [8 warps][REP]
    int *s_last = reinterpret_cast<int *>(red + 8 * REP);
    MLXD_TRACE_START

    const int pos = *a.d_pos;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int bfirst = lo / AB, blast = pos / AB, nbt = blast - bfirst + 1;
    const int mb0 = bfirst + (int)((long long)nbt * rank / NS), mb1 = bfirst + (int)((long long)nbt * (rank + 1) / NS);
    int nbm = mb1 - mb0;
    if (nbt > a.nbmax) {   // cannot happen for a cache sized by the host; report and do no work
        if (tid == 0) atomicExch(&g_attn_err, 1);
        nbm = 0;
    }
    const bool has_new = nbm > 0 && mb0 <= blast && blast < mb1;
    const uint16_t *kc = a.kc + (size_t)kh * a.cap * D;
    const uint16_t *vc = a.vc + (size_t)kh * a.cap * D;

    // block i (< nbm) of K (isv 0) or V into ring slot i % DR; rows outside
    // [lo, pos) zero-filled (the new position's row comes from this step)
    auto load_block = [&](int i, bool isv) {
        if (i >= nbm) return;
        const int b = mb0 + i;
        unsigned char *dst = (isv ? vring : kring) + (size_t)(i % DR) * AB * D * 2;
        const uint16_t *src = isv ? vc : kc;
        const int slot0 = (b * AB) % a.cap;   // cache slot of the block's first position
        for (int e = tid; e < AB * NCH; e += DA_THREADS) {
            const int r = e / NCH, c = e % NCH;
            const int j = b * AB + r;
            const bool valid = j >= lo && j < pos;
            int sl = slot0 + r;
            if (sl >= a.cap) sl -= a.cap;
            cp_async16_zfill(dst + blk_off<D>(r, c), src + (size_t)(valid ? sl : 0) * D + c * 8, valid);
        }
    };
    for (int i = 0; i < DR; i++) load_block(i, false);
    cp_async_commit();
    for (int i = 0; i < DR; i++) load_block(i, true);
    cp_async_commit();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    const bool regs_rope = a.rope.rope_dims == D;
    float nwq[DS], nwk[DS], rc[DS / 2], rs[DS / 2];
    if (regs_rope) {
        const float *cs = a.rope.cs + (size_t)pos * (D / 2) * 2;
#pragma unroll
        for (int i = 0; i < DS; i++) {
            nwq[i] = a.qn ? bf2f(a.qn[lane + 32 * i]) : 1.f;
            nwk[i] = a.kn ? bf2f(a.kn[lane + 32 * i]) : 1.f;
        }
#pragma unroll
        for (int i = 0; i < DS / 2; i++) {
            rc[i] = cs[2 * (lane + 32 * i)];
            rs[i] = cs[2 * (lane + 32 * i) + 1];
        }
    }
    pdl_trigger();
    pdl_wait();
    MLXD_TRACE_WAITED
    if constexpr (CL > 0) cluster_wait();

    // q heads (and the new k) of the group: warp h takes heads h, h + 8, ...
    const int qstride = D * (a.gate ? 2 : 1);
    if (nbm > 0) {
        for (int h = warp; h < REP + 1; h += 8) {
            const bool isk = h == REP;
            if (isk && !has_new) continue;
            const uint16_t *src = isk ? a.qkv + a.qdim + (size_t)kh * D : a.qkv + (size_t)(kh * REP + h) * qstride;
            if (regs_rope) {
                float v[DS];
#pragma unroll
                for (int i = 0; i < DS; i++) v[i] = bf2f(src[lane + 32 * i]);
                norm_rope_regs<DS>(v, isk ? nwk : nwq, isk ? a.kn != nullptr : a.qn != nullptr, a.eps, rc, rs, D);
                if (isk) {
                    const uint16_t *vsrc = a.qkv + a.qdim + (size_t)(a.hkv + kh) * D;
#pragma unroll
                    for (int i = 0; i < DS; i++) {
                        newk[lane + 32 * i] = f2bf(v[i]);
                        newv[lane + 32 * i] = vsrc[lane + 32 * i];
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < DS; i++) qs[(lane + 32 * i) * REP + h] = __fmul_rn(scale, v[i]);
                }
            } else {
                for (int d = lane; d < D; d += 32) stage[d] = bf2f(src[d]);
                __syncwarp();
                head_norm_rope(stage, D, isk ? a.kn : a.qn, a.eps, a.rope.cs, a.rope.rope_dims, pos);
                if (isk) {
                    const uint16_t *vsrc = a.qkv + a.qdim + (size_t)(a.hkv + kh) * D;
                    for (int d = lane; d < D; d += 32) {
                        newk[d] = f2bf(stage[d]);
                        newv[d] = vsrc[d];
                    }
                } else {
                    for (int d = lane; d < D; d += 32) qs[d * REP + h] = __fmul_rn(scale, stage[d]);
                }
                __syncwarp();
            }
        }
    }

    MLXD_TRACE_T(tr_q_)
    const int pp = tid % AB, s1 = tid / AB;      // phase A: (position, slot)
    const int dp = tid % NP, s2 = tid / NP;      // phase B: (feature pair, slot)
    const size_t gbase = (size_t)kh * a.nbmax;   // the head group's block results
#ifdef MLXD_TRACE
    unsigned long long tr_r_[4] = {0, 0, 0, 0};
#define DA_TR(i) if (r0 == 0) tr_r_[i] = gtime();
#else
#define DA_TR(i)
#endif
    for (int r0 = 0; r0 < nbm; r0 += DR) {
        cp_async_wait<1>();   // this round's K (V may still be in flight)
        __syncthreads();      // (first round: also orders the q and new-k stores)
        DA_TR(0)
        if (has_new && blast - mb0 >= r0 && blast - mb0 < r0 + DR) {
            unsigned char *blk = kring + (size_t)((blast - mb0) % DR) * AB * D * 2;
            const int r = pos - blast * AB;
            for (int c = tid; c < NCH; c += DA_THREADS)
                *reinterpret_cast<uint4 *>(blk + blk_off<D>(r, c)) = *reinterpret_cast<const uint4 *>(newk + c * 8);
            __syncthreads();
        }
        // phase A: scores of position pp of block r0 + s1, all REP heads
        const int i = r0 + s1;
        float z[REP];
        if (i < nbm) {
            const unsigned char *blk = kring + (size_t)s1 * AB * D * 2;
            float acc[REP];
#pragma unroll
            for (int h = 0; h < REP; h++) acc[h] = 0.f;
#pragma unroll 2
            for (int c = 0; c < NCH; c++) {
                const uint4 kv = *reinterpret_cast<const uint4 *>(blk + blk_off<D>(pp, c));
                const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float kf = (e & 1) ? hi_bf(kw[e >> 1]) : lo_bf(kw[e >> 1]);
                    float q[REP];
                    lds_rep<REP>(q, qs + (c * 8 + e) * REP);
#pragma unroll
                    for (int h = 0; h < REP; h++) acc[h] = __fmaf_rn(q[h], kf, acc[h]);
                }
            }
            const int j = (mb0 + i) * AB + pp;
            const bool valid = j >= lo && j <= pos;
#pragma unroll
            for (int h = 0; h < REP; h++) z[h] = valid ? acc[h] : -INFINITY;
        } else {
#pragma unroll
            for (int h = 0; h < REP; h++) z[h] = -INFINITY;
        }
        // block maxima: the two warps of a slot
#pragma unroll
        for (int h = 0; h < REP; h++) {
            const float v = warp_max(z[h]);
            if (lane == 0) red[warp * REP + h] = v;
        }
        __syncthreads();
        // the K ring is free: the next round's K blocks stream during the rest
        if (r0 + DR < nbm) {
            for (int s = 0; s < DR; s++) load_block(r0 + DR + s, false);
        }
        cp_async_commit();
#pragma unroll
        for (int h = 0; h < REP; h++) {
            const float mb = fmaxf(red[(2 * s1) * REP + h], red[(2 * s1 + 1) * REP + h]);
            sc[(s1 * AB + pp) * REP + h] = z[h] == -INFINITY ? 0.f : own_expf(__fsub_rn(z[h], mb));
        }
        DA_TR(1)
        cp_async_wait<1>();   // this round's V
        __syncthreads();
        DA_TR(2)
        if (has_new && blast - mb0 >= r0 && blast - mb0 < r0 + DR) {
            unsigned char *blk = vring + (size_t)((blast - mb0) % DR) * AB * D * 2;
            const int r = pos - blast * AB;
            for (int c = tid; c < NCH; c += DA_THREADS)
                *reinterpret_cast<uint4 *>(blk + blk_off<D>(r, c)) = *reinterpret_cast<const uint4 *>(newv + c * 8);
            __syncthreads();
        }
        // phase B: thread (dp, s2) runs the o chains of feature pair dp of
        // block r0 + s2 for all heads, and the l chain of head dp (dp < REP)
        const int ib = r0 + s2;
        if (s2 < DR && ib < nbm) {
            const unsigned char *blk = vring + (size_t)s2 * AB * D * 2;
            const float *ps = sc + (size_t)s2 * AB * REP;
            const int c = dp >> 2, off = (dp & 3) * 4;
            const int lh = dp < REP ? dp : 0;
            float o0[REP], o1[REP], l = 0.f;
#pragma unroll
            for (int h = 0; h < REP; h++) o0[h] = o1[h] = 0.f;
#pragma unroll 4
            for (int q = 0; q < AB; q++) {
                float pv[REP];
                lds_rep<REP>(pv, ps + q * REP);
                const uint32_t v2 = *reinterpret_cast<const uint32_t *>(blk + blk_off<D>(q, c) + off);
                const float va = lo_bf(v2), vb = hi_bf(v2);
#pragma unroll
                for (int h = 0; h < REP; h++) {
                    o0[h] = __fmaf_rn(pv[h], va, o0[h]);
                    o1[h] = __fmaf_rn(pv[h], vb, o1[h]);
                }
                l = __fadd_rn(l, ps[q * REP + lh]);
            }
            const int bi = mb0 + ib - bfirst;
            if constexpr (CL == 0) {
                const size_t gb = (gbase + (size_t)bi) * REP;
#pragma unroll
                for (int h = 0; h < REP; h++)
                    *reinterpret_cast<float2 *>(a.part_o + (gb + h) * D + 2 * dp) = make_float2(o0[h], o1[h]);
                if (dp < REP) {
                    a.part_l[gb + dp] = l;
                    a.part_m[gb + dp] = fmaxf(red[(2 * s2) * REP + dp], red[(2 * s2 + 1) * REP + dp]);
                }
            } else {
                cg::cluster_group cluster = cg::this_cluster();
#pragma unroll
                for (int h = 0; h < REP; h++) {
                    const int e = h * D + 2 * dp, dst = e / ES;
                    *reinterpret_cast<float2 *>(cluster.map_shared_rank(inbox_o + (size_t)bi * ES + (e - dst * ES),
                                                                        dst)) = make_float2(o0[h], o1[h]);
                }
                if (dp < REP) {
                    const float2 ml = make_float2(fmaxf(red[(2 * s2) * REP + dp], red[(2 * s2 + 1) * REP + dp]), l);
                    for (int r = dp * (D / ES); r < (dp + 1) * (D / ES); r++)
                        *reinterpret_cast<float2 *>(cluster.map_shared_rank(inbox_ml + (size_t)bi * 2, r)) = ml;
                }
            }
        }
        __syncthreads();
        DA_TR(3)
        if (r0 + DR < nbm) {
            for (int s = 0; s < DR; s++) load_block(r0 + DR + s, true);
        }
        cp_async_commit();
    }
#undef DA_TR
    MLXD_TRACE_REC(tid == 0 && nbm > 0, 0x25, tr_r_[0], tr_r_[1], tr_r_[2])
    MLXD_TRACE_REC(tid == 0 && nbm > 0, 0x26, tr_r_[3], tr_q_, (unsigned long long)nbm)
    cp_async_wait<0>();
    MLXD_TRACE_T(tr_ab_)
    // the new position's k/v rows into the cache
    if (has_new) {
        uint16_t *kd = a.kc + ((size_t)kh * a.cap + pos % a.cap) * D;
        uint16_t *vd = a.vc + ((size_t)kh * a.cap + pos % a.cap) * D;
        for (int d = tid; d < D; d += DA_THREADS) {
            kd[d] = newk[d];
            vd[d] = newv[d];
        }
    }
    if constexpr (CL > 0) {
        // every block result is in its owner's inbox after the barrier; this
        // CTA merges its slice (outputs rank*ES .. +ES of the group, one head)
        cg::this_cluster().sync();
        MLXD_TRACE_T(tr_cs_)
        const int e0 = rank * ES, hh = e0 / D, d0 = e0 % D;
        const int nmerge = nbt <= a.nbmax ? nbt : 0;
        float *f_s = reinterpret_cast<float *>(sm + Ly.kring);   // the rings are free
        int *g_s = reinterpret_cast<int *>(f_s + DA_NBX);
        for (int b = tid; b < nmerge; b += DA_THREADS) {
            float mp = -INFINITY;
            for (int bb = 0; bb < b; bb++) mp = fmaxf(mp, inbox_ml[2 * bb]);
            const float mb = inbox_ml[2 * b];
            int g = 0;
            float f = 1.f;
            if (mp != -INFINITY) {
                g = mb > mp ? 1 : 2;
                f = own_expf(g == 1 ? __fsub_rn(mp, mb) : __fsub_rn(mb, mp));
            }
            f_s[b] = f;
            g_s[b] = g;
        }
        __syncthreads();
        for (int p = tid; p < ES / 2; p += DA_THREADS) {
            double L = 0.0, O0 = 0.0, O1 = 0.0;
#pragma unroll 4
            for (int b = 0; b < nmerge; b++) {
                const float2 o = *reinterpret_cast<const float2 *>(inbox_o + (size_t)b * ES + 2 * p);
                const double l = (double)inbox_ml[2 * b + 1], f = (double)f_s[b];
                const int g = g_s[b];
                if (g == 0) {
                    L = l;
                    O0 = (double)o.x;
                    O1 = (double)o.y;
                } else if (g == 1) {
                    L = __fma_rn(L, f, l);
                    O0 = __fma_rn(O0, f, (double)o.x);
                    O1 = __fma_rn(O1, f, (double)o.y);
                } else {
                    L = __fma_rn(l, f, L);
                    O0 = __fma_rn((double)o.x, f, O0);
                    O1 = __fma_rn((double)o.y, f, O1);
                }
            }
            const int hg = kh * REP + hh, d = d0 + 2 * p;
            uint16_t v0 = d2bf(O0 / L), v1 = d2bf(O1 / L);
            if (a.gate) {
                const uint16_t *gp = a.qkv + (size_t)hg * qstride + D + d;
                v0 = f2bf(__fmul_rn(bf2f(v0), sigmoid_bf16(bf2f(gp[0]))));
                v1 = f2bf(__fmul_rn(bf2f(v1), sigmoid_bf16(bf2f(gp[1]))));
            }
            *reinterpret_cast<uint32_t *>(a.out + (size_t)hg * D + d) = (uint32_t)v0 | ((uint32_t)v1 << 16);
        }
        MLXD_TRACE_T(tr_ce_)
        MLXD_TRACE_REC(tid == 0, 0x27, tr_ab_, tr_cs_, tr_ce_)
        MLXD_TRACE_END(0x24)
        return;
    }
    // the last CTA of the head group merges its blocks
    __threadfence();
    __syncthreads();
    if (tid == 0) *s_last = atomicAdd(a.cnt + kh, 1) == NS - 1;
    __syncthreads();
    MLXD_TRACE_T(tr_arr_)
    MLXD_TRACE_REC(tid == 0, 0x22, tr_q_, tr_ab_, tr_arr_)
    if (!*s_last) {
        MLXD_TRACE_END(0x20)
        return;
    }
    MLXD_TRACE_RESTART
    __threadfence();
    const int nmerge = nbt <= a.nbmax ? nbt : 0;
    // The merge runs in chunks of MCH blocks staged in shared memory (the
    // rings are free): the blocks' results are loaded together, each
    // (block, head) gets its factor from the running maximum before it (a
    // prefix maximum, in parallel), then thread (head, feature pair) runs its
    // f64 chain over the chunk in key order.
    constexpr int MCH = (2 * DR * AB * D * 2 - 64 * 4) / (REP * (D + 4) * 4) / 4 * 4;
    constexpr int NE = (REP * NP + DA_THREADS - 1) / DA_THREADS;
    float *o_s = reinterpret_cast<float *>(sm);                 // [MCH][REP][D]
    float *m_s = o_s + (size_t)MCH * REP * D;                    // [MCH][REP] (+ REP: the chunk's maximum)
    float *l_s = m_s + MCH * REP + 16;
    float *f_s = l_s + MCH * REP;
    int *g_s = reinterpret_cast<int *>(f_s + MCH * REP);         // 1 new maximum (or first), 2 other
    float *Mrun = reinterpret_cast<float *>(g_s + MCH * REP);    // [REP]
    double L[NE], O0[NE], O1[NE];
#pragma unroll
    for (int q = 0; q < NE; q++) L[q] = O0[q] = O1[q] = 0.0;
    if (tid < REP) Mrun[tid] = -INFINITY;
    for (int c0 = 0; c0 < nmerge; c0 += MCH) {
        const int nb = min(MCH, nmerge - c0);
        __syncthreads();   // the previous chunk is consumed (first: Mrun is set)
        // the chunk's results into shared memory, every copy in flight at once
        const size_t r0 = (gbase + c0) * REP;
        const float *src = a.part_o + r0 * D;
        for (int i = tid; i < nb * REP * D / 4; i += DA_THREADS) cp_async16(o_s + 4 * i, src + 4 * i);
        cp_async_commit();
        for (int i = tid; i < nb * REP; i += DA_THREADS) {
            m_s[i] = __ldcg(a.part_m + r0 + i);
            l_s[i] = __ldcg(a.part_l + r0 + i);
        }
        cp_async_wait<0>();
        __syncthreads();
        MLXD_TRACE_T(tr_ld_)
        // factor of (block b, head h): the running maximum before it is the
        // maximum of the earlier blocks; the thread of the chunk's last block
        // also leaves the maximum after the chunk
        for (int i = tid; i < nb * REP; i += DA_THREADS) {
            const int b = i / REP, h = i % REP;
            float mp = Mrun[h];
            for (int bb = 0; bb < b; bb++) mp = fmaxf(mp, m_s[bb * REP + h]);
            const float mb = m_s[i];
            // first block (sums still zero): fma(0, 1, x) = x
            float f = 1.f;
            int g = 1;
            if (mp != -INFINITY) {
                g = mb > mp ? 1 : 2;
                f = own_expf(g == 1 ? __fsub_rn(mp, mb) : __fsub_rn(mb, mp));
            }
            g_s[i] = g;
            f_s[i] = f;
            if (b == nb - 1) m_s[MCH * REP + h] = fmaxf(mp, mb);
        }
        __syncthreads();
        MLXD_TRACE_T(tr_f_)
#pragma unroll
        for (int q = 0; q < NE; q++) {
            const int e = tid + q * DA_THREADS;
            if (e < REP * NP) {
                const int h = e / NP, fp = e % NP;
#pragma unroll 8
                for (int b = 0; b < nb; b++) {
                    const int i = b * REP + h;
                    const float2 o = *reinterpret_cast<const float2 *>(o_s + (size_t)i * D + 2 * fp);
                    const double l = (double)l_s[i], f = (double)f_s[i];
                    // new maximum: S = fma(S, s, x); otherwise S = fma(x, e, S)
                    const bool nm = g_s[i] == 1;
                    L[q] = __fma_rn(nm ? L[q] : l, f, nm ? l : L[q]);
                    O0[q] = __fma_rn(nm ? O0[q] : (double)o.x, f, nm ? (double)o.x : O0[q]);
                    O1[q] = __fma_rn(nm ? O1[q] : (double)o.y, f, nm ? (double)o.y : O1[q]);
                }
            }
        }
        __syncthreads();
        MLXD_TRACE_T(tr_c_)
        MLXD_TRACE_REC(tid == 0 && c0 == 0, 0x23, tr_ld_, tr_f_, tr_c_)
        if (tid < REP) Mrun[tid] = m_s[MCH * REP + tid];
    }
#pragma unroll
    for (int q = 0; q < NE; q++) {
        const int e = tid + q * DA_THREADS;
        if (e >= REP * NP) continue;
        const int h = e / NP, fp = e % NP;
        const int hg = kh * REP + h;
        uint16_t v0 = d2bf(O0[q] / L[q]), v1 = d2bf(O1[q] / L[q]);
        if (a.gate) {
            const uint16_t *gp = a.qkv + (size_t)hg * qstride + D + 2 * fp;
            v0 = f2bf(__fmul_rn(bf2f(v0), sigmoid_bf16(bf2f(gp[0]))));
            v1 = f2bf(__fmul_rn(bf2f(v1), sigmoid_bf16(bf2f(gp[1]))));
        }
        *reinterpret_cast<uint32_t *>(a.out + (size_t)hg * D + 2 * fp) = (uint32_t)v0 | ((uint32_t)v1 << 16);
    }
    if (tid == 0) a.cnt[kh] = 0;   // ready for the next launch
    MLXD_TRACE_END(0x21)
}

// global path: CTAs per kv head, as many as the SMs allow (one block each
// at most, if the span is short), all kv heads' CTAs on distinct SMs
static int da_splits(const AttnDecodeArgs &a) {
    const int sms = num_sms();
    int ns = a.nbmax;
    const int cap_ns = sms / a.hkv > 0 ? sms / a.hkv : 1;
    if (ns > cap_ns) ns = cap_ns;
    return ns < 1 ? 1 : ns;
}

// One CTA per SM (dynamic shared memory above half of an SM's): with two
// attention CTAs on one SM the projections that follow ran slower on those
// SMs for the rest of the step
template <int D, int REP, int CL>
static size_t da_smem(const AttnDecodeArgs &a) {
    const size_t t = da_layout(D, REP, CL > 0 ? da_inbox_floats<D, REP, CL>(a.nbmax) : 0).total;
    return t > 116 * 1024 ? t : 116 * 1024;
}

// cudaFuncSetAttribute is per device: clusters above 8 CTAs allowed once per
// (kernel, device)
static bool nonportable_allowed(const void *kern) {
    static std::mutex mu;
    static std::vector<std::pair<const void *, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (auto &e : done)
        if (e.first == kern && e.second == dev) return true;
    if (!cuda_ok(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1), "cluster attribute"))
        return false;
    done.push_back({kern, dev});
    return true;
}

template <int D, int REP, int CL>
static cudaLaunchConfig_t da_config(const AttnDecodeArgs &a, size_t smem, cudaLaunchAttribute *attr, bool pdl,
                                    cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL > 0 ? CL : da_splits(a), a.hkv);
    cfg.blockDim = dim3(DA_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    int n = 0;
    if (CL > 0) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = CL;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        n++;
    }
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cfg;
}

template <int D, int REP, int CL>
static bool da_prepare(const AttnDecodeArgs &a) {
    auto kern = attn_decode_kernel<D, REP, CL>;
    const size_t smem = da_smem<D, REP, CL>(a);
    if (smem > 227 * 1024 || !smem_allowed((const void *)kern, smem)) return false;
    return CL <= 8 || nonportable_allowed((const void *)kern);
}

// whether hkv clusters of CL CTAs are resident at once on this device
template <int D, int REP, int CL>
static bool da_fits(const AttnDecodeArgs &a) {
    if (a.nbmax > DA_NBX || !da_prepare<D, REP, CL>(a)) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = da_config<D, REP, CL>(a, da_smem<D, REP, CL>(a), attr, false, nullptr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<D, REP, CL>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n >= a.hkv;
}

// the path per (device, kv heads, inbox size): clusters of 16 when hkv of
// them are resident at once, else the global path (spans beyond the inbox
// too)
template <int D, int REP>
static int da_choice(const AttnDecodeArgs &a) {
    static std::mutex mu;
    static std::vector<std::pair<std::pair<int, long long>, int>> memo;
    int dev = 0;
    cudaGetDevice(&dev);
    const long long key = ((long long)a.hkv << 32) | (unsigned)a.nbmax;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (auto &m : memo)
            if (m.first.first == dev && m.first.second == key) return m.second;
    }
    // clusters of 8 (hkv x 8 CTAs, 4+ blocks each at 2k positions) measured
    // slower than the global path over all SMs
    const int cl = da_fits<D, REP, 16>(a) ? 16 : 0;
    std::lock_guard<std::mutex> lock(mu);
    memo.push_back({{dev, key}, cl});
    return cl;
}

template <int D, int REP, int CL>
static int da_launch_cl(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    if (!da_prepare<D, REP, CL>(a)) return -1;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = da_config<D, REP, CL>(a, da_smem<D, REP, CL>(a), attr, pdl, st);
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, REP, CL>, a));
    return 0;
}

template <int D, int REP>
static int da_launch(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    if (da_choice<D, REP>(a) == 16) return da_launch_cl<D, REP, 16>(a, st, pdl);
    return da_launch_cl<D, REP, 0>(a, st, pdl);
}

template <int D, int REP>
static int da_sms(const AttnDecodeArgs &a) {
    const int cl = da_choice<D, REP>(a);
    return (cl > 0 ? cl : da_splits(a)) * a.hkv;
}

// result floats per kv head of a cache whose attended span holds at most
// nbmax blocks: (m, l, o[D]) per (block, query head of the group)
size_t attention_decode_part_floats(int nbmax, int hkv, int rep, int D) {
    return (size_t)hkv * nbmax * rep * (D + 2);
}

bool attention_decode_supported(int D, int rep, int rope_dims) {
    return (D == 64 || D == 128) && (rep == 1 || rep == 2 || rep == 4 || rep == 8) && rope_dims <= D;
}

#define MLXD_DA_DISPATCH(FN, ...)                                                       \
    switch (D * 16 + rep) {                                                             \
    case 128 * 16 + 1: return FN<128, 1>(__VA_ARGS__);                                  \
    case 128 * 16 + 2: return FN<128, 2>(__VA_ARGS__);                                  \
    case 128 * 16 + 4: return FN<128, 4>(__VA_ARGS__);                                  \
    case 128 * 16 + 8: return FN<128, 8>(__VA_ARGS__);                                  \
    case 64 * 16 + 1: return FN<64, 1>(__VA_ARGS__);                                    \
    case 64 * 16 + 2: return FN<64, 2>(__VA_ARGS__);                                    \
    case 64 * 16 + 4: return FN<64, 4>(__VA_ARGS__);                                    \
    case 64 * 16 + 8: return FN<64, 8>(__VA_ARGS__);                                    \
    }

int attention_decode(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    const int D = a.rope.D, rep = a.hq / a.hkv;
    if (!attention_decode_supported(D, rep, a.rope.rope_dims)) {
        set_error("decode attention: head dim %d with %d query heads per kv head not supported", D, rep);
        return -1;
    }
    if (!a.part_o || !a.part_l || !a.part_m || !a.cnt || a.nbmax <= 0) {
        set_error("decode attention: the cache has no step partials");
        return -1;
    }
    MLXD_DA_DISPATCH(da_launch, a, st, pdl)
    return -1;
}

int attention_decode_sms(const AttnDecodeArgs &a) {
    const int D = a.rope.D, rep = a.hq / a.hkv;
    if (!attention_decode_supported(D, rep, a.rope.rope_dims)) return 0;
    MLXD_DA_DISPATCH(da_sms, a)
    return 0;
}
#undef MLXD_DA_DISPATCH

int attention_timeouts() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_attn_err, sizeof v) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_attn_err, &z, sizeof z);
    return v;
}

// ======================================================= prefill (S > 1)
//
// CTA = (64 queries, one q head), 256 threads, one pass over the keys in
// blocks of 64 absolute positions (the union of the tile's key ranges):
//   the 64 x 64 score tile on CUDA cores, thread (tq, tk) holding queries
//   4tq.. and keys 4tk.. (16 fmaf chains stepping through d together; q'
//   and k transposed to f32 in shared memory so that each step is two
//   16-byte loads); per query the block maximum (the 16 threads of a tq);
//   p = own_expf(z - m_b) into shared memory; thread (tq, td) runs the
//   chains of queries 4tq.. x features 8td.. over the block's keys (l_b by
//   every td, the same chain) and merges the block into its f64 running
//   sums. The next block's key and value rows are requested into registers
//   while the current one is computed.
constexpr int PF_T = 256, PF_Q = 64;

template <int D>
struct PfLayout {
    static constexpr size_t qT = 0;                               // [D][64] f32
    static constexpr size_t kT = qT + (size_t)D * PF_Q * 4;        // [D][64] f32
    static constexpr size_t pT = kT + (size_t)D * AB * 4;          // [64 keys][64 q] f32
    static constexpr size_t vb = pT + (size_t)AB * PF_Q * 4;       // [64][D] bf16
    static constexpr size_t mx = vb + (size_t)AB * D * 2;          // [64] f32 block maxima
    static constexpr size_t total = mx + (size_t)PF_Q * 4;
};

template <int D>
__global__ void __launch_bounds__(PF_T) attn_prefill_kernel(const uint16_t *__restrict__ q, int S, int pos0,
                                                           const uint16_t *__restrict__ kc,
                                                           const uint16_t *__restrict__ vc, int cap, int window,
                                                           int hq, int hkv, const uint16_t *__restrict__ gate_src,
                                                           int row_stride, uint16_t *__restrict__ out) {
    using L = PfLayout<D>;
    extern __shared__ __align__(128) unsigned char sm[];
    float *qT = reinterpret_cast<float *>(sm + L::qT);
    float *kT = reinterpret_cast<float *>(sm + L::kT);
    float *pT = reinterpret_cast<float *>(sm + L::pT);
    uint16_t *vb = reinterpret_cast<uint16_t *>(sm + L::vb);
    float *smx = reinterpret_cast<float *>(sm + L::mx);
    const int tid = threadIdx.x;
    const int qt0 = blockIdx.x * PF_Q, h = blockIdx.y, kh = h / (hq / hkv);
    const int nq = min(PF_Q, S - qt0);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    // key range of the tile: union of the rows' (j0, j1]
    const int qpos_lo = pos0 + qt0, qpos_hi = pos0 + qt0 + nq - 1;
    const int jlo = window > 0 ? max(0, qpos_lo - window + 1) : 0;
    const int jhi = qpos_hi + 1;   // exclusive
    const int b0 = jlo / AB, b1 = (jhi - 1) / AB;
    const int nb = b1 - b0 + 1;
    const uint16_t *K = kc + (size_t)kh * cap * D;
    const uint16_t *V = vc + (size_t)kh * cap * D;

    // q' transposed: qT[d][i] = f32(scale * q[i][d]) (0 for rows past S)
    for (int e = tid; e < PF_Q * D; e += PF_T) {
        const int d = e / PF_Q, i = e % PF_Q;
        qT[d * PF_Q + i] = i < nq ? __fmul_rn(scale, bf2f(q[((size_t)(qt0 + i) * hq + h) * D + d])) : 0.f;
    }
    const int tq = tid >> 4, tk = tid & 15;   // scores: queries 4tq.., keys 4tk..
    int qp[4], j0r[4];
#pragma unroll
    for (int a = 0; a < 4; a++) {
        qp[a] = pos0 + qt0 + 4 * tq + a;
        j0r[a] = window > 0 ? max(0, qp[a] - window + 1) : 0;
    }
    // o/l chains: thread (tq2, td): queries QPT tq2.., features 8td..
    constexpr int FT = D / 8;           // feature groups
    constexpr int QT = PF_T / FT;       // query groups (16 for D=128, 32 for D=64)
    constexpr int QPT = PF_Q / QT;      // queries per thread (4 or 2)
    const int td = tid % FT, tq2 = tid / FT;
    float Mq[QPT];
    double O[QPT][8], Lq[QPT];
#pragma unroll
    for (int x = 0; x < QPT; x++) {
        Mq[x] = -INFINITY;
        Lq[x] = 0.0;
#pragma unroll
        for (int y = 0; y < 8; y++) O[x][y] = 0.0;
    }
    // the rows of a key or value block, 16 B per (row r, chunk c), thread
    // share e = tid + 256 x, c = e / 64, r = e % 64: requested one block
    // ahead into registers
    constexpr int NPF = AB * D / 8 / PF_T;   // 16-byte pieces per thread (4 for D = 128)
    auto fetch_rows = [&](const uint16_t *base, int b, uint4 (&buf)[NPF]) {
#pragma unroll
        for (int x = 0; x < NPF; x++) {
            const int e = tid + PF_T * x, c = e / AB, r = e % AB;
            const int j = b * AB + r;
            buf[x] = j < jhi ? *reinterpret_cast<const uint4 *>(base + (size_t)(j % cap) * D + c * 8)
                             : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    uint4 kpre[NPF], vpre[NPF];
    fetch_rows(K, b0, kpre);
    fetch_rows(V, b0, vpre);
    for (int bi = 0; bi < nb; bi++) {
        const int b = b0 + bi;
        __syncthreads();   // the previous block's kT, pT, vb and maxima are consumed
        // k block transposed to f32: kT[d][r]; the v block as it is
#pragma unroll
        for (int x = 0; x < NPF; x++) {
            const int e = tid + PF_T * x, c = e / AB, r = e % AB;
            const uint32_t w[4] = {kpre[x].x, kpre[x].y, kpre[x].z, kpre[x].w};
#pragma unroll
            for (int y = 0; y < 4; y++) {
                kT[(c * 8 + 2 * y) * AB + r] = lo_bf(w[y]);
                kT[(c * 8 + 2 * y + 1) * AB + r] = hi_bf(w[y]);
            }
            *reinterpret_cast<uint4 *>(vb + r * D + c * 8) = vpre[x];
        }
        if (bi + 1 < nb) {
            fetch_rows(K, b + 1, kpre);
            fetch_rows(V, b + 1, vpre);
        }
        __syncthreads();
        float acc[4][4] = {};
#pragma unroll 4
        for (int d = 0; d < D; d++) {
            const float4 qv = *reinterpret_cast<const float4 *>(qT + d * PF_Q + 4 * tq);
            const float4 kv = *reinterpret_cast<const float4 *>(kT + d * AB + 4 * tk);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int x = 0; x < 4; x++)
#pragma unroll
                for (int y = 0; y < 4; y++) acc[x][y] = __fmaf_rn(qa[x], ka[y], acc[x][y]);
        }
        // masks and the per-query block maxima (16 consecutive lanes per tq)
        float mrow[4];
#pragma unroll
        for (int x = 0; x < 4; x++) {
            float v = -INFINITY;
#pragma unroll
            for (int y = 0; y < 4; y++) {
                const int j = b * AB + 4 * tk + y;
                const bool ok = 4 * tq + x < nq && j >= j0r[x] && j <= qp[x];
                acc[x][y] = ok ? acc[x][y] : -INFINITY;
                v = fmaxf(v, acc[x][y]);
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            mrow[x] = v;
        }
        if (tk == 0) {
#pragma unroll
            for (int x = 0; x < 4; x++) smx[4 * tq + x] = mrow[x];
        }
        // p tile, transposed: pT[key][query]
#pragma unroll
        for (int y = 0; y < 4; y++) {
            float4 pv;
            float *pp = &pv.x;
#pragma unroll
            for (int x = 0; x < 4; x++)
                pp[x] = acc[x][y] == -INFINITY ? 0.f : own_expf(__fsub_rn(acc[x][y], mrow[x]));
            *reinterpret_cast<float4 *>(pT + (4 * tk + y) * PF_Q + 4 * tq) = pv;
        }
        __syncthreads();
        float o[QPT][8] = {}, l[QPT] = {};
#pragma unroll 2
        for (int r = 0; r < AB; r++) {
            float pv[QPT];
            if constexpr (QPT == 4) {
                const float4 p4 = *reinterpret_cast<const float4 *>(pT + r * PF_Q + QPT * tq2);
                pv[0] = p4.x; pv[1] = p4.y; pv[2] = p4.z; pv[3] = p4.w;
            } else {
                const float2 p2 = *reinterpret_cast<const float2 *>(pT + r * PF_Q + QPT * tq2);
                pv[0] = p2.x; pv[1] = p2.y;
            }
            const uint4 v4 = *reinterpret_cast<const uint4 *>(vb + r * D + td * 8);
            const uint32_t vw[4] = {v4.x, v4.y, v4.z, v4.w};
            float vf[8];
#pragma unroll
            for (int y = 0; y < 4; y++) {
                vf[2 * y] = lo_bf(vw[y]);
                vf[2 * y + 1] = hi_bf(vw[y]);
            }
#pragma unroll
            for (int x = 0; x < QPT; x++) {
#pragma unroll
                for (int y = 0; y < 8; y++) o[x][y] = __fmaf_rn(pv[x], vf[y], o[x][y]);
                l[x] = __fadd_rn(l[x], pv[x]);
            }
        }
        // merge the block (queries with attended keys in it)
#pragma unroll
        for (int x = 0; x < QPT; x++) {
            const float mb = smx[QPT * tq2 + x];
            if (mb == -INFINITY) continue;
            if (Mq[x] == -INFINITY) {
                Mq[x] = mb;
                Lq[x] = (double)l[x];
#pragma unroll
                for (int y = 0; y < 8; y++) O[x][y] = (double)o[x][y];
            } else if (mb > Mq[x]) {
                const double s = (double)own_expf(__fsub_rn(Mq[x], mb));
                Mq[x] = mb;
                Lq[x] = __fma_rn(Lq[x], s, (double)l[x]);
#pragma unroll
                for (int y = 0; y < 8; y++) O[x][y] = __fma_rn(O[x][y], s, (double)o[x][y]);
            } else {
                const double e = (double)own_expf(__fsub_rn(mb, Mq[x]));
                Lq[x] = __fma_rn((double)l[x], e, Lq[x]);
#pragma unroll
                for (int y = 0; y < 8; y++) O[x][y] = __fma_rn((double)o[x][y], e, O[x][y]);
            }
        }
    }
#pragma unroll
    for (int x = 0; x < QPT; x++) {
        const int i = QPT * tq2 + x;
        if (i >= nq) continue;
        uint16_t *dst = out + ((size_t)(qt0 + i) * hq + h) * D + td * 8;
        const uint16_t *gp = gate_src ? gate_src + (size_t)(qt0 + i) * row_stride + (size_t)h * 2 * D + D + td * 8
                                      : nullptr;
        uint32_t pk[4];
#pragma unroll
        for (int y = 0; y < 8; y += 2) {
            uint16_t v0 = d2bf(O[x][y] / Lq[x]), v1 = d2bf(O[x][y + 1] / Lq[x]);
            if (gp) {
                v0 = f2bf(__fmul_rn(bf2f(v0), sigmoid_bf16(bf2f(gp[y]))));
                v1 = f2bf(__fmul_rn(bf2f(v1), sigmoid_bf16(bf2f(gp[y + 1]))));
            }
            pk[y / 2] = (uint32_t)v0 | ((uint32_t)v1 << 16);
        }
        *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
}

// ------------------------------------------------------------ small head dims
// mlx composed fallback, one warp per (query, head): the oracle's order
// (fmaf chains over features and keys, in-order f32 softmax sum).
__global__ void attn_small_kernel(const uint16_t *__restrict__ q, int S, int pos0,
                                  const uint16_t *__restrict__ kc, const uint16_t *__restrict__ vc, int cap,
                                  int window, int hq, int hkv, int D, const uint16_t *__restrict__ gate_src,
                                  int row_stride, uint16_t *__restrict__ out, float *scratch, int tmax) {
    const int i = blockIdx.x, h = blockIdx.y, kh = h / (hq / hkv), lane = threadIdx.x;
    float *sc = scratch + ((size_t)i * hq + h) * tmax;
    const int qp = pos0 + i;
    const int T = qp + 1;
    const int j0 = window > 0 ? max(0, T - window) : 0;
    const uint16_t *qv = q + ((size_t)i * hq + h) * D;
    const uint16_t *K = kc + (size_t)kh * cap * D;
    const uint16_t *V = vc + (size_t)kh * cap * D;
    const float sbf = rbf(__fdiv_rn(1.0f, __fsqrt_rn((float)D)));
    for (int j = j0 + lane; j < T; j += 32) {
        float a = 0.f;
        for (int d = 0; d < D; d++) {
            const float qs = rbf(__fmul_rn(sbf, bf2f(qv[d])));
            a = __fmaf_rn(qs, bf2f(K[(size_t)(j % cap) * D + d]), a);
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
            const float p = rbf(__fdiv_rn(sc[j], l));
            o = __fmaf_rn(p, bf2f(V[(size_t)((j0 + j) % cap) * D + d]), o);
        }
        float val = rbf(o);
        if (gate_src) {
            const float g = bf2f(gate_src[(size_t)i * row_stride + (size_t)h * 2 * D + D + d]);
            val = rbf(__fmul_rn(val, sigmoid_bf16(g)));
        }
        out[((size_t)i * hq + h) * D + d] = f2bf(val);
    }
}

// scratch floats a prefill launch needs (the composed path for other head
// dims keeps its scores there; head dims 64 and 128 need none)
size_t attention_prefill_scratch(int S, int pos0, int window, int hq, int D) {
    if (D == 64 || D == 128) return 0;
    int tmax = pos0 + S;
    if (window > 0 && tmax > window + S) tmax = window + S;
    return (size_t)S * hq * tmax;
}

int attention_prefill(const uint16_t *q, int S, int pos0, const uint16_t *kc, const uint16_t *vc, int cap,
                      int window, int hq, int hkv, int D, const uint16_t *gate_src, int qdim, uint16_t *out,
                      float *scr, size_t scr_floats, cudaStream_t st) {
    const int row_stride = qdim + 2 * hkv * D;
    if (D == 64 || D == 128) {
        const int ntile = (S + PF_Q - 1) / PF_Q;
        dim3 grid(ntile, hq);
        if (D == 128) {
            const size_t smem = PfLayout<128>::total;
            if (!smem_allowed((const void *)attn_prefill_kernel<128>, smem)) return -1;
            attn_prefill_kernel<128><<<grid, PF_T, smem, st>>>(q, S, pos0, kc, vc, cap, window, hq, hkv, gate_src,
                                                               row_stride, out);
        } else {
            const size_t smem = PfLayout<64>::total;
            if (!smem_allowed((const void *)attn_prefill_kernel<64>, smem)) return -1;
            attn_prefill_kernel<64><<<grid, PF_T, smem, st>>>(q, S, pos0, kc, vc, cap, window, hq, hkv, gate_src,
                                                              row_stride, out);
        }
        MLXD_CHECK(cudaGetLastError());
        return 0;
    }
    const size_t need = attention_prefill_scratch(S, pos0, window, hq, D);
    if (!scr || scr_floats < need) {
        set_error("prefill attention: scratch of %zu floats too small (%zu needed)", scr_floats, need);
        return -1;
    }
    int tmax = pos0 + S;
    if (window > 0 && tmax > window + S) tmax = window + S;
    dim3 grid(S, hq);
    attn_small_kernel<<<grid, 32, 0, st>>>(q, S, pos0, kc, vc, cap, window, hq, hkv, D, gate_src, row_stride, out,
                                           scr, tmax);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace mlxd
