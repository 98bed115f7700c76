// Attention: mlx_fast_scaled_dot_product_attention as fwd_attention calls it
// (src/engine/forward.c:713-731), with the q/k RMSNorm + RoPE of :591-697 and
// the KV append of kvcache.c:98-180 fused into the decode kernel.
//
// One arithmetic for decode and prefill (the oracle restates it): for a
// query q at position i over the keys it attends (causal, bottom-right
// aligned; with a window w, positions (i - w, i]),
//   q_d' = f32(scale * q_d), scale = 1/sqrtf(D);
//   z_j  = fmaf chain over d = 0..D-1 of q_d' * k_jd;
//   m    = max_j z_j;  p_j = own_expf(z_j - m)  (exactly 0 for masked keys);
//   per block of 64 absolute positions [64b, 64b + 64): l_b = in-order f32
//   sum of p_j, o_bd = fmaf chain of p_j v_jd in key order;
//   out_d = bf16(sum_b o_bd / sum_b l_b), the sums and the quotient in f64
//   (exact while a sum spans 53 bits), rounded once.
// Blocks are absolute positions, so a decode step and the prefill row at the
// same position give the same bits, whatever the split of the keys over
// CTAs. Head dims other than 64/128 take mlx's composed fallback (q scaled
// in bf16, bf16 scores, precise softmax rounded to bf16, bf16 output).
#include <cooperative_groups.h>
#include <mutex>
#include <stdlib.h>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

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
// One cluster of CL CTAs (8 warps) per kv head; the attended blocks
// (lo/64 .. pos/64) are split into CL contiguous ranges, one per CTA. A CTA
// streams its K blocks (padded to an even count), then its V blocks, through
// a 4-slot shared-memory ring (cp.async; the first four loads, the norm
// weights and this position's cos/sin are requested before waiting on the
// q|k|v projection, on which none of them depends). After the wait warp h
// normalises and rotates q head h in registers (lane l holds features
// l, l + 32, ...: the oracle's per-head RMSNorm association, and rotation
// pairs i, i + D/2 in one lane), and the CTA holding the new position also
// the new k, whose row (and v's) replaces the not yet appended cache row in
// its ring slot. Phase 1, two blocks at a time: scores (thread = (position,
// head)). Each CTA pushes its per-head maxima into every CTA's inbox through
// distributed shared memory; one cluster barrier. Phase 2, two blocks at a
// time: p, then per block the f32 chains (thread = (head, feature pair)),
// added into f64 partials, which are pushed into the inbox of the CTA owning
// that slice of the outputs; one cluster barrier; each CTA adds its slice
// locally. Remote accesses are stores only, all before a barrier.
constexpr int DA_THREADS = 256;
constexpr int DA_BS1 = DA_THREADS / AB;   // blocks per round in phase 1 (thread = position)

template <int D>
struct DaConst {
    static constexpr int NP = D / 2;                 // feature pairs
    static constexpr int BS2 = DA_THREADS / NP;      // blocks per round in phase 2
};

struct DaLayout {
    size_t ring, qs, stage, newkv, sc, P, red, gmax, inmax, inO, inL, total;
};
// nslots: K and V block slots (resident: 2 * scap/64; streaming: 2 * DA_BS1)
static __host__ __device__ inline DaLayout da_layout(int D, int REP, int scap, int CL, int nslots) {
    const int BS2 = DA_THREADS / (D / 2);
    DaLayout l;
    l.ring = 0;
    l.qs = l.ring + (size_t)nslots * AB * D * 2;
    l.stage = l.qs + (size_t)REP * D * 4;
    l.newkv = l.stage + (size_t)8 * D * 4;
    l.sc = l.newkv + (size_t)2 * D * 2;
    l.P = l.sc + (size_t)REP * scap * 4;
    l.red = l.P + (size_t)BS2 * AB * REP * 4;
    l.gmax = l.red + (size_t)8 * REP * 4;
    l.inmax = l.gmax + 64;
    l.inO = l.inmax + (((size_t)CL * REP * 4 + 15) / 16) * 16;
    l.inL = l.inO + (size_t)BS2 * REP * D * 8;
    l.total = l.inL + (size_t)CL * BS2 * REP * 8;
    return l;
}

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

// RES: every K and V block of the CTA resident in shared memory (all K rows
// requested as one commit group, all V rows as a second, before the wait);
// otherwise rounds of DA_BS1 K blocks (then V blocks) in a ring of
// 2 * DA_BS1 slots, the first round of each requested before the wait.
template <int D, int REP, int CL, bool RES>
__global__ void __launch_bounds__(DA_THREADS, 1) attn_decode_kernel(AttnDecodeArgs a, int scap) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    constexpr int NCH = D / 8;               // 16-byte chunks per row
    constexpr int NP = DaConst<D>::NP, BS2 = DaConst<D>::BS2;
    constexpr int DS = D / 32;
    constexpr int E = REP * D, ES = E / CL;   // outputs of the group, per owner CTA
    static_assert(ES % 2 == 0, "output slices hold whole feature pairs");
    const int rank = (int)cluster.block_rank();
    const int kh = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    extern __shared__ __align__(128) unsigned char sm[];
    const int NB = scap / AB;
    const int NSLOT = RES ? 2 * NB : 2 * DA_BS1;
    const DaLayout Ly = da_layout(D, REP, scap, CL, NSLOT);
    unsigned char *ring = sm + Ly.ring;
    float *qs = reinterpret_cast<float *>(sm + Ly.qs);          // [D][REP], scaled
    float *stage = reinterpret_cast<float *>(sm + Ly.stage) + (size_t)warp * D;
    uint16_t *newk = reinterpret_cast<uint16_t *>(sm + Ly.newkv), *newv = newk + D;
    float *sc = reinterpret_cast<float *>(sm + Ly.sc);          // [scap][REP]
    float *P = reinterpret_cast<float *>(sm + Ly.P);            // [BS2][AB][REP]
    float *red = reinterpret_cast<float *>(sm + Ly.red);        // [8 warps][REP]
    float *gmax = reinterpret_cast<float *>(sm + Ly.gmax);
    float *inmax = reinterpret_cast<float *>(sm + Ly.inmax);    // [CL][REP]
    double *inO = reinterpret_cast<double *>(sm + Ly.inO);      // [CL][BS2][ES]
    double *inL = reinterpret_cast<double *>(sm + Ly.inL);      // [CL][BS2][REP]

    const int pos = *a.d_pos;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int bfirst = lo / AB, blast = pos / AB, nbt = blast - bfirst + 1;
    const int mb0 = bfirst + (int)((long long)nbt * rank / CL), mb1 = bfirst + (int)((long long)nbt * (rank + 1) / CL);
    int nbm = mb1 - mb0;
    if (nbm > NB) {   // cannot happen for a launch sized by the host; report and do no work
        if (tid == 0) atomicExch(&g_attn_err, 1);
        nbm = 0;
    }
    const bool has_new = nbm > 0 && mb0 <= blast && blast < mb1;
    const uint16_t *kc = a.kc + (size_t)kh * a.cap * D;
    const uint16_t *vc = a.vc + (size_t)kh * a.cap * D;

    // block i (< nbm) of K (isv 0) or V into slot `slot`; rows outside
    // [lo, pos) zero-filled (the new position's row comes from this step)
    auto load_block = [&](int i, bool isv, int slot) {
        if (i >= nbm) return;
        const int b = mb0 + i;
        unsigned char *dst = ring + (size_t)slot * AB * D * 2;
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
    auto kslot = [&](int i) { return RES ? i : i % DA_BS1; };
    auto vslot = [&](int i) { return RES ? NB + i : DA_BS1 + i % DA_BS1; };
    if (RES) {
        for (int i = 0; i < nbm; i++) load_block(i, false, kslot(i));
        cp_async_commit();
        for (int i = 0; i < nbm; i++) load_block(i, true, vslot(i));
        cp_async_commit();
    } else {
        for (int i = 0; i < DA_BS1; i++) load_block(i, false, kslot(i));
        cp_async_commit();
        for (int i = 0; i < DA_BS1; i++) load_block(i, true, vslot(i));
        cp_async_commit();
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
    // per-warp head work: q heads h = warp, warp + 8; the new k after them
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

    const int qstride = D * (a.gate ? 2 : 1);
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

    // phase 1: thread (position pp, block slot s1) scores all REP heads of
    // blocks s1, s1 + DA_BS1, ... (one fmaf chain over d per head)
    const int pp = tid % AB, s1 = tid / AB;
    float lmax[REP];
#pragma unroll
    for (int h = 0; h < REP; h++) lmax[h] = -INFINITY;
    for (int r0 = 0; r0 < nbm; r0 += DA_BS1) {
        if (r0 == 0) cp_async_wait<1>();   // the first K round (V may still be in flight)
        else if (!RES) cp_async_wait<0>();  // the K round requested after the previous one
        __syncthreads();   // (first round: also orders the q and new-k stores)
        if (has_new && blast - mb0 >= r0 && blast - mb0 < r0 + DA_BS1) {
            unsigned char *blk = ring + (size_t)kslot(blast - mb0) * AB * D * 2;
            const int r = pos - blast * AB;
            for (int c = tid; c < NCH; c += DA_THREADS)
                *reinterpret_cast<uint4 *>(blk + blk_off<D>(r, c)) = *reinterpret_cast<const uint4 *>(newk + c * 8);
            __syncthreads();
        }
        const int i = r0 + s1;
        if (i < nbm) {
            const unsigned char *blk = ring + (size_t)kslot(i) * AB * D * 2;
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
            for (int h = 0; h < REP; h++) {
                const float z = valid ? acc[h] : -INFINITY;
                sc[(i * AB + pp) * REP + h] = z;
                lmax[h] = fmaxf(lmax[h], z);
            }
        }
        if (!RES && r0 + DA_BS1 < nbm) {
            __syncthreads();
            for (int s = 0; s < DA_BS1; s++) load_block(r0 + DA_BS1 + s, false, kslot(r0 + DA_BS1 + s));
            cp_async_commit();
        }
    }
    // per-head maxima of the CTA, pushed into every CTA's inbox
#pragma unroll
    for (int h = 0; h < REP; h++) {
        const float v = warp_max(lmax[h]);
        if (lane == 0) red[warp * REP + h] = v;
    }
    __syncthreads();
    if (tid < CL * REP) {
        const int dst = tid / REP, h = tid % REP;
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; w++) m = fmaxf(m, red[w * REP + h]);
        *cluster.map_shared_rank(inmax + rank * REP + h, dst) = m;
    }
    cluster.sync();
    if (tid < REP) {
        float m = -INFINITY;
#pragma unroll
        for (int r = 0; r < CL; r++) m = fmaxf(m, inmax[r * REP + tid]);
        gmax[tid] = m;
    }

    // phase 2: per round of BS2 blocks, p of the round's blocks (thread =
    // position), then thread (feature pair dp, block slot s2) runs the
    // 2 * REP chains of block s2 (v pair unpacked once for all heads) and
    // l for all heads (dp == 0), added into f64 partials of its slot
    const int dp = tid % NP, s2 = tid / NP;
    double Oa[REP][2], La[REP];
#pragma unroll
    for (int h = 0; h < REP; h++) Oa[h][0] = Oa[h][1] = La[h] = 0.0;
    if (RES) cp_async_wait<0>();
    for (int r0 = 0; r0 < nbm; r0 += BS2) {
        if (!RES) cp_async_wait<0>();
        __syncthreads();   // (first round: also orders gmax and the V rows)
        if (has_new && blast - mb0 >= r0 && blast - mb0 < r0 + BS2) {
            unsigned char *blk = ring + (size_t)vslot(blast - mb0) * AB * D * 2;
            const int r = pos - blast * AB;
            for (int c = tid; c < NCH; c += DA_THREADS)
                *reinterpret_cast<uint4 *>(blk + blk_off<D>(r, c)) = *reinterpret_cast<const uint4 *>(newv + c * 8);
        }
        for (int e = tid; e < BS2 * AB; e += DA_THREADS) {
            const int s = e / AB, q = e % AB, i = r0 + s;
#pragma unroll
            for (int h = 0; h < REP; h++) {
                const float z = i < nbm ? sc[(i * AB + q) * REP + h] : -INFINITY;
                P[(s * AB + q) * REP + h] = z == -INFINITY ? 0.f : own_expf(__fsub_rn(z, gmax[h]));
            }
        }
        __syncthreads();
        const int i = r0 + s2;
        if (i < nbm) {
            const unsigned char *blk = ring + (size_t)vslot(i) * AB * D * 2;
            const float *ps = P + (size_t)s2 * AB * REP;
            const int c = dp >> 2, off = (dp & 3) * 4;
            // l of head lh (threads dp < REP; the others' chain is unused)
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
#pragma unroll
            for (int h = 0; h < REP; h++) {
                Oa[h][0] += (double)o0[h];
                Oa[h][1] += (double)o1[h];
            }
            if (dp < REP) La[dp] += (double)l;
        }
        if (!RES && r0 + BS2 < nbm) {
            __syncthreads();
            for (int s = 0; s < BS2; s++) load_block(r0 + BS2 + s, true, vslot(r0 + BS2 + s));
            cp_async_commit();
        }
    }
    cp_async_wait<0>();
    // the slot partials into the inbox of the CTA owning each output slice
#pragma unroll
    for (int h = 0; h < REP; h++) {
        const int e = h * D + 2 * dp, dst = e / ES;
        *reinterpret_cast<double2 *>(cluster.map_shared_rank(inO + ((size_t)rank * BS2 + s2) * ES + (e - dst * ES), dst)) =
            make_double2(Oa[h][0], Oa[h][1]);
    }
    if (dp < REP)
        for (int r = 0; r < CL; r++) *cluster.map_shared_rank(inL + ((size_t)rank * BS2 + s2) * REP + dp, r) = La[dp];
    cluster.sync();
    for (int el = tid; el < ES; el += DA_THREADS) {
        const int e = rank * ES + el, h = e / D, d = e % D;
        double os = 0.0, ls = 0.0;
        for (int r = 0; r < CL * BS2; r++) {
            os += inO[(size_t)r * ES + el];
            ls += inL[(size_t)r * REP + h];
        }
        const int hg = kh * REP + h;
        uint16_t val = d2bf(os / ls);
        if (a.gate) {
            const float gv = bf2f(a.qkv[(size_t)hg * qstride + D + d]);
            val = f2bf(__fmul_rn(bf2f(val), sigmoid_bf16(gv)));
        }
        a.out[(size_t)hg * D + d] = val;
    }
    // the new position's k/v rows into the cache
    if (has_new) {
        uint16_t *kd = a.kc + ((size_t)kh * a.cap + pos % a.cap) * D;
        uint16_t *vd = a.vc + ((size_t)kh * a.cap + pos % a.cap) * D;
        for (int d = tid; d < D; d += DA_THREADS) {
            kd[d] = newk[d];
            vd[d] = newv[d];
        }
    }
}

// blocks one CTA may hold for a cache of `cap` slots (window: at most
// `window` attended positions)
static int da_scap(const AttnDecodeArgs &a, int CL) {
    const int span = a.window > 0 && a.window < a.cap ? a.window : a.cap;
    const int nbt = span / AB + 2;
    return ((nbt + CL - 1) / CL) * AB;
}

// One CTA per SM (dynamic shared memory above half of an SM's): with two
// attention CTAs on one SM the projections that follow ran slower on those
// SMs for the rest of the step.
template <int D, int REP>
static size_t da_smem(int scap, int CL, bool res) {
    const size_t t = da_layout(D, REP, scap, CL, res ? 2 * (scap / AB) : 2 * DA_BS1).total;
    return t > 116 * 1024 ? t : 116 * 1024;
}
// every block resident when it fits in a CTA's shared memory
template <int D, int REP>
static bool da_resident(int scap, int CL) {
    return da_layout(D, REP, scap, CL, 2 * (scap / AB)).total <= 220 * 1024;
}

template <int D, int REP, int CL, bool RES>
static bool da_prepare(const AttnDecodeArgs &a, size_t smem) {
    auto kern = attn_decode_kernel<D, REP, CL, RES>;
    if (!smem_allowed((const void *)kern, smem)) return false;
    if (CL > 8) {
        static std::mutex mu;
        static bool np[64] = {};   // per instantiation and device
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lock(mu);
        if (dev >= 0 && dev < 64 && !np[dev]) {
            if (!cuda_ok(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                         "cluster attribute"))
                return false;
            np[dev] = true;
        }
    }
    return true;
}

template <int D, int REP, int CL>
static cudaLaunchConfig_t da_config(const AttnDecodeArgs &a, size_t smem, cudaLaunchAttribute *attr, bool pdl,
                                    cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL, a.hkv);
    cfg.blockDim = dim3(DA_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cfg;
}

// whether `hkv` clusters of CL CTAs are resident at once on this device
template <int D, int REP, int CL>
static bool da_fits(const AttnDecodeArgs &a) {
    const int scap = da_scap(a, CL);
    const bool res = da_resident<D, REP>(scap, CL);
    const size_t smem = da_smem<D, REP>(scap, CL, res);
    if (smem > 227 * 1024 || !(res ? da_prepare<D, REP, CL, true>(a, smem) : da_prepare<D, REP, CL, false>(a, smem))) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = da_config<D, REP, CL>(a, smem, attr, false, nullptr);
    int n = 0;
    cudaError_t e = res ? cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<D, REP, CL, true>, &cfg)
                        : cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<D, REP, CL, false>, &cfg);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n >= a.hkv;
}

// cluster size per (device, kv heads, cache span): 16 when hkv clusters of
// 16 are resident at once, else 8
template <int D, int REP>
static int da_cluster(const AttnDecodeArgs &a) {
    static std::mutex mu;
    static std::vector<std::pair<std::pair<int, long long>, int>> memo;
    int dev = 0;
    cudaGetDevice(&dev);
    const long long key = ((long long)a.hkv << 32) | (unsigned)da_scap(a, 8);
    std::lock_guard<std::mutex> lock(mu);
    for (auto &m : memo)
        if (m.first.first == dev && m.first.second == key) return m.second;
    const int cl = da_fits<D, REP, 16>(a) ? 16 : 8;
    memo.push_back({{dev, key}, cl});
    return cl;
}

template <int D, int REP, int CL>
static int da_launch(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    const int scap = da_scap(a, CL);
    const bool res = da_resident<D, REP>(scap, CL);
    const size_t smem = da_smem<D, REP>(scap, CL, res);
    if (smem > 227 * 1024) {
        set_error("decode attention: a cache of %d slots needs %zu bytes of shared memory per CTA", a.cap, smem);
        return -1;
    }
    if (!(res ? da_prepare<D, REP, CL, true>(a, smem) : da_prepare<D, REP, CL, false>(a, smem))) return -1;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = da_config<D, REP, CL>(a, smem, attr, pdl, st);
    if (res) MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, REP, CL, true>, a, scap));
    else MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_decode_kernel<D, REP, CL, false>, a, scap));
    return 0;
}

template <int D, int REP>
static int da_dispatch(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    return da_cluster<D, REP>(a) == 16 ? da_launch<D, REP, 16>(a, st, pdl) : da_launch<D, REP, 8>(a, st, pdl);
}

template <int D, int REP>
static int da_sms(const AttnDecodeArgs &a) {
    return da_cluster<D, REP>(a) * a.hkv;
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
    MLXD_DA_DISPATCH(da_dispatch, a, st, pdl)
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
// CTA = (64 queries, one q head), 256 threads. Keys are walked in blocks of
// 64 absolute positions over the union of the tile's key ranges.
//   pass 1: the 64 x 64 score tile of a block on CUDA cores, thread (tq, tk)
//           holding queries 4tq.. and keys 4tk.. (16 fmaf chains stepping
//           through d together; q' and k transposed to f32 in shared memory
//           so that each step is two 16-byte loads); scores go to the CTA's
//           own region of a global scratch (read back from L2) and the
//           per-query maxima are kept;
//   pass 2: per block, p = own_expf(z - m) into shared memory, then thread
//           (tq, td) runs the chains of queries 4tq.. x features 8td.. over
//           the block's keys and adds them into f64 registers; l_b by the
//           threads with td = 0.
constexpr int PF_T = 256, PF_Q = 64;

template <int D>
struct PfLayout {
    static constexpr size_t qT = 0;                               // [D][64] f32
    static constexpr size_t kT = qT + (size_t)D * PF_Q * 4;        // [D][64] f32
    static constexpr size_t pT = kT + (size_t)D * AB * 4;          // [64 keys][64 q] f32
    static constexpr size_t vb = pT + (size_t)AB * PF_Q * 4;       // [64][D] bf16
    static constexpr size_t mx = vb + (size_t)AB * D * 2;          // [64] f32 + red
    static constexpr size_t total = mx + (size_t)PF_Q * 4 * 16;
};

template <int D>
__global__ void __launch_bounds__(PF_T) attn_prefill_kernel(const uint16_t *__restrict__ q, int S, int pos0,
                                                           const uint16_t *__restrict__ kc,
                                                           const uint16_t *__restrict__ vc, int cap, int window,
                                                           int hq, int hkv, const uint16_t *__restrict__ gate_src,
                                                           int row_stride, uint16_t *__restrict__ out,
                                                           float *__restrict__ scr, int span_max) {
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
    float *myscr = scr + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * PF_Q * (size_t)span_max;
    const uint16_t *K = kc + (size_t)kh * cap * D;
    const uint16_t *V = vc + (size_t)kh * cap * D;

    // q' transposed: qT[d][i] = f32(scale * q[i][d]) (0 for rows past S)
    for (int e = tid; e < PF_Q * D; e += PF_T) {
        const int d = e / PF_Q, i = e % PF_Q;
        qT[d * PF_Q + i] = i < nq ? __fmul_rn(scale, bf2f(q[((size_t)(qt0 + i) * hq + h) * D + d])) : 0.f;
    }
    const int tq = tid >> 4, tk = tid & 15;   // pass 1: queries 4tq.., keys 4tk..
    float rmax[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    int qp[4], j0r[4];
#pragma unroll
    for (int a = 0; a < 4; a++) {
        qp[a] = pos0 + qt0 + 4 * tq + a;
        j0r[a] = window > 0 ? max(0, qp[a] - window + 1) : 0;
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
    uint4 kpre[NPF];
    fetch_rows(K, b0, kpre);
    for (int bi = 0; bi < nb; bi++) {
        const int b = b0 + bi;
        __syncthreads();
        // k block transposed to f32: kT[d][r]
#pragma unroll
        for (int x = 0; x < NPF; x++) {
            const int e = tid + PF_T * x, c = e / AB, r = e % AB;
            const uint32_t w[4] = {kpre[x].x, kpre[x].y, kpre[x].z, kpre[x].w};
#pragma unroll
            for (int y = 0; y < 4; y++) {
                kT[(c * 8 + 2 * y) * AB + r] = lo_bf(w[y]);
                kT[(c * 8 + 2 * y + 1) * AB + r] = hi_bf(w[y]);
            }
        }
        if (bi + 1 < nb) fetch_rows(K, b + 1, kpre);
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
#pragma unroll
        for (int y = 0; y < 4; y++) {
            const int j = b * AB + 4 * tk + y;
            float4 o;
            float *ov = &o.x;
#pragma unroll
            for (int x = 0; x < 4; x++) {
                const bool ok = 4 * tq + x < nq && j >= j0r[x] && j <= qp[x];
                ov[x] = ok ? acc[x][y] : -INFINITY;
                rmax[x] = fmaxf(rmax[x], ov[x]);
            }
            *reinterpret_cast<float4 *>(myscr + (size_t)(bi * AB + 4 * tk + y) * PF_Q + 4 * tq) = o;
        }
    }
    // per-query maxima: the 16 threads of a tq (consecutive lanes) reduce
#pragma unroll
    for (int x = 0; x < 4; x++) {
        float v = rmax[x];
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (tk == 0) smx[4 * tq + x] = v;
    }
    __syncthreads();   // also orders the score stores before pass 2 reads them

    // pass 2: thread (tq, td): queries 4tq.., features 8td.. (D = 128: td < 16)
    constexpr int FT = D / 8;           // feature groups
    constexpr int QT = PF_T / FT;       // query groups (16 for D=128, 32 for D=64)
    constexpr int QPT = PF_Q / QT;      // queries per thread (4 or 2)
    const int td = tid % FT, tq2 = tid / FT;
    double O[QPT][8], Lq[QPT];
#pragma unroll
    for (int x = 0; x < QPT; x++) {
        Lq[x] = 0.0;
#pragma unroll
        for (int y = 0; y < 8; y++) O[x][y] = 0.0;
    }
    // scores of a block (16 per thread: 4 float4 of key r, queries 4i4..)
    // and its value rows, requested one block ahead into registers
    float4 zpre[4];
    uint4 vpre[NPF];
    auto fetch_scores = [&](int bi) {
#pragma unroll
        for (int x = 0; x < 4; x++) {
            const int e = tid + PF_T * x, r = e / (PF_Q / 4), i4 = e % (PF_Q / 4);
            zpre[x] = __ldcg(reinterpret_cast<const float4 *>(myscr + (size_t)(bi * AB + r) * PF_Q) + i4);
        }
    };
    fetch_scores(0);
    fetch_rows(V, b0, vpre);
    for (int bi = 0; bi < nb; bi++) {
        __syncthreads();
        // p tile (transposed: pT[key][query]) and the v block
#pragma unroll
        for (int x = 0; x < 4; x++) {
            const int e = tid + PF_T * x, r = e / (PF_Q / 4), i4 = e % (PF_Q / 4);
            const float z[4] = {zpre[x].x, zpre[x].y, zpre[x].z, zpre[x].w};
            float4 pv;
            float *pp = &pv.x;
#pragma unroll
            for (int k = 0; k < 4; k++) pp[k] = z[k] == -INFINITY ? 0.f : own_expf(__fsub_rn(z[k], smx[4 * i4 + k]));
            *reinterpret_cast<float4 *>(pT + r * PF_Q + 4 * i4) = pv;
        }
#pragma unroll
        for (int x = 0; x < NPF; x++) {
            const int e = tid + PF_T * x, c = e / AB, r = e % AB;
            *reinterpret_cast<uint4 *>(vb + r * D + c * 8) = vpre[x];
        }
        if (bi + 1 < nb) {
            fetch_scores(bi + 1);
            fetch_rows(V, b0 + bi + 1, vpre);
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
#pragma unroll
        for (int x = 0; x < QPT; x++) {
            Lq[x] += (double)l[x];
#pragma unroll
            for (int y = 0; y < 8; y++) O[x][y] += (double)o[x][y];
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

// scratch floats a prefill launch needs
size_t attention_prefill_scratch(int S, int pos0, int window, int hq, int D) {
    if (D == 64 || D == 128) {
        const int ntile = (S + PF_Q - 1) / PF_Q;
        int span = (pos0 + S) + AB;   // keys of a tile, rounded out to blocks
        if (window > 0 && span > window + PF_Q + 2 * AB) span = window + PF_Q + 2 * AB;
        span = ((span + AB - 1) / AB) * AB;
        return (size_t)ntile * hq * PF_Q * span;
    }
    int tmax = pos0 + S;
    if (window > 0 && tmax > window + S) tmax = window + S;
    return (size_t)S * hq * tmax;
}

int attention_prefill(const uint16_t *q, int S, int pos0, const uint16_t *kc, const uint16_t *vc, int cap,
                      int window, int hq, int hkv, int D, const uint16_t *gate_src, int qdim, uint16_t *out,
                      float *scr, size_t scr_floats, cudaStream_t st) {
    const int row_stride = qdim + 2 * hkv * D;
    const size_t need = attention_prefill_scratch(S, pos0, window, hq, D);
    if (!scr || scr_floats < need) {
        set_error("prefill attention: scratch of %zu floats too small (%zu needed)", scr_floats, need);
        return -1;
    }
    if (D == 64 || D == 128) {
        const int ntile = (S + PF_Q - 1) / PF_Q;
        const int span_max = (int)(need / ((size_t)ntile * hq * PF_Q));
        dim3 grid(ntile, hq);
        if (D == 128) {
            const size_t smem = PfLayout<128>::total;
            if (!smem_allowed((const void *)attn_prefill_kernel<128>, smem)) return -1;
            attn_prefill_kernel<128><<<grid, PF_T, smem, st>>>(q, S, pos0, kc, vc, cap, window, hq, hkv, gate_src,
                                                               row_stride, out, scr, span_max);
        } else {
            const size_t smem = PfLayout<64>::total;
            if (!smem_allowed((const void *)attn_prefill_kernel<64>, smem)) return -1;
            attn_prefill_kernel<64><<<grid, PF_T, smem, st>>>(q, S, pos0, kc, vc, cap, window, hq, hkv, gate_src,
                                                              row_stride, out, scr, span_max);
        }
        MLXD_CHECK(cudaGetLastError());
        return 0;
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
