// Decode attention for one new token on the tensor pipe, one thread-block
// cluster per kv head (mlx_fast_scaled_dot_product_attention for one query,
// src/engine/forward.c:713-731, with the q/k RMSNorm + RoPE of :591-697 and
// the KV append of kvcache.c:98-180).
//
// Cluster (CL CTAs of 8 warps) per kv head; CTA r of the cluster takes the
// r-th of CL equal slices of the attended positions (lo, pos], each warp an
// equal part of that slice, in chunks of 16 positions. Before waiting on the
// q|k|v projection a warp requests its first two chunks of cached K and V
// rows into a private shared-memory ring (cp.async, rows XOR-swizzled in
// 16-byte pieces so that ldmatrix reads are conflict-free); the cached rows
// do not depend on this step. After the wait every warp normalises and
// rotates the group's q heads and the new k in registers (lane L holds
// features L, L+32, ...: the per-head RMSNorm association of the oracle, and
// RoPE pairs i, i + rope_dims/2 in the same lane), then per chunk
//   S^T = q K^T   mma.m16n8k16 bf16: A = q (rows: the group's heads), B = K
//                 rows through ldmatrix, f32 accumulate;
//   online softmax in the log2 domain, f32, per head;
//   O += P V      mma.m16n8k16: A = P as bf16 hi + lo (P = hi + lo to 2^-17,
//                 so P.V keeps f32 precision), B = V rows through ldmatrix.trans.
// A row r < REP of both MMAs is head r; rows REP..2REP-1 repeat the heads, so
// that P's hi part (rows < REP) and lo part (the repeats) share one P.V MMA
// and are added once after the loop (REP 8: the lo rows are 8..15, in the
// same lanes as their hi rows).
// The chunk holding the new position gets the new k/v rows written over its
// (not yet appended) cache rows. Warps merge in shared memory, the cluster
// synchronises, and CTA r merges the r-th slice of the group's outputs from
// all CL CTAs' partials through distributed shared memory: no global
// partials, no atomics, no last-arriver. CTA 0 of the cluster appends the new
// k/v row to the cache.
#include <cooperative_groups.h>
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(attention_tc)

constexpr int TC_WARPS = 8, TC_THREADS = 256, TC_ROWS = 16, TC_NBUF = 2;

template <int D, int REP>
struct TcSmem {
    static constexpr size_t CB = (size_t)TC_ROWS * D * 2;              // K (or V) rows of a chunk
    static constexpr size_t ring = (size_t)TC_WARPS * TC_NBUF * 2 * CB;
    static constexpr size_t q = ring;                                   // [warps][REP][D] bf16
    static constexpr size_t wo = q + (size_t)TC_WARPS * REP * D * 2;     // [warps][REP][D] f32
    static constexpr size_t wml = wo + (size_t)TC_WARPS * REP * D * 4;   // [warps][REP][2]
    static constexpr size_t cml = wml + (size_t)TC_WARPS * REP * 2 * 4;  // [REP][2] CTA partial
    static constexpr size_t co = cml + (size_t)REP * 2 * 4;             // [REP][D] CTA partial
    // inbox of the cluster merge: per source CTA (at most 16), (m, l) of the
    // slice's head and the slice's REP*D/CL partial outputs
    static constexpr size_t inbox = co + (size_t)REP * D * 4;
    static constexpr size_t total = inbox + (size_t)16 * (2 + REP * D / 8) * 4;
};

// byte offset of 16-byte piece c of row r in a chunk's K or V rows
template <int D>
MLXD_DEV int tc_sw(int r, int c) {
    return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

template <int D, int REP, int CL>
__global__ void __launch_bounds__(TC_THREADS, 1) attn_tc_kernel(AttnDecodeArgs a) {
    MLXD_TRACE_START
    namespace cg = cooperative_groups;
    using L = TcSmem<D, REP>;
    constexpr int DS = D / 32;     // features per lane (strided)
    constexpr int NKK = D / 16;    // k-steps of q K^T
    constexpr int NTO = D / 8;     // n-tiles of P V
    constexpr int PR = D / 8;      // 16-byte pieces per row
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int kh = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3, gq = lane >> 2;
    // first cluster barrier phase: every CTA of the cluster has started before
    // any of them writes into another's shared memory (waited before the push)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    extern __shared__ __align__(128) unsigned char sm[];
    unsigned char *ring = sm + (size_t)warp * TC_NBUF * 2 * L::CB;
    uint16_t *sq = reinterpret_cast<uint16_t *>(sm + L::q) + (size_t)warp * REP * D;
    float *wo = reinterpret_cast<float *>(sm + L::wo);
    float *wml = reinterpret_cast<float *>(sm + L::wml);
    float *cml = reinterpret_cast<float *>(sm + L::cml);
    float *co = reinterpret_cast<float *>(sm + L::co);

    const int pos = *a.d_pos;
    const int T = pos + 1;
    const int lo = a.window > 0 ? max(0, T - a.window) : 0;
    const int span = T - lo;
    const int r0 = lo + (int)((long long)span * rank / CL), r1 = lo + (int)((long long)span * (rank + 1) / CL);
    const int per = (r1 - r0 + TC_WARPS - 1) / TC_WARPS;
    const int w0 = r0 + warp * per, w1 = min(r1, w0 + per);
    const int nchunks = w1 > w0 ? (w1 - w0 + TC_ROWS - 1) / TC_ROWS : 0;
    uint16_t *kc = a.kc + (size_t)kh * a.cap * D;
    uint16_t *vc = a.vc + (size_t)kh * a.cap * D;

    // chunk c of this warp's rows into ring slot c % TC_NBUF (rows past the
    // warp's range are zero-filled); one commit group per call
    auto issue = [&](int c) {
        if (c < nchunks) {
            unsigned char *kb = ring + (size_t)(c % TC_NBUF) * 2 * L::CB, *vb = kb + L::CB;
            const int j0 = w0 + c * TC_ROWS;
            for (int i = lane; i < TC_ROWS * PR; i += 32) {
                const int r = i / PR, p = i % PR;
                const bool valid = j0 + r < w1;
                const int j = valid ? j0 + r : w0;
                const size_t off = (size_t)(j % a.cap) * D + p * 8;
                cp_async16_zfill(kb + tc_sw<D>(r, p), kc + off, valid);
                cp_async16_zfill(vb + tc_sw<D>(r, p), vc + off, valid);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int c = 0; c < TC_NBUF; c++) issue(c);
    // the norm weights and this position's rotation (rotate-half over all D
    // features: pairs i, i + D/2 sit in one lane), fixed for the step
    constexpr int HL = DS / 2;
    const int half = D / 2;
    float qnw[DS], knw[DS], rc[DS], rs[DS];
#pragma unroll
    for (int i = 0; i < DS; i++) {
        const int d = lane + 32 * i;
        qnw[i] = a.qn ? bf2f(a.qn[d]) : 1.f;
        knw[i] = a.kn ? bf2f(a.kn[d]) : 1.f;
        const float *cs = a.rope.cs + (size_t)pos * half * 2;
        rc[i] = d < half ? cs[2 * d] : 1.f;
        rs[i] = d < half ? cs[2 * d + 1] : 0.f;
    }
    pdl_trigger();
    pdl_wait();
    MLXD_TRACE_WAITED

    // head_norm_rope in registers for the group's q heads and the new k
    // (vector REP), their reductions interleaved: the oracle's association
    // (lane-strided fmaf partials, butterfly o = 16..1), its rounding points
    const bool norm = a.qn != nullptr;
    const uint16_t *qkv = a.qkv;
    const int qstride = D * (a.gate ? 2 : 1);
    // every load of the new q/k/v rows in flight before any arithmetic
    uint16_t raw[REP + 1][DS], vn[DS];
#pragma unroll
    for (int i = 0; i < DS; i++) {
        raw[REP][i] = qkv[a.qdim + (size_t)kh * D + lane + 32 * i];
        vn[i] = qkv[a.qdim + (size_t)(a.hkv + kh) * D + lane + 32 * i];
#pragma unroll
        for (int h = 0; h < REP; h++) raw[h][i] = qkv[(size_t)(kh * REP + h) * qstride + lane + 32 * i];
    }
    float vv[REP + 1][DS];
#pragma unroll
    for (int h = 0; h <= REP; h++)
#pragma unroll
        for (int i = 0; i < DS; i++) vv[h][i] = bf2f(raw[h][i]);
    if (norm) {
        float acc[REP + 1];
#pragma unroll
        for (int h = 0; h <= REP; h++) {
            acc[h] = 0.f;
#pragma unroll
            for (int i = 0; i < DS; i++) acc[h] = fmaf(vv[h][i], vv[h][i], acc[h]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int h = 0; h <= REP; h++) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
#pragma unroll
        for (int h = 0; h <= REP; h++) {
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc[h], (float)D), a.eps)));
#pragma unroll
            for (int i = 0; i < DS; i++)
                vv[h][i] = rbf(__fmul_rn(h < REP ? qnw[i] : knw[i], rbf(__fmul_rn(vv[h][i], inv))));
        }
    }
#pragma unroll
    for (int h = 0; h <= REP; h++)
#pragma unroll
        for (int i = 0; i < HL; i++) {
            const float x1 = vv[h][i], x2 = vv[h][i + HL];
            vv[h][i] = rbf(__fsub_rn(__fmul_rn(x1, rc[i]), __fmul_rn(x2, rs[i])));
            vv[h][i + HL] = rbf(__fadd_rn(__fmul_rn(x1, rs[i]), __fmul_rn(x2, rc[i])));
        }
#pragma unroll
    for (int h = 0; h < REP; h++)
#pragma unroll
        for (int i = 0; i < DS; i++) sq[h * D + lane + 32 * i] = f2bf(vv[h][i]);
    float kn[DS];
#pragma unroll
    for (int i = 0; i < DS; i++) kn[i] = vv[REP][i];
    if (rank == 0 && warp == 0) {
        const size_t slot = (size_t)(pos % a.cap) * D;
#pragma unroll
        for (int i = 0; i < DS; i++) {
            kc[slot + lane + 32 * i] = f2bf(kn[i]);
            vc[slot + lane + 32 * i] = vn[i];
        }
    }
    __syncwarp();
    // A fragments of q: row gq holds head gq % REP for gq < 2 REP (REP 8:
    // head gq, rows gq + 8 unused in q K^T), other rows are zero
    constexpr bool LO8 = REP == 8;            // lo rows are gq + 8, same lane
    const bool rowv = LO8 || gq < 2 * REP;
    const int hrow = LO8 ? gq : gq % REP;
    uint32_t qa[NKK][2];
#pragma unroll
    for (int kk = 0; kk < NKK; kk++) {
        qa[kk][0] = rowv ? *reinterpret_cast<const uint32_t *>(sq + hrow * D + 16 * kk + 2 * t) : 0u;
        qa[kk][1] = rowv ? *reinterpret_cast<const uint32_t *>(sq + hrow * D + 16 * kk + 8 + 2 * t) : 0u;
    }

    MLXD_TRACE_T(tr_prep_)
    const float qscale = rsqrtf((float)D) * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    float o[NTO][4];
#pragma unroll
    for (int n = 0; n < NTO; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    for (int c = 0; c < nchunks; c++) {
        cp_async_wait<TC_NBUF - 1>();
        __syncwarp();
        unsigned char *kb = ring + (size_t)(c % TC_NBUF) * 2 * L::CB, *vb = kb + L::CB;
        const int j0 = w0 + c * TC_ROWS;
        if (pos >= j0 && pos < j0 + TC_ROWS && pos < w1) {
            // the new position: this step's k/v, not the cache row
            const int r = pos - j0;
#pragma unroll
            for (int i = 0; i < DS; i++) {
                const int d = lane + 32 * i;
                *reinterpret_cast<uint16_t *>(kb + tc_sw<D>(r, d >> 3) + (d & 7) * 2) = f2bf(kn[i]);
                *reinterpret_cast<uint16_t *>(vb + tc_sw<D>(r, d >> 3) + (d & 7) * 2) = vn[i];
            }
            __syncwarp();
        }
        // S^T = q K^T for positions j0 + 8 nt + (0..7)
        float s[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
            for (int k2 = 0; k2 < NKK / 2; k2++) {
                uint32_t b[4];
                ldmatrix_x4(b, kb + tc_sw<D>(nt * 8 + (lane & 7), 4 * k2 + (lane >> 3)));
                const uint32_t a0[4] = {qa[2 * k2][0], 0u, qa[2 * k2][1], 0u};
                const uint32_t a1[4] = {qa[2 * k2 + 1][0], 0u, qa[2 * k2 + 1][1], 0u};
                mma_bf16_16816(s[nt], a0, b[0], b[1]);
                mma_bf16_16816(s[nt], a1, b[2], b[3]);
            }
        }
        // online softmax of head gq over the chunk (log2 domain)
        float sc[2][2], mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int j = j0 + nt * 8 + 2 * t + e;
                sc[nt][e] = j < w1 ? s[nt][e] * qscale : -INFINITY;
                mx = fmaxf(mx, sc[nt][e]);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);
        const float al = m == -INFINITY ? 0.f : exp2f(m - mn);
        float p[2][2], ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                p[nt][e] = sc[nt][e] == -INFINITY ? 0.f : exp2f(sc[nt][e] - mn);
                ps += p[nt][e];
            }
        l = fmaf(l, al, ps);
        m = mn;
#pragma unroll
        for (int n = 0; n < NTO; n++) {
            o[n][0] *= al;
            o[n][1] *= al;
            if (LO8) {
                o[n][2] *= al;
                o[n][3] *= al;
            }
        }
        // P as bf16 hi + lo: hi in rows < REP, lo in the repeated rows
        const uint32_t h0 = pack_bf2(p[0][0], p[0][1]), h1 = pack_bf2(p[1][0], p[1][1]);
        const uint32_t l0 = pack_bf2(p[0][0] - lo_bf(h0), p[0][1] - hi_bf(h0));
        const uint32_t l1 = pack_bf2(p[1][0] - lo_bf(h1), p[1][1] - hi_bf(h1));
        uint32_t ap[4];
        if (LO8) {
            ap[0] = h0, ap[1] = l0, ap[2] = h1, ap[3] = l1;
        } else {
            ap[0] = gq < REP ? h0 : gq < 2 * REP ? l0 : 0u;
            ap[2] = gq < REP ? h1 : gq < 2 * REP ? l1 : 0u;
            ap[1] = ap[3] = 0u;
        }
#pragma unroll
        for (int n2 = 0; n2 < NTO / 2; n2++) {
            uint32_t b[4];
            ldmatrix_x4_trans(b, vb + tc_sw<D>(((lane >> 3) & 1) * 8 + (lane & 7), 2 * n2 + (lane >> 4)));
            mma_bf16_16816(o[2 * n2], ap, b[0], b[1]);
            mma_bf16_16816(o[2 * n2 + 1], ap, b[2], b[3]);
        }
        __syncwarp();
        issue(c + TC_NBUF);
    }
    cp_async_wait<0>();
    MLXD_TRACE_T(tr_loop_)
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    // O of head gq: its hi rows plus its lo rows
#pragma unroll
    for (int n = 0; n < NTO; n++) {
        if (LO8) {
            o[n][0] += o[n][2];
            o[n][1] += o[n][3];
        } else {
            o[n][0] += __shfl_down_sync(0xffffffffu, o[n][0], 4 * REP);
            o[n][1] += __shfl_down_sync(0xffffffffu, o[n][1], 4 * REP);
        }
    }
    // the warps' partials, then the CTA's
    if (gq < REP) {
        if (t == 0) {
            wml[(warp * REP + gq) * 2] = m;
            wml[(warp * REP + gq) * 2 + 1] = l;
        }
#pragma unroll
        for (int n = 0; n < NTO; n++)
            *reinterpret_cast<float2 *>(wo + ((size_t)warp * REP + gq) * D + n * 8 + 2 * t) =
                make_float2(o[n][0], o[n][1]);
    }
    __syncthreads();
    for (int idx = tid; idx < REP * D; idx += TC_THREADS) {
        const int h = idx / D, d = idx % D;
        float mm = -INFINITY;
#pragma unroll
        for (int w = 0; w < TC_WARPS; w++) mm = fmaxf(mm, wml[(w * REP + h) * 2]);
        float ls = 0.f, os = 0.f;
#pragma unroll
        for (int w = 0; w < TC_WARPS; w++) {
            const float mw = wml[(w * REP + h) * 2];
            const float e = mw == -INFINITY ? 0.f : exp2f(mw - mm);
            ls = fmaf(wml[(w * REP + h) * 2 + 1], e, ls);
            os = fmaf(wo[((size_t)w * REP + h) * D + d], e, os);
        }
        co[h * D + d] = os;
        if (d == 0) {
            cml[2 * h] = mm;
            cml[2 * h + 1] = ls;
        }
    }
    __syncthreads();
    MLXD_TRACE_T(tr_cmerge_)
    // push: CTA s owns outputs [s*SL, (s+1)*SL) of the group (SL = REP*D/CL,
    // within one head); every CTA writes its partial of that slice, with the
    // head's (m, l), into the owner's inbox row `rank`
    constexpr int SL = REP * D / CL;
    constexpr int ROW = 2 + SL;
    float *inbox = reinterpret_cast<float *>(sm + L::inbox);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    for (int e = tid; e < CL * ROW; e += TC_THREADS) {
        const int sidx = e / ROW, k = e % ROW;
        const int oi = sidx * SL + (k >= 2 ? k - 2 : 0);
        const float v = k == 0 ? cml[2 * (oi / D)] : k == 1 ? cml[2 * (oi / D) + 1] : co[oi];
        float *dst = cluster.map_shared_rank(inbox, sidx);
        dst[rank * ROW + k] = v;
    }
    cluster.sync();   // every partial has landed in its owner's inbox
    MLXD_TRACE_T(tr_csync_)
    MLXD_TRACE_REC(tid == 0, 0x71, tr_prep_, tr_loop_, tr_cmerge_)
    if (tid < SL) {
        const int oi = rank * SL + tid;
        const int h = oi / D, d = oi % D;
        float mm = -INFINITY;
#pragma unroll
        for (int r = 0; r < CL; r++) mm = fmaxf(mm, inbox[r * ROW]);
        float ls = 0.f, os = 0.f;
#pragma unroll
        for (int r = 0; r < CL; r++) {
            const float mr = inbox[r * ROW];
            const float e = mr == -INFINITY ? 0.f : exp2f(mr - mm);
            ls = fmaf(inbox[r * ROW + 1], e, ls);
            os = fmaf(inbox[r * ROW + 2 + tid], e, os);
        }
        const int hg = kh * REP + h;
        float val = rbf(os / ls);
        if (a.gate) {
            const float gv = bf2f(qkv[(size_t)hg * qstride + D + d]);
            val = rbf(__fmul_rn(val, sigmoid_bf16(gv)));
        }
        a.out[(size_t)hg * D + d] = f2bf(val);
    }
    MLXD_TRACE_REC(tid == 0, 0x72, tr_csync_, gtime(), gtime())
    MLXD_TRACE_END(0x70)
}

// The dynamic shared memory of a CTA, raised above half of an SM's 228 KB so
// that the device places one CTA per SM: with two attention CTAs on one SM
// the GEMVs that follow ran up to 50% slower on those SMs for the rest of
// the step (Qwen3-8B: 525 tokens/s packed, 585 spread).
template <int D, int REP>
static constexpr size_t tc_smem() {
    return TcSmem<D, REP>::total > 116 * 1024 ? TcSmem<D, REP>::total : 116 * 1024;
}
template <int D, int REP, int CL>
static int tc_prepare() {
    auto kern = attn_tc_kernel<D, REP, CL>;
    static bool configured = false;
    if (!configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem<D, REP>()));
        if (CL > 8) MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        configured = true;
    }
    return 0;
}

// whether `hkv` clusters of CL CTAs can be resident at once
template <int D, int REP, int CL>
static bool tc_fits(int hkv) {
    if (tc_prepare<D, REP, CL>()) {
        cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL, hkv);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = tc_smem<D, REP>();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_tc_kernel<D, REP, CL>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return n >= hkv;
}

template <int D, int REP, int CL>
static int tc_launch_cl(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL, a.hkv);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = tc_smem<D, REP>();
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, attn_tc_kernel<D, REP, CL>, a));
    return 0;
}

// clusters of 16 CTAs per kv head when hkv of them fit at once, else 8;
// -1 when neither fits (the split-merge kernel serves)
template <int D, int REP>
static int tc_cluster(int hkv) {
    static int cl_for[65] = {};   // per hkv: 0 unknown, 16, 8 or -1 (none)
    const int key = hkv <= 64 ? hkv : 64;
    if (cl_for[key] == 0) cl_for[key] = tc_fits<D, REP, 16>(hkv) ? 16 : tc_fits<D, REP, 8>(hkv) ? 8 : -1;
    return cl_for[key];
}
template <int D, int REP>
static int tc_launch(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    const int cl = tc_cluster<D, REP>(a.hkv);
    if (cl == 16) return tc_launch_cl<D, REP, 16>(a, st, pdl);
    if (cl == 8) return tc_launch_cl<D, REP, 8>(a, st, pdl);
    return 1;
}
template <int D, int REP>
static int tc_sms(const AttnDecodeArgs &a) {
    const int cl = tc_cluster<D, REP>(a.hkv);
    return cl > 0 ? cl * a.hkv : 0;
}

static bool tc_on() {
    static const bool on = [] {
        const char *e = getenv("MLXD_ATTN_TC");
        return !e || atoi(e) != 0;
    }();
    return on;
}

#define MLXD_TC_DISPATCH(FN, ...)                                   \
    const int D = a.rope.D, rep = a.hq / a.hkv;                     \
    if (a.rope.rope_dims != D || a.hkv > 64) return NONE;           \
    if (D == 128) {                                                 \
        switch (rep) {                                              \
        case 1: return FN<128, 1>(__VA_ARGS__);                     \
        case 2: return FN<128, 2>(__VA_ARGS__);                     \
        case 4: return FN<128, 4>(__VA_ARGS__);                     \
        case 8: return FN<128, 8>(__VA_ARGS__);                     \
        }                                                           \
    } else if (D == 64) {                                           \
        switch (rep) {                                              \
        case 1: return FN<64, 1>(__VA_ARGS__);                      \
        case 2: return FN<64, 2>(__VA_ARGS__);                      \
        case 4: return FN<64, 4>(__VA_ARGS__);                      \
        case 8: return FN<64, 8>(__VA_ARGS__);                      \
        }                                                           \
    }                                                               \
    return NONE;

// 0: launched; 1: this kernel does not serve the shape (the caller falls back);
// -1: error. MLXD_ATTN_TC=0 turns it off.
int attention_decode_tc(const AttnDecodeArgs &a, cudaStream_t st, bool pdl) {
    constexpr int NONE = 1;
    if (!tc_on()) return NONE;
    MLXD_TC_DISPATCH(tc_launch, a, st, pdl)
}

int attention_decode_tc_sms(const AttnDecodeArgs &a) {
    constexpr int NONE = 0;
    if (!tc_on()) return NONE;
    MLXD_TC_DISPATCH(tc_sms, a)
}
#undef MLXD_TC_DISPATCH

}  // namespace mlxd
