// Integer-MMA decode GEMV building blocks (group 64, bf16 scales/biases),
// shared by the per-projection kernel (qgemv.cu) and the persistent decode
// step (megastep.cu). The arithmetic is described in qgemv.cu above
// qgemv_i8_kernel: x as a fixed-point vector X = round(x * 2^(20-E)) split
// into three int8 digits, u8 weight nibbles, mma.m16n8k32 with s32
// accumulation, scale and bias applied per group pair in f32.
#pragma once
#include "common.cuh"

namespace mlxd {

constexpr int I8_DIGITS = 3;
constexpr int I8_ENT = 4 * I8_DIGITS;   // B-fragment entries per group: (digit, t)

MLXD_DEV void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Stage x (bf16 [cols], optionally RMS-normalised with the oracle's
// association: Ta element-strided partials, butterfly within each warp, warp
// totals in order) as B fragments xb[group][digit][t] (16 B: b0, b1 of the
// low-nibble MMA, b0, b1 of the high-nibble MMA) plus, per block of 8 groups,
// the bias multipliers xsum4[t][j] (group 8bk + 2j + (t >> 1): its sum for
// even t, 0 for odd t). xraw: cols bf16 of scratch; zero16: a 16-byte entry
// set to zero. Returns 2^(E-20) (NaN when x holds a non-finite value, so that
// the outputs are NaN as in the f32 sum). Ends with a CTA barrier.
//
// Work unit: item it = 16 g + 8 m + 4 b + t covers the 4 features
// 64 g + 32 m + 16 b + 4 t .. +3, i.e. one byte of each digit plane; the 16
// items of a group sit in 16 consecutive threads. x is read once from global
// memory in this layout (and, for the norm, also in the strided layout of the
// sum of squares, both loads in flight together); the norm weights are read
// before the caller waits on the producer (i8_stage_pre).
template <int NT>
struct I8Pre {
    static constexpr int MAXI = 4;       // items per thread kept in registers
    uint2 w[MAXI];                       // norm weights of the thread's items
};
template <int NT>
MLXD_DEV void i8_stage_pre(I8Pre<NT> &pre, const uint16_t *norm_w, int n) {
    if (!norm_w) return;
    const int ni = n / 4;
#pragma unroll
    for (int k = 0; k < I8Pre<NT>::MAXI; k++) {
        const int it = threadIdx.x + k * NT;
        if (it < ni) {
            const int g = it >> 4, r = it & 15;
            pre.w[k] = *reinterpret_cast<const uint2 *>(norm_w + g * 64 + (r >> 3) * 32 + ((r >> 2) & 1) * 16 + (r & 3) * 4);
        }
    }
}
MLXD_DEV int i8_feature(int it) {
    const int g = it >> 4, r = it & 15;
    return g * 64 + (r >> 3) * 32 + ((r >> 2) & 1) * 16 + (r & 3) * 4;
}
// s_red, s_max: NT/32 entries each, 16-byte aligned (NT a multiple of 128)
template <int NT>
MLXD_DEV float i8_stage(const uint16_t *x, const uint16_t *norm_w, int n, float eps, uint16_t *xraw,
                        uint32_t *xbw, float *xsum4, uint32_t *zero16, float *s_red, unsigned *s_max,
                        const I8Pre<NT> &pre) {
    constexpr int MAXI = I8Pre<NT>::MAXI;
    const bool NORM = norm_w != nullptr;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ni = n / 4, ng = n / 64;
    if (tid < 4) zero16[tid] = 0u;
    // x in the item layout (the first MAXI items of the thread in registers)
    uint2 xv[MAXI];
#pragma unroll
    for (int k = 0; k < MAXI; k++) {
        const int it = tid + k * NT;
        if (it < ni) xv[k] = *reinterpret_cast<const uint2 *>(x + i8_feature(it));
    }
    MLXD_TRACE_T(st0_)
    float inv = 1.f;
    if (NORM) {
        const int Ta = n >= 1024 ? 256 : (n >= 256 ? 128 : 32);
        float acc = 0.f;
        if (tid < Ta)
            for (int base = tid; base < n; base += 16 * Ta) {
                // 16 strided loads in flight, then the partial in element order
                float f[16];
#pragma unroll
                for (int j = 0; j < 16; j++) f[j] = base + j * Ta < n ? bf2f(x[base + j * Ta]) : 0.f;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (base + j * Ta < n) acc = fmaf(f[j], f[j], acc);
            }
        acc = warp_sum(acc);
        if (lane == 0) s_red[warp] = acc;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < NT / 32; w += 4) {   // 16-byte loads in flight together, sum in order
            const float4 r4 = *reinterpret_cast<const float4 *>(s_red + w);
            tot += r4.x;
            tot += r4.y;
            tot += r4.z;
            tot += r4.w;
        }
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    }
    MLXD_TRACE_T(st1_)
    // normalised values (bf16) of the thread's items, group sums, max |x|
    unsigned mx = 0u;
    for (int k0 = 0; k0 * NT < ni; k0 += MAXI) {
#pragma unroll
        for (int k = 0; k < MAXI; k++) {
            const int it = tid + (k0 + k) * NT;
            const bool in = it < ni;
            uint2 v = make_uint2(0u, 0u);
            if (in) {
                if (k0 == 0) {
                    v = xv[k];
                } else {
                    v = *reinterpret_cast<const uint2 *>(x + i8_feature(it));
                }
                if (NORM) {
                    const uint2 wv = k0 == 0 ? pre.w[k]
                                             : *reinterpret_cast<const uint2 *>(norm_w + i8_feature(it));
                    uint32_t *e = &v.x;
                    const uint32_t w2[2] = {wv.x, wv.y};
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const float lo = rbf(__fmul_rn(lo_bf(w2[q]), rbf(__fmul_rn(lo_bf(e[q]), inv))));
                        const float hi = rbf(__fmul_rn(hi_bf(w2[q]), rbf(__fmul_rn(hi_bf(e[q]), inv))));
                        e[q] = pack_bf2(lo, hi);
                    }
                }
                *reinterpret_cast<uint2 *>(xraw + 4 * it) = v;   // item order
                mx = max(mx, max(max(v.x & 0x7fffu, (v.x >> 16) & 0x7fffu),
                                 max(v.y & 0x7fffu, (v.y >> 16) & 0x7fffu)));
            }
            // group sum: the 16 items of a group are 16 consecutive threads
            float sm = (lo_bf(v.x) + hi_bf(v.x)) + (lo_bf(v.y) + hi_bf(v.y));
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            sm += __shfl_xor_sync(0xffffffffu, sm, 2);
            sm += __shfl_xor_sync(0xffffffffu, sm, 4);
            sm += __shfl_xor_sync(0xffffffffu, sm, 8);
            if (in && (it & 15) == 0) {
                const int g = it >> 4;
                const int bk = g >> 3, j = (g & 7) >> 1, h = g & 1;
                xsum4[bk * 16 + (2 * h) * 4 + j] = sm;
                xsum4[bk * 16 + (2 * h + 1) * 4 + j] = 0.f;
            }
        }
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    if (lane == 0) s_max[warp] = mx;
    __syncthreads();
    mx = 0u;
#pragma unroll
    for (int w = 0; w < NT / 32; w += 4) {
        const uint4 m4 = *reinterpret_cast<const uint4 *>(s_max + w);
        mx = max(max(mx, max(m4.x, m4.y)), max(m4.z, m4.w));
    }
    MLXD_TRACE_T(st2_)
    int E = (int)(mx >> 7) - 127;            // exponent of the largest |x|
    if (E < -100) E = -100;                  // zero / subnormal: digits round to 0
    const float sc = __int_as_float((127 + 20 - E) << 23);
    // round(x * sc) + 1.5 * 2^23 as an f32 (|x * sc| < 2^21, one rounding):
    // its low 22 bits are those of X = round(x * sc), so the digits come
    // straight from the bits (d0 = bits 0-6, d1 = 7-13, d2 = 14-21 signed)
    constexpr float MAGIC = 12582912.0f;
    const float lscale = mx >= 0x7f80u ? __int_as_float(0x7fc00000) : __int_as_float((127 + E - 20) << 23);
    // digit planes of each item: one byte per digit
    for (int it = tid; it < ni; it += NT) {
        const int t = it & 3, b = (it >> 2) & 1, m = (it >> 3) & 1, g = it >> 4;
        const uint2 raw = *reinterpret_cast<const uint2 *>(xraw + 4 * it);
        const float xf[4] = {lo_bf(raw.x), hi_bf(raw.x), lo_bf(raw.y), hi_bf(raw.y)};
        uint32_t R[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t X = __float_as_uint(__fmaf_rn(xf[j], sc, MAGIC));
            R[j] = (X & 0x7fu) | ((X << 1) & 0x7f00u) | ((X << 2) & 0xff0000u);
        }
        const uint32_t lo01 = __byte_perm(R[0], R[1], 0x5140), lo23 = __byte_perm(R[2], R[3], 0x5140);
        const uint32_t p0 = __byte_perm(lo01, lo23, 0x5410);
        const uint32_t p1 = __byte_perm(lo01, lo23, 0x7632);
        const uint32_t p2 = __byte_perm(__byte_perm(R[0], R[1], 0x0062), __byte_perm(R[2], R[3], 0x0062), 0x5410);
        uint32_t *e = xbw + ((size_t)g * I8_ENT + t) * 4 + 2 * m + b;
        e[0] = p0;
        e[16] = p1;
        e[32] = p2;
    }
    __syncthreads();
    MLXD_TRACE_REC(threadIdx.x == 0, 0x80 + (NORM ? 1 : 0), st1_ - st0_, st2_ - st1_, gtime() - st2_)
    return lscale;
}

// A lane's view of the staged x: its B-fragment entries for the two groups of
// a pair (group parity h = gq >> 2, digit gq & 3; digit 3 and the other
// parity read the zero entry), its bias multipliers and its digit weight
struct I8Lane {
    const uint4 *xb0, *xb1;
    int st0, st1;
    const float *xsum4;
    float lt;
};
MLXD_DEV I8Lane i8_lane(const uint32_t *xbw, const float *xsum4, const uint32_t *zero16, float lscale) {
    const int lane = threadIdx.x & 31, t = lane & 3, gq = lane >> 2;
    const int dg = gq & 3, hh = gq >> 2;
    const uint4 *xb = reinterpret_cast<const uint4 *>(xbw);
    const uint4 *zero = reinterpret_cast<const uint4 *>(zero16);
    const bool act0 = dg < I8_DIGITS && hh == 0, act1 = dg < I8_DIGITS && hh == 1;
    I8Lane L;
    L.xb0 = act0 ? xb + dg * 4 + t : zero;
    L.xb1 = act1 ? xb + I8_ENT + dg * 4 + t : zero;
    L.st0 = act0 ? 2 * I8_ENT : 0;   // per group pair
    L.st1 = act1 ? 2 * I8_ENT : 0;
    L.xsum4 = xsum4 + t * 4;
    L.lt = (t & 1) ? lscale * 16384.f : lscale;
    return L;
}

// One item (8 tiles of one row block, groups 8bk..8bk+7): the lane's words w
// of the 8 tiles and its two scale/bias words sA (pairs 0, 1), sB (pairs 2,
// 3). refill(p) runs as soon as w[p] has been read (a register pipeline loads
// the next item's tile p there). Returns the item's partial sums of rows g
// and g+8 (quad-reduced: every lane of a quad holds them).
struct I8NoRefill {
    MLXD_DEV void operator()(int) const {}
};
template <typename W, typename F>
MLXD_DEV void i8_item(W &w, const uint4 &sA, const uint4 &sB, const I8Lane &L, int bk, float &y0_out,
                      float &y1_out, F refill) {
    constexpr uint32_t M4 = 0x0f0f0f0fu;
    const float4 xs = *reinterpret_cast<const float4 *>(L.xsum4 + bk * 16);
    const float xsj[4] = {xs.x, xs.y, xs.z, xs.w};
    const uint32_t sbw[8] = {sA.x, sA.y, sA.z, sA.w, sB.x, sB.y, sB.z, sB.w};
    float y0 = 0.f, y1 = 0.f, yb0 = 0.f, yb1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        int acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const uint4 wv = w[2 * j + u];
            refill(2 * j + u);
            const int pair = bk * 4 + j;
            const uint4 bq = u == 0 ? L.xb0[pair * L.st0] : L.xb1[pair * L.st1];
            const uint32_t alo[4] = {wv.x & M4, wv.y & M4, wv.z & M4, wv.w & M4};
            const uint32_t ahi[4] = {(wv.x >> 4) & M4, (wv.y >> 4) & M4, (wv.z >> 4) & M4, (wv.w >> 4) & M4};
            mma_u8s8_16832(acc, alo, bq.x, bq.y);
            mma_u8s8_16832(acc, ahi, bq.z, bq.w);
        }
        const float a0 = fmaf((float)acc[1], 128.f, (float)acc[0]);
        const float a1 = fmaf((float)acc[3], 128.f, (float)acc[2]);
        const uint32_t r0 = sbw[2 * j], r1 = sbw[2 * j + 1];
        y0 = fmaf(lo_bf(r0), a0, y0);
        y1 = fmaf(lo_bf(r1), a1, y1);
        yb0 = fmaf(hi_bf(r0), xsj[j], yb0);
        yb1 = fmaf(hi_bf(r1), xsj[j], yb1);
    }
    y0 = fmaf(y0, L.lt, yb0);
    y1 = fmaf(y1, L.lt, yb1);
    y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
    y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
    y0_out = y0;
    y1_out = y1;
}

}  // namespace mlxd
