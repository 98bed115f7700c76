// Integer-MMA decode GEMV building blocks (group 64, bf16 scales/biases).
//
// The arithmetic (shared with the oracle, the generic GEMV and the prefill
// GEMM): each group of 64 inputs is written in fixed point on the grid of
// its largest magnitude, E_g = exponent of max|x_k| over the group (clamped
// at -100), X_k = round-to-nearest-even(x_k * 2^(20 - E_g)), |X_k| < 2^21,
// split into three int8 digits X = d0 + 128 d1 + 16384 d2 (d0, d1 in
// [0, 127], d2 signed). u8 weight nibbles x s8 digits on mma.m16n8k32 (s32
// accumulate) give the exact integers P_g = sum_k q_k X_k; the group terms
// s_g P_g 2^(E_g-20) + b_g T_g 2^(E_g-20) (T_g = sum_k X_k) are exact f64
// products, summed in f64 and rounded once to bf16 in the epilogue.
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

// Per-group entry of the staged input (16 bytes): tf = T_g * 2^(E_g - 20)
// (exact; NaN when the group holds a non-finite input) and E_g.
struct GTab {
    double tf;
    int e;
    int pad;
};

// v * 2^(k) for an integer |v| < 2^31, exactly, with one f64 add: the bits of
// (2^52 + 2^31 + v) * 2^k minus (2^52 + 2^31) * 2^k (both exact, Sterbenz).
// k in [-1000, 1000].
MLXD_DEV double int_times_pow2(int v, int k) {
    const int hi = 0x43300000 + k * (1 << 20);
    return __hiloint2double(hi, v ^ (int)0x80000000) - __hiloint2double(hi, (int)0x80000000);
}

// Stage x (bf16 [cols], optionally RMS-normalised with the oracle's
// association: Ta element-strided partials, butterfly within each warp, warp
// totals in order) as B fragments xb[group][digit][t] (16 B: b0, b1 of the
// low-nibble MMA, b0, b1 of the high-nibble MMA) and the group table gt.
// zero16: a 16-byte entry set to zero. Ends with a CTA barrier.
//
// Work unit: item it = 16 g + 8 m + 4 b + t covers the 4 features
// 64 g + 32 m + 16 b + 4 t .. +3, i.e. one byte of each digit plane; the 16
// items of a group sit in 16 consecutive threads, so the group's maximum and
// its digit sum are shuffle reductions within half a warp. The norm weights
// are read before the caller waits on the producer (i8_stage_pre).
template <int NT>
struct I8Pre {
    static constexpr int MAXI = 4;       // items per thread kept in registers
    uint2 w[MAXI];                       // norm weights of the thread's items
};
MLXD_DEV int i8_feature(int it) {
    const int g = it >> 4, r = it & 15;
    return g * 64 + (r >> 3) * 32 + ((r >> 2) & 1) * 16 + (r & 3) * 4;
}
template <int NT>
MLXD_DEV void i8_stage_pre(I8Pre<NT> &pre, const uint16_t *norm_w, int n) {
    if (!norm_w) return;
    const int ni = n / 4;
#pragma unroll
    for (int k = 0; k < I8Pre<NT>::MAXI; k++) {
        const int it = threadIdx.x + k * NT;
        if (it < ni) pre.w[k] = *reinterpret_cast<const uint2 *>(norm_w + i8_feature(it));
    }
}
// s_red: NT/32 floats, 16-byte aligned (NT a multiple of 128)
template <int NT>
MLXD_DEV void i8_stage(const uint16_t *x, const uint16_t *norm_w, int n, float eps, uint32_t *xbw, GTab *gt,
                       uint32_t *zero16, float *s_red, const I8Pre<NT> &pre) {
    constexpr int MAXI = I8Pre<NT>::MAXI;
    const bool NORM = norm_w != nullptr;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ni = n / 4;
    if (tid < 4) zero16[tid] = 0u;
    // x in the item layout (the first MAXI items of the thread in registers)
    uint2 xv[MAXI];
#pragma unroll
    for (int k = 0; k < MAXI; k++) {
        const int it = tid + k * NT;
        if (it < ni) xv[k] = *reinterpret_cast<const uint2 *>(x + i8_feature(it));
    }
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
    // round(x * sc) + 1.5 * 2^23 as an f32 (|x * sc| < 2^21, one rounding):
    // its low 22 bits are those of X = round(x * sc), so the digits come
    // straight from the bits (d0 = bits 0-6, d1 = 7-13, d2 = 14-21 signed)
    constexpr float MAGIC = 12582912.0f;
    for (int k0 = 0; k0 * NT < ni; k0 += MAXI) {
#pragma unroll
        for (int k = 0; k < MAXI; k++) {
            const int it = tid + (k0 + k) * NT;
            const bool in = it < ni;
            uint2 v = make_uint2(0u, 0u);
            if (in) {
                v = k0 == 0 ? xv[k] : *reinterpret_cast<const uint2 *>(x + i8_feature(it));
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
            }
            // the group's largest magnitude (bf16 bits) over its 16 items
            unsigned mx = max(max(v.x & 0x7fffu, (v.x >> 16) & 0x7fffu), max(v.y & 0x7fffu, (v.y >> 16) & 0x7fffu));
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const int eb = (int)(mx >> 7);
            const bool bad = eb == 0xff;
            int E = bad ? 0 : eb - 127;
            if (E < -100) E = -100;
            const float sc = __int_as_float((127 + 20 - E) << 23);
            const float xf[4] = {lo_bf(v.x), hi_bf(v.x), lo_bf(v.y), hi_bf(v.y)};
            uint32_t R[4];
            int tsum = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t X = __float_as_uint(__fmaf_rn(xf[j], sc, MAGIC));
                tsum += (int)X - 0x4B400000;
                R[j] = (X & 0x7fu) | ((X << 1) & 0x7f00u) | ((X << 2) & 0xff0000u);
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, o);
            if (in) {
                const int t = it & 3, b = (it >> 2) & 1, m = (it >> 3) & 1, g = it >> 4;
                const uint32_t lo01 = __byte_perm(R[0], R[1], 0x5140), lo23 = __byte_perm(R[2], R[3], 0x5140);
                const uint32_t p0 = __byte_perm(lo01, lo23, 0x5410);
                const uint32_t p1 = __byte_perm(lo01, lo23, 0x7632);
                const uint32_t p2 =
                    __byte_perm(__byte_perm(R[0], R[1], 0x0062), __byte_perm(R[2], R[3], 0x0062), 0x5410);
                uint32_t *e = xbw + ((size_t)g * I8_ENT + t) * 4 + 2 * m + b;
                e[0] = p0;
                e[16] = p1;
                e[32] = p2;
                if ((it & 15) == 0) {
                    GTab gv;
                    gv.tf = bad ? __longlong_as_double(0x7ff8000000000000ll) : int_times_pow2(tsum, E - 20);
                    gv.e = E;
                    gv.pad = 0;
                    gt[g] = gv;
                }
            }
        }
    }
    __syncthreads();
}

// A lane's view of the staged x: its B-fragment entries for the two groups of
// a pair (group parity h = gq >> 2, digit gq & 3; digit 3 and the other
// parity read the zero entry), its group table and its digit weight
struct I8Lane {
    const uint4 *xb0, *xb1;
    int st0, st1;
    const GTab *gt;   // entry of group 2j + (t >> 1) of block 0 (add 8 bk + 2 j)
    int kshift;       // 14 for the lanes holding digit 2, else 0
    bool bias;        // lanes holding digits 0 and 1 add the bias term
};
MLXD_DEV I8Lane i8_lane(const uint32_t *xbw, const GTab *gt, const uint32_t *zero16) {
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
    L.gt = gt + (t >> 1);
    L.kshift = (t & 1) ? 14 : 0;
    L.bias = (t & 1) == 0;
    return L;
}

// One item (8 tiles of one row block, groups 8bk..8bk+7): the lane's words w
// of the 8 tiles and its two scale/bias words sA (pairs 0, 1), sB (pairs 2,
// 3). refill(p) runs as soon as w[p] has been read (a register pipeline loads
// the next item's tile p there). Returns the item's f64 partial sums of rows
// g and g+8 (quad-reduced: every lane of a quad holds them).
struct I8NoRefill {
    MLXD_DEV void operator()(int) const {}
};
template <typename W, typename F>
MLXD_DEV void i8_item(W &w, const uint4 &sA, const uint4 &sB, const I8Lane &L, int bk, double &y0_out,
                      double &y1_out, F refill) {
    constexpr uint32_t M4 = 0x0f0f0f0fu;
    const uint32_t sbw[8] = {sA.x, sA.y, sA.z, sA.w, sB.x, sB.y, sB.z, sB.w};
    double y0 = 0.0, y1 = 0.0;
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
        // digits 0 and 1 (even t: d0 + 128 d1) or digit 2 (odd t, weight 2^14)
        const int a0 = acc[0] + (acc[1] << 7);
        const int a1 = acc[2] + (acc[3] << 7);
        const GTab g = L.gt[bk * 8 + 2 * j];
        const int k = g.e - 20 + L.kshift;
        const double tf = L.bias ? g.tf : 0.0;
        const uint32_t r0 = sbw[2 * j], r1 = sbw[2 * j + 1];
        y0 = fma((double)lo_bf(r0), int_times_pow2(a0, k), y0);
        y1 = fma((double)lo_bf(r1), int_times_pow2(a1, k), y1);
        y0 = fma((double)hi_bf(r0), tf, y0);
        y1 = fma((double)hi_bf(r1), tf, y1);
    }
    y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
    y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
    y0_out = y0;
    y1_out = y1;
}

// f64 -> bf16 with one correct rounding (to nearest, ties to even): cut to
// f32 toward zero with the lowest bit set when anything was cut (round to
// odd: 24 >= 8 + 2 bits), then round to bf16. The oracle does the same.
MLXD_DEV uint16_t d2bf(double d) {
    if (d != d) return 0x7fc0;
    float f = __double2float_rz(d);
    if ((double)f != d) f = __uint_as_float(__float_as_uint(f) | 1u);
    return f2bf(f);
}

}  // namespace mlxd
