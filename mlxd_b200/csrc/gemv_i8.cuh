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
template <int NT>
MLXD_DEV float i8_stage(const uint16_t *x, const uint16_t *norm_w, int n, float eps, uint16_t *xraw,
                        uint32_t *xbw, float *xsum4, uint32_t *zero16, float *s_red, unsigned *s_max) {
    constexpr int MAXV = 4;
    const bool NORM = norm_w != nullptr;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nv = n / 8, ng = n / 64;
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
    const uint4 *w4 = reinterpret_cast<const uint4 *>(norm_w);
    if (tid < 4) zero16[tid] = 0u;
    for (int base = 0; base < nv; base += NT * MAXV) {
        uint4 v[MAXV];
#pragma unroll
        for (int j = 0; j < MAXV; j++) {
            const int i = base + tid + j * NT;
            if (i < nv) v[j] = x4[i];
        }
#pragma unroll
        for (int j = 0; j < MAXV; j++) {
            const int i = base + tid + j * NT;
            if (i < nv) reinterpret_cast<uint4 *>(xraw)[i] = v[j];
        }
    }
    if (NORM) {
        __syncthreads();
        const int Ta = n >= 1024 ? 256 : (n >= 256 ? 128 : 32);
        float acc = 0.f;
        if (tid < Ta)
            for (int i = tid; i < n; i += Ta) {
                const float f = bf2f(xraw[i]);
                acc = fmaf(f, f, acc);
            }
        acc = warp_sum(acc);
        if (lane == 0) s_red[warp] = acc;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < NT / 32; w++) tot += s_red[w];
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
        for (int base = 0; base < nv; base += NT * MAXV) {
            uint4 wv[MAXV];
#pragma unroll
            for (int j = 0; j < MAXV; j++) {
                const int i = base + tid + j * NT;
                if (i < nv) wv[j] = w4[i];
            }
#pragma unroll
            for (int j = 0; j < MAXV; j++) {
                const int i = base + tid + j * NT;
                if (i >= nv) continue;
                uint4 xv = reinterpret_cast<const uint4 *>(xraw)[i];
                uint32_t *xs4 = &xv.x;
                const uint32_t ws4[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float lo = rbf(__fmul_rn(lo_bf(ws4[q]), rbf(__fmul_rn(lo_bf(xs4[q]), inv))));
                    const float hi = rbf(__fmul_rn(hi_bf(ws4[q]), rbf(__fmul_rn(hi_bf(xs4[q]), inv))));
                    xs4[q] = pack_bf2(lo, hi);
                }
                reinterpret_cast<uint4 *>(xraw)[i] = xv;
            }
        }
    }
    __syncthreads();
    // group sums (bias multipliers) and the largest magnitude
    unsigned mx = 0u;
    for (int g = warp; g < ng; g += NT / 32) {
        const uint32_t v = reinterpret_cast<const uint32_t *>(xraw)[g * 32 + lane];
        mx = max(mx, max(v & 0x7fffu, (v >> 16) & 0x7fffu));
        const float sm = warp_sum(lo_bf(v) + hi_bf(v));
        if (lane == 0) {
            const int bk = g >> 3, j = (g & 7) >> 1, h = g & 1;
            xsum4[bk * 16 + (2 * h) * 4 + j] = sm;
            xsum4[bk * 16 + (2 * h + 1) * 4 + j] = 0.f;
        }
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    if (lane == 0) s_max[warp] = mx;
    __syncthreads();
    mx = 0u;
#pragma unroll
    for (int w = 0; w < NT / 32; w++) mx = max(mx, s_max[w]);
    int E = (int)(mx >> 7) - 127;            // exponent of the largest |x|
    if (E < -100) E = -100;                  // zero / subnormal: digits round to 0
    const float sc = __int_as_float((127 + 20 - E) << 23);
    const float lscale = mx >= 0x7f80u ? __int_as_float(0x7fc00000) : __int_as_float((127 + E - 20) << 23);
    // digit planes: item (g, m, b, t) covers group columns 32m + 16b + 4t + j
    for (int it = tid; it < ng * 16; it += NT) {
        const int t = it & 3, b = (it >> 2) & 1, m = (it >> 3) & 1, g = it >> 4;
        const int k0 = g * 64 + 32 * m + 16 * b + 4 * t;
        const uint2 raw = *reinterpret_cast<const uint2 *>(xraw + k0);
        const float xf[4] = {lo_bf(raw.x), hi_bf(raw.x), lo_bf(raw.y), hi_bf(raw.y)};
        uint32_t R[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int X = __float2int_rn(__fmul_rn(xf[j], sc));
            R[j] = ((uint32_t)X & 0x7fu) | (((uint32_t)X << 1) & 0x7f00u) | (((uint32_t)X << 2) & 0xff0000u);
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
