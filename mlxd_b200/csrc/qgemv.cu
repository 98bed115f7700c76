// Decode quantized GEMV (batch 1) and the MLX -> tile repack.
//
// Replaces mlx_quantized_matmul(transpose=true, group, 4, "affine") for one
// token (src/engine/forward.c:17-32, cast to bf16 :46-54). HBM-bound: every
// packed weight byte is read exactly once per token.
//
// Tile layout (written once at load by repack): a row block of 16 output rows
// and one quantisation group (G = 64 or 32 input columns) forms one tile of
// 16*G/2 bytes. Lane L = 4*g + t of a warp owns G/4 contiguous bytes of the
// tile: the nibbles of rows g and g+8 that mma.sync.m16n8k16 needs in its A
// fragment, already in fragment order, so one coalesced 16-byte load per lane
// (512 contiguous bytes per warp) feeds four tensor-core MMAs without a trip
// through shared memory. Dequantisation happens in registers: a LOP3 merges
// two nibbles into the mantissas of bf16 128.0, giving exact bf16 (128 + q);
// the f32 accumulator then yields sum(x*(128+q)) and the affine part is
// applied per group in f32 as
//     y += s * d + (b - 128 s) * sum(x over the group)
// which is mlx's qmv factorisation (scale * sum(x*q) + bias * sum(x)).
#include <mutex>
#include <stdlib.h>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

// ------------------------------------------------------------------ repack

template <int G>
__global__ void repack_tiles_kernel(const uint32_t *__restrict__ w, int ldw, int r0, int c0,
                                    int nrb, int ng, uint8_t *__restrict__ tiles, int dst_rb0,
                                    int dst_rb_stride, int dst_ng) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t total = (size_t)nrb * ng * 32;
    if (idx >= total) return;
    int lane = (int)(idx & 31);
    int g = (int)((idx >> 5) % ng);
    int rb = (int)((idx >> 5) / ng);
    int gq = lane >> 2, t = lane & 3;
    int rowA = r0 + rb * 16 + gq, rowB = rowA + 8;
    auto q = [&](int row, int k) -> uint32_t {
        int col = c0 + g * G + k;
        return (w[(size_t)row * ldw + (col >> 3)] >> (4 * (col & 7))) & 0xFu;
    };
    auto word = [&](int row, const int (&first)[4]) -> uint32_t {
        uint32_t r = 0;
        for (int i = 0; i < 4; i++) {
            r |= q(row, first[i]) << (4 * i);
            r |= q(row, first[i] + 1) << (4 * (i + 4));
        }
        return r;
    };
    int drb = dst_rb0 + dst_rb_stride * rb;
    size_t tile = (size_t)drb * dst_ng + g;
    if (G == 64) {
        const int lo[4] = {2 * t, 16 + 2 * t, 32 + 2 * t, 48 + 2 * t};
        const int hi[4] = {8 + 2 * t, 24 + 2 * t, 40 + 2 * t, 56 + 2 * t};
        uint4 o;
        o.x = word(rowA, lo);
        o.y = word(rowA, hi);
        o.z = word(rowB, lo);
        o.w = word(rowB, hi);
        *reinterpret_cast<uint4 *>(tiles + (tile * 32 + lane) * 16) = o;
    } else {
        const int pr[4] = {2 * t, 8 + 2 * t, 16 + 2 * t, 24 + 2 * t};
        uint2 o;
        o.x = word(rowA, pr);
        o.y = word(rowB, pr);
        *reinterpret_cast<uint2 *>(tiles + (tile * 32 + lane) * 8) = o;
    }
}

template <bool F32>
__global__ void repack_sb_kernel(const void *__restrict__ s, const void *__restrict__ b, int lds,
                                 int r0, int g0, int nrb, int ng, uint8_t *__restrict__ sb,
                                 int dst_rb0, int dst_rb_stride, int dst_ng) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t total = (size_t)nrb * ng * 8;
    if (idx >= total) return;
    int gq = (int)(idx & 7);
    int g = (int)((idx >> 3) % ng);
    int rb = (int)((idx >> 3) / ng);
    int rowA = r0 + rb * 16 + gq, rowB = rowA + 8;
    size_t ia = (size_t)rowA * lds + g0 + g, ib = (size_t)rowB * lds + g0 + g;
    int drb = dst_rb0 + dst_rb_stride * rb;
    size_t rec = ((size_t)drb * dst_ng + g) * 8 + gq;
    if (F32) {
        const float *sf = (const float *)s, *bf = (const float *)b;
        float4 o = make_float4(sf[ia], bf[ia], sf[ib], bf[ib]);
        *reinterpret_cast<float4 *>(sb + rec * 16) = o;
    } else {
        const uint16_t *sh = (const uint16_t *)s, *bh = (const uint16_t *)b;
        uint2 o;
        o.x = (uint32_t)sh[ia] | ((uint32_t)bh[ia] << 16);
        o.y = (uint32_t)sh[ib] | ((uint32_t)bh[ib] << 16);
        *reinterpret_cast<uint2 *>(sb + rec * 8) = o;
    }
}

// scales/biases of the decode fast path: record (rb, bk, lane) = bf16x2 (s, b)
// for (row g, group 8bk+2t), (row g, 8bk+2t+1), (row g+8, 8bk+2t), (row g+8, 8bk+2t+1)
__global__ void repack_sb8_kernel(const uint16_t *__restrict__ s, const uint16_t *__restrict__ b,
                                  int lds, int r0, int g0, int nrb, int nbk,
                                  uint8_t *__restrict__ sb8, int dst_rb0, int dst_rb_stride) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)nrb * nbk * 32) return;
    int lane = (int)(idx & 31);
    int bk = (int)((idx >> 5) % nbk);
    int rb = (int)((idx >> 5) / nbk);
    int gq = lane >> 2, t = lane & 3;
    int rowA = r0 + rb * 16 + gq, rowB = rowA + 8;
    int ga = g0 + bk * 8 + 2 * t, gb = ga + 1;
    auto rec = [&](int row, int grp) -> uint32_t {
        size_t i = (size_t)row * lds + grp;
        return (uint32_t)s[i] | ((uint32_t)b[i] << 16);
    };
    uint4 o = make_uint4(rec(rowA, ga), rec(rowA, gb), rec(rowB, ga), rec(rowB, gb));
    int drb = dst_rb0 + dst_rb_stride * rb;
    *reinterpret_cast<uint4 *>(sb8 + (((size_t)drb * nbk + bk) * 32 + lane) * 16) = o;
}

// Integer-MMA tile layout (group 64): lane L = 4g + t of tile (rb, grp) holds
// four words; word i covers row g + 8(i&1) and group columns
// k = 16(i>>1) + 4t + j (j = 0..3, byte j): its low nibble is q(row, k), its
// high nibble q(row, k + 32). Masking the low nibbles gives the u8 A fragment
// of mma.m16n8k32 for columns 0-31 of the group, shifting and masking the
// high nibbles the one for columns 32-63.
__global__ void repack_i8_kernel(const uint32_t *__restrict__ w, int ldw, int r0, int c0, int nrb,
                                 int ng, uint8_t *__restrict__ tiles, int dst_rb0, int dst_rb_stride,
                                 int dst_ng) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)nrb * ng * 32) return;
    const int lane = (int)(idx & 31);
    const int g = (int)((idx >> 5) % ng);
    const int rb = (int)((idx >> 5) / ng);
    const int gq = lane >> 2, t = lane & 3;
    auto q = [&](int row, int k) -> uint32_t {
        const int col = c0 + g * 64 + k;
        return (w[(size_t)row * ldw + (col >> 3)] >> (4 * (col & 7))) & 0xFu;
    };
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = r0 + rb * 16 + gq + 8 * (i & 1);
        const int kb = 16 * (i >> 1) + 4 * t;
        uint32_t v = 0;
        for (int j = 0; j < 4; j++) v |= (q(row, kb + j) | (q(row, kb + j + 32) << 4)) << (8 * j);
        o[i] = v;
    }
    const size_t tile = (size_t)(dst_rb0 + dst_rb_stride * rb) * dst_ng + g;
    *reinterpret_cast<uint4 *>(tiles + (tile * 32 + lane) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
}

// scale/bias records of the integer-MMA layout: record (rb, bk, g, h), 32 B:
// for j = 0..3, (s, b) of row g then of row g + 8 for group 8bk + 2j + h
__global__ void repack_sbi_kernel(const uint16_t *__restrict__ s, const uint16_t *__restrict__ b,
                                  int lds, int r0, int g0, int nrb, int nbk,
                                  uint8_t *__restrict__ sbi, int dst_rb0, int dst_rb_stride) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)nrb * nbk * 16) return;
    const int h = (int)(idx & 1);
    const int gq = (int)((idx >> 1) & 7);
    const int bk = (int)((idx >> 4) % nbk);
    const int rb = (int)((idx >> 4) / nbk);
    const int rowA = r0 + rb * 16 + gq, rowB = rowA + 8;
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const size_t grp = (size_t)g0 + bk * 8 + 2 * j + h;
        const size_t ia = (size_t)rowA * lds + grp, ib = (size_t)rowB * lds + grp;
        o[2 * j] = (uint32_t)s[ia] | ((uint32_t)b[ia] << 16);
        o[2 * j + 1] = (uint32_t)s[ib] | ((uint32_t)b[ib] << 16);
    }
    const size_t rec = ((size_t)(dst_rb0 + dst_rb_stride * rb) * nbk + bk) * 16 + gq * 2 + h;
    uint4 *dst = reinterpret_cast<uint4 *>(sbi + rec * 32);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

int repack_quant(QMat &dst, const uint32_t *w, const void *s, const void *b, int sdtype, int ldw,
                 int lds, int r0, int nrows, int c0, int dst_rb0, int dst_rb_stride,
                 cudaStream_t st) {
    int G = dst.group;
    if (nrows % 16 || c0 % G || dst.cols % G) {
        set_error("repack: rows must be a multiple of 16 and columns of the group size");
        return -1;
    }
    int nrb = nrows / 16, ng = dst.cols / G;
    size_t nt = (size_t)nrb * ng * 32;
    int blocks = (int)((nt + 255) / 256);
    if (G == 64)
        repack_tiles_kernel<64><<<blocks, 256, 0, st>>>(w, ldw, r0, c0, nrb, ng, dst.tiles, dst_rb0,
                                                       dst_rb_stride, ng);
    else if (G == 32)
        repack_tiles_kernel<32><<<blocks, 256, 0, st>>>(w, ldw, r0, c0, nrb, ng, dst.tiles, dst_rb0,
                                                       dst_rb_stride, ng);
    else {
        set_error("repack: group size %d not supported (32 or 64)", G);
        return -1;
    }
    size_t ns = (size_t)nrb * ng * 8;
    int sblocks = (int)((ns + 255) / 256);
    if (sdtype == MLXD_F32)
        repack_sb_kernel<true><<<sblocks, 256, 0, st>>>(s, b, lds, r0, c0 / G, nrb, ng, dst.sb,
                                                        dst_rb0, dst_rb_stride, ng);
    else
        repack_sb_kernel<false><<<sblocks, 256, 0, st>>>(s, b, lds, r0, c0 / G, nrb, ng, dst.sb,
                                                         dst_rb0, dst_rb_stride, ng);
    if (dst.sb8) {
        int nbk = ng / 8;
        size_t n8 = (size_t)nrb * nbk * 32;
        repack_sb8_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, st>>>(
            (const uint16_t *)s, (const uint16_t *)b, lds, r0, c0 / G, nrb, nbk, dst.sb8, dst_rb0,
            dst_rb_stride);
    }
    if (dst.ti8 && dst.sbi) {
        repack_i8_kernel<<<blocks, 256, 0, st>>>(w, ldw, r0, c0, nrb, ng, dst.ti8, dst_rb0,
                                                 dst_rb_stride, ng);
        const int nbk = ng / 8;
        const size_t ni = (size_t)nrb * nbk * 16;
        repack_sbi_kernel<<<(unsigned)((ni + 255) / 256), 256, 0, st>>>(
            (const uint16_t *)s, (const uint16_t *)b, lds, r0, c0 / G, nrb, nbk, dst.sbi, dst_rb0,
            dst_rb_stride);
    }
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

// ------------------------------------------------------------------ GEMV

template <int G, bool SBF32>
struct Ld {
    using W = typename std::conditional<G == 64, uint4, uint2>::type;
    using S = typename std::conditional<SBF32, uint4, uint2>::type;
};

template <int G>
MLXD_DEV typename Ld<G, false>::W load_w(const uint8_t *p) {
    if constexpr (G == 64) return ldg_nc_v4(p);
    else return ldg_nc_v2(p);
}
template <bool F32>
MLXD_DEV typename std::conditional<F32, uint4, uint2>::type load_sb(const uint8_t *p) {
    if constexpr (F32) return ldg_nc_v4(p);
    else return ldg_nc_v2(p);
}


constexpr int GEMV_THREADS = 512;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int GEMV_P = 8;            // tiles in flight per warp

// Persistent stream-K GEMV. The T = (rows/16) * (cols/G) tiles, in memory
// order, are cut into one contiguous range per warp (equal to within one
// tile), so every warp streams its share of the weights with GEMV_P tile loads
// in flight, issued before the prologue. An epilogue unit is one row block
// (two, gate and up, for SwiGLU); a warp that covers a whole unit finishes it
// from registers, otherwise each contributing warp writes its 16 (or 32)
// partial sums to its own slot of the workspace and the last one to arrive
// (atomic counter) adds the slots in order and runs the epilogue, so the
// result does not depend on arrival order.

// stream-K bookkeeping in "items": one tile (generic kernel) or one block
// of 8 tiles (fast kernel); ipr = items per row block
struct FlushCtx {
    long long T, TW, gw, t_begin, t_end;
    int ipr;
};

template <int EPI>
MLXD_DEV void epilogue_row(const GemvArgs &a, int row, float acc) {
    if constexpr (EPI == EPI_STORE) {
        a.y[row] = f2bf(acc);
    } else if constexpr (EPI == EPI_RESIDUAL) {
        a.y[row] = f2bf(__fadd_rn(bf2f(a.residual[row]), rbf(acc)));
    } else if constexpr (EPI == EPI_PARTIAL_F32) {
        a.yf[row] = acc;
    }
}

MLXD_DEV void argmax_rows(const GemvArgs &a, int lane, int row0, float v0, bool has0, int row1,
                          float v1, bool has1) {
    unsigned long long key = 0ull;
    if (has0) {
        a.y[row0] = f2bf(v0);
        key = argmax_key(rbf(v0), a.row_offset + row0);
    }
    if (has1) {
        a.y[row1] = f2bf(v1);
        unsigned long long k1 = argmax_key(rbf(v1), a.row_offset + row1);
        key = k1 > key ? k1 : key;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if (lane == 0) atomicMax(a.amax, key);
}

// out of line: runs once per row block a warp leaves
template <int EPI>
__device__ __noinline__ void gemv_flush(const GemvArgs &a, const FlushCtx &f, int rb, float y0,
                                        float y1, int count) {
    constexpr int UNIT_RB = EPI == EPI_SWIGLU ? 2 : 1;
    const int lane = threadIdx.x & 31, t = lane & 3, gq = lane >> 2;
    const int ng = f.ipr;
    const int unit = rb / UNIT_RB;
    const int unit_tiles = ng * UNIT_RB;
    if (UNIT_RB == 1 && count == ng) {
        // whole row block in registers: lanes t == 0 hold rows gq, gq + 8
        const int r0 = rb * 16 + gq, r1 = r0 + 8;
        if constexpr (EPI == EPI_ARGMAX) {
            argmax_rows(a, lane, r0, y0, t == 0, r1, y1, t == 0);
        } else if (t == 0) {
            epilogue_row<EPI>(a, r0, y0);
            epilogue_row<EPI>(a, r1, y1);
        }
        return;
    }
    // contributor slot: order of this warp among the unit's warps
    const long long first_tile = (long long)unit * unit_tiles;
    const long long first_w = ((first_tile + 1) * f.TW + f.T - 1) / f.T - 1;
    const int slot = (int)(f.gw - first_w);
    float *rec = a.ws + ((size_t)unit * a.ws_slots + slot) * (16 * UNIT_RB);
    const int half = (rb % UNIT_RB) * 16;
    if (t == 0) {
        rec[half + gq] = y0;
        rec[half + gq + 8] = y1;
        if (UNIT_RB == 2) {
            // a half this warp does not cover is zero in its slot
            if ((rb % 2) == 0 && (long long)(rb + 1) * ng >= f.t_end) {
                rec[16 + gq] = 0.f;
                rec[16 + gq + 8] = 0.f;
            }
            if ((rb % 2) == 1 && (long long)rb * ng <= f.t_begin) {
                rec[gq] = 0.f;
                rec[gq + 8] = 0.f;
            }
        }
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        int old = atomicAdd(&a.cnt[unit], count);
        last = (old + count == unit_tiles);
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    const int nslots = (int)(((first_tile + unit_tiles) * f.TW + f.T - 1) / f.T - 1 - first_w) + 1;
    float accs[UNIT_RB] = {};
    if (lane < 16) {
        for (int sl = 0; sl < nslots; sl++) {
            const float *r = a.ws + ((size_t)unit * a.ws_slots + sl) * (16 * UNIT_RB);
#pragma unroll
            for (int u = 0; u < UNIT_RB; u++) accs[u] += __ldcg(r + u * 16 + lane);
        }
    }
    if (lane == 0) a.cnt[unit] = 0;
    if constexpr (EPI == EPI_SWIGLU) {
        if (lane < 16) a.y[unit * 16 + lane] = f2bf(swiglu_bf16(rbf(accs[0]), rbf(accs[UNIT_RB - 1])));
    } else if constexpr (EPI == EPI_ARGMAX) {
        argmax_rows(a, lane, rb * 16 + lane, accs[0], lane < 16, 0, 0.f, false);
    } else {
        if (lane < 16) epilogue_row<EPI>(a, rb * 16 + lane, accs[0]);
    }
}

// Stage x (bf16 [cols]) for the decode GEMV into shared memory: optional
// RMSNorm with the oracle's association (Ta element-strided partials,
// butterfly within each warp, warp totals in order), then the fragment order
// xp[(gi*4 + tt)*XW + j*2 + hi] and the per-group sums xs[gi]. Global reads
// are 16-byte loads issued MAXV at a time per thread, so the prologue costs a
// few memory latencies instead of one per element. xraw: cols bf16 of scratch
// (used when NORM).
// byte offset of the raw-x scratch after xp (ng*4*XW words) and xs (ng floats)
static __host__ __device__ inline size_t xraw_offset(int ng, int XW) {
    return (((size_t)ng * 4 * XW * 4 + (size_t)ng * 4 + 15) / 16) * 16;
}
template <int G, int NT, bool NORM>
MLXD_DEV void stage_x(const GemvArgs &a, uint32_t *xp, float *xs, uint16_t *xraw, float *s_red) {
    constexpr int XW = G / 8, MAXV = 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nv = a.cols / 8, ng = a.cols / G;
    const uint4 *x4 = reinterpret_cast<const uint4 *>(a.x);
    const uint4 *w4 = reinterpret_cast<const uint4 *>(a.norm_w);
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
            if (i >= nv) continue;
            if (NORM) {
                reinterpret_cast<uint4 *>(xraw)[i] = v[j];
            } else {
                put_pair(xp, G, XW, i * 8 + 0, v[j].x);
                put_pair(xp, G, XW, i * 8 + 2, v[j].y);
                put_pair(xp, G, XW, i * 8 + 4, v[j].z);
                put_pair(xp, G, XW, i * 8 + 6, v[j].w);
            }
        }
    }
    if (NORM) {
        __syncthreads();
        const int n = a.cols;
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
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), a.eps)));
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
                const uint4 xv = reinterpret_cast<const uint4 *>(xraw)[i];
                const uint32_t xs4[4] = {xv.x, xv.y, xv.z, xv.w};
                const uint32_t ws4[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float lo = rbf(__fmul_rn(lo_bf(ws4[q]), rbf(__fmul_rn(lo_bf(xs4[q]), inv))));
                    const float hi = rbf(__fmul_rn(hi_bf(ws4[q]), rbf(__fmul_rn(hi_bf(xs4[q]), inv))));
                    put_pair(xp, G, XW, i * 8 + 2 * q, pack_bf2(lo, hi));
                }
            }
        }
    }
    __syncthreads();
    for (int gi = warp; gi < ng; gi += NT / 32) {
        float sm = 0.f;
        if (lane < 4 * XW) {
            const uint32_t v = xp[gi * 4 * XW + lane];
            sm = lo_bf(v) + hi_bf(v);
        }
        sm = warp_sum(sm);
        if (lane == 0) xs[gi] = sm;
    }
    __syncthreads();
}

template <int G, bool SBF32, int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS, 1) qgemv_kernel(GemvArgs a) {
    constexpr int XW = G / 8;            // x words per (group, t)
    constexpr int WB = G / 4;            // tile bytes per lane
    constexpr int SBB = SBF32 ? 16 : 8;  // sb bytes per record
    using WT = typename Ld<G, false>::W;
    using ST = typename std::conditional<SBF32, uint4, uint2>::type;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int ng = a.cols / G;
    uint32_t *xp = reinterpret_cast<uint32_t *>(smem_raw);
    float *xs = reinterpret_cast<float *>(xp + (size_t)ng * 4 * XW);
    uint16_t *xraw = reinterpret_cast<uint16_t *>(smem_raw + xraw_offset(ng, XW));
    __shared__ float s_red[GEMV_WARPS];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3, gq = lane >> 2;
    FlushCtx f;
    f.ipr = ng;
    f.T = (long long)(a.rows / 16) * ng;
    // active warps: at most one per tile, so every active warp owns >= 1 tile
    f.TW = min((long long)gridDim.x * GEMV_WARPS, f.T);
    f.gw = (long long)blockIdx.x * GEMV_WARPS + warp;
    f.t_begin = f.gw < f.TW ? f.T * f.gw / f.TW : f.T;
    f.t_end = f.gw < f.TW ? f.T * (f.gw + 1) / f.TW : f.T;
    const int n_items = (int)(f.t_end - f.t_begin);
    const uint8_t *pw0 = a.tiles + ((size_t)f.t_begin * 32 + lane) * WB;
    const uint8_t *ps0 = a.sb + ((size_t)f.t_begin * 8 + gq) * SBB;

    WT wbuf[GEMV_P];
    ST sbuf[GEMV_P];
#pragma unroll
    for (int p = 0; p < GEMV_P; p++) {
        if (p < n_items) {
            wbuf[p] = load_w<G>(pw0 + p * 32 * WB);
            sbuf[p] = load_sb<SBF32>(ps0 + p * 8 * SBB);
        }
    }

    // ---- prologue: x (optionally RMS-normalised) into the fragment order
    pdl_wait();
    stage_x<G, GEMV_THREADS, PRO == PRO_RMSNORM>(a, xp, xs, xraw, s_red);
    pdl_trigger();
    if (n_items <= 0) return;

    // ---- main loop: segments of one row block; one compare per tile
    int rb = (int)(f.t_begin / ng);
    int g = (int)(f.t_begin % ng);
    int seg_first = 0;
    int seg_last = min(ng - g, n_items) - 1;
    const uint32_t *xptr = xp + (g * 4 + t) * XW;
    const float *xsp = xs + g;
    float y0 = 0.f, y1 = 0.f;
    for (int base = 0; base < n_items; base += GEMV_P) {
        const uint8_t *pwn = pw0 + (size_t)(base + GEMV_P) * 32 * WB;
        const uint8_t *psn = ps0 + (size_t)(base + GEMV_P) * 8 * SBB;
#pragma unroll
        for (int p = 0; p < GEMV_P; p++) {
            const int i = base + p;
            if (i >= n_items) break;
            WT wv = wbuf[p];
            ST sv = sbuf[p];
            if (i + GEMV_P < n_items) {
                wbuf[p] = load_w<G>(pwn + p * 32 * WB);
                sbuf[p] = load_sb<SBF32>(psn + p * 8 * SBB);
            }
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            const uint4 *xq = reinterpret_cast<const uint4 *>(xptr);
            if constexpr (G == 64) {
                uint4 xa = xq[0], xb = xq[1];
                uint32_t xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint32_t af[4] = {nib_pair(wv.x, j), nib_pair(wv.z, j), nib_pair(wv.y, j),
                                      nib_pair(wv.w, j)};
                    mma_bf16_16816(d, af, xv[2 * j], xv[2 * j + 1]);
                }
            } else {
                uint4 xa = xq[0];
                uint32_t xv[4] = {xa.x, xa.y, xa.z, xa.w};
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    uint32_t af[4] = {nib_pair(wv.x, 2 * j), nib_pair(wv.y, 2 * j),
                                      nib_pair(wv.x, 2 * j + 1), nib_pair(wv.y, 2 * j + 1)};
                    mma_bf16_16816(d, af, xv[2 * j], xv[2 * j + 1]);
                }
            }
            float sA, bA, sB, bB;
            if constexpr (SBF32) {
                sA = __uint_as_float(sv.x); bA = __uint_as_float(sv.y);
                sB = __uint_as_float(sv.z); bB = __uint_as_float(sv.w);
            } else {
                sA = lo_bf(sv.x); bA = hi_bf(sv.x);
                sB = lo_bf(sv.y); bB = hi_bf(sv.y);
            }
            const float xsg = *xsp;
            y0 = fmaf(sA, d[0], y0);
            y0 = fmaf(fmaf(-128.f, sA, bA), xsg, y0);
            y1 = fmaf(sB, d[2], y1);
            y1 = fmaf(fmaf(-128.f, sB, bB), xsg, y1);
            xptr += 4 * XW;
            xsp++;
            if (i == seg_last) {
                gemv_flush<EPI>(a, f, rb, y0, y1, i - seg_first + 1);
                y0 = 0.f;
                y1 = 0.f;
                rb++;
                seg_first = i + 1;
                seg_last = min(i + ng, n_items - 1);
                xptr = xp + t * XW;
                xsp = xs;
            }
        }
    }
}

// Decode fast path (group 64, bf16 scales, cols/64 a multiple of 8). The
// unit of work is a block of 8 consecutive groups of one row block (8 tiles,
// 4 KB contiguous). Its 8 tiles accumulate into ONE mma accumulator, tile p
// feeding N-column p: the B operand is x for the lanes of column p and zero
// for the rest, so after the block the accumulator holds the 8 group partial
// sums of rows g and g+8 spread over the 4 lanes of a quad (columns 2t, 2t+1)
// and the affine step (scale, bias) runs once per (row, group) instead of
// once per lane. Scales/biases arrive as one 16-byte record per lane per
// block (sb8 layout).
template <int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS, 1) qgemv8_kernel(GemvArgs a) {
    MLXD_TRACE_START
    constexpr int G = 64, XW = 8;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int ng = a.cols / G, nbk = ng / 8;
    uint32_t *xp = reinterpret_cast<uint32_t *>(smem_raw);
    float *xs = reinterpret_cast<float *>(xp + (size_t)ng * 4 * XW);
    uint16_t *xraw = reinterpret_cast<uint16_t *>(smem_raw + xraw_offset(ng, XW));
    __shared__ __align__(16) uint32_t s_zero[8];
    __shared__ float s_red[GEMV_WARPS];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3, gq = lane >> 2;
    FlushCtx f;
    f.ipr = nbk;
    f.T = (long long)(a.rows / 16) * nbk;
    f.TW = min((long long)gridDim.x * GEMV_WARPS, f.T);
    f.gw = (long long)blockIdx.x * GEMV_WARPS + warp;
    f.t_begin = f.gw < f.TW ? f.T * f.gw / f.TW : f.T;
    f.t_end = f.gw < f.TW ? f.T * (f.gw + 1) / f.TW : f.T;
    const int n_items = (int)(f.t_end - f.t_begin);
    const uint8_t *pw = a.tiles + ((size_t)f.t_begin * 8 * 32 + lane) * 16;
    const uint8_t *ps = a.sb8 + ((size_t)f.t_begin * 32 + lane) * 16;

    uint4 wbuf[8];
    uint4 sbuf = make_uint4(0, 0, 0, 0);
    if (n_items > 0) {
#pragma unroll
        for (int p = 0; p < 8; p++) wbuf[p] = ldg_nc_v4(pw + p * 512);
        sbuf = ldg_nc_v4(ps);
    }

    // ---- prologue: x (optionally RMS-normalised) into the fragment order
    pdl_wait();
    if (tid < 8) s_zero[tid] = 0u;
    MLXD_TRACE_WAITED
    stage_x<G, GEMV_THREADS, PRO == PRO_RMSNORM>(a, xp, xs, xraw, s_red);
    MLXD_TRACE_END(0x10 + EPI)
    pdl_trigger();
    if (n_items <= 0) return;

    int rb = (int)(f.t_begin / nbk);
    int bk = (int)(f.t_begin % nbk);
    int seg_first = 0;
    int seg_last = min(nbk - bk, n_items) - 1;
    float y0 = 0.f, y1 = 0.f;
    for (int i = 0; i < n_items; i++) {
        const bool pre = i + 1 < n_items;
        const uint8_t *pwn = pw + (size_t)(i + 1) * 4096;
        const uint32_t *xb = xp + ((size_t)bk * 32 + t) * XW;   // group 8bk at +0, +p*32
        // four independent accumulators (one per 16-column chunk of a tile)
        float dj[4][4] = {};
#pragma unroll
        for (int p = 0; p < 8; p++) {
            const uint4 wv = wbuf[p];
            if (pre) wbuf[p] = ldg_nc_v4(pwn + p * 512);
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
        for (int c = 0; c < 4; c++) d[c] = (dj[0][c] + dj[1][c]) + (dj[2][c] + dj[3][c]);
        const uint4 sv = sbuf;
        if (pre) sbuf = ldg_nc_v4(ps + (size_t)(i + 1) * 512);
        const float2 xsv = *reinterpret_cast<const float2 *>(xs + bk * 8 + 2 * t);
        const float s00 = lo_bf(sv.x), b00 = hi_bf(sv.x), s01 = lo_bf(sv.y), b01 = hi_bf(sv.y);
        const float s10 = lo_bf(sv.z), b10 = hi_bf(sv.z), s11 = lo_bf(sv.w), b11 = hi_bf(sv.w);
        y0 = fmaf(s00, d[0], y0);
        y0 = fmaf(fmaf(-128.f, s00, b00), xsv.x, y0);
        y0 = fmaf(s01, d[1], y0);
        y0 = fmaf(fmaf(-128.f, s01, b01), xsv.y, y0);
        y1 = fmaf(s10, d[2], y1);
        y1 = fmaf(fmaf(-128.f, s10, b10), xsv.x, y1);
        y1 = fmaf(s11, d[3], y1);
        y1 = fmaf(fmaf(-128.f, s11, b11), xsv.y, y1);
        if (i == seg_last) {
            // the quad's four lanes hold disjoint groups of rows g, g+8
            y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
            y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
            y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
            y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
            gemv_flush<EPI>(a, f, rb, y0, y1, i - seg_first + 1);
            y0 = 0.f;
            y1 = 0.f;
            rb++;
            bk = 0;
            seg_first = i + 1;
            seg_last = min(i + nbk, n_items - 1);
        } else {
            bk++;
        }
    }
}

// Decode fast path with whole row blocks per CTA (group 64, bf16 scales,
// cols/64 a multiple of 8). CTA c owns units [c*U/G, (c+1)*U/G) (a unit is a
// row block, or a gate|up pair for SwiGLU); warp w takes items w, w+16, ...
// of that range (an item is one block of 8 groups of one row block) and
// holds the next one in registers while computing the current one. Each
// item's 16 partial sums go to their own place in shared memory and the warp
// that completes a unit adds them in item order and runs the epilogue: no
// global workspace, no grid-wide atomics, deterministic.
MLXD_TRACE_BINDER(qgemv)

constexpr int RB_THREADS = 512, RB_WARPS = 16;

// res_s: EPI_RESIDUAL, the unit's 16 residual rows already in shared memory
// (nullptr: read from global memory)
template <int EPI>
MLXD_DEV void rb_epilogue(const GemvArgs &a, const float *ps, int nbk, int unit, int lane,
                          unsigned long long &best, const uint16_t *res_s = nullptr) {
    constexpr int UNIT_RB = EPI == EPI_SWIGLU ? 2 : 1;
    if (lane >= 16) return;
    float acc[UNIT_RB];
#pragma unroll
    for (int u = 0; u < UNIT_RB; u++) {
        float sum = 0.f;
        for (int i = u * nbk; i < (u + 1) * nbk; i++) sum += ps[i * 16 + lane];
        acc[u] = sum;
    }
    const int row = unit * 16 + lane;
    if constexpr (EPI == EPI_SWIGLU) {
        a.y[row] = f2bf(swiglu_bf16(rbf(acc[0]), rbf(acc[UNIT_RB - 1])));
    } else if constexpr (EPI == EPI_ARGMAX) {
        a.y[row] = f2bf(acc[0]);
        const unsigned long long key = argmax_key(rbf(acc[0]), a.row_offset + row);
        best = key > best ? key : best;
    } else if (EPI == EPI_RESIDUAL && res_s) {
        a.y[row] = f2bf(__fadd_rn(bf2f(res_s[lane]), rbf(acc[0])));
    } else {
        epilogue_row<EPI>(a, row, acc[0]);
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(RB_THREADS, 1) qgemv8r_kernel(GemvArgs a, int pool_items) {
    MLXD_TRACE_START
    constexpr int G = 64, XW = 8;
    constexpr int UNIT_RB = EPI == EPI_SWIGLU ? 2 : 1;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(16) uint32_t s_zero[8];
    __shared__ float s_red[RB_WARPS];
    __shared__ unsigned long long s_key[RB_WARPS];
    const int ng = a.cols / G, nbk = ng / 8;
    uint32_t *xp = reinterpret_cast<uint32_t *>(smem_raw);
    float *xs = reinterpret_cast<float *>(xp + (size_t)ng * 4 * XW);
    uint16_t *xraw = reinterpret_cast<uint16_t *>(smem_raw + xraw_offset(ng, XW));
    float *pool = reinterpret_cast<float *>(smem_raw + ((xraw_offset(ng, XW) + (size_t)a.cols * 2 + 15) / 16) * 16);
    int *s_cnt = reinterpret_cast<int *>(pool + (size_t)pool_items * 16);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3, gq = lane >> 2;
    const int n_units = a.rows / 16 / UNIT_RB;
    const int u0 = (int)((long long)n_units * blockIdx.x / gridDim.x);
    const int u1 = (int)((long long)n_units * (blockIdx.x + 1) / gridDim.x);
    const int ipu = nbk * UNIT_RB;
    const int n = (u1 - u0) * ipu;
    const long long i0 = (long long)u0 * ipu;
    for (int i = tid; i < u1 - u0; i += RB_THREADS) s_cnt[i] = 0;

    // the warp's first item streams while the previous kernel finishes
    uint4 wbuf[8];
    uint4 sbuf = make_uint4(0, 0, 0, 0);
    if (warp < n) {
        const uint8_t *pw = a.tiles + (i0 + warp) * 4096 + lane * 16;
#pragma unroll
        for (int p = 0; p < 8; p++) wbuf[p] = ldg_nc_v4(pw + p * 512);
        sbuf = ldg_nc_v4(a.sb8 + (i0 + warp) * 512 + lane * 16);
    }
    l2_prefetch_share(a.pf);
    pdl_wait();
    MLXD_TRACE_WAITED
    if (tid < 8) s_zero[tid] = 0u;
    stage_x<G, RB_THREADS, PRO == PRO_RMSNORM>(a, xp, xs, xraw, s_red);
    pdl_trigger();

    unsigned long long best = 0ull;
    for (int k = warp; k < n; k += RB_WARPS) {
        const bool pre = k + RB_WARPS < n;
        const uint8_t *pwn = a.tiles + (i0 + k + RB_WARPS) * 4096 + lane * 16;
        const int unit = k / ipu;
        const int iu = k - unit * ipu;
        const int bk = iu % nbk;
        const uint32_t *xb = xp + ((size_t)bk * 32 + t) * XW;
        // four independent accumulators (one per 16-column chunk of a tile)
        float dj[4][4] = {};
#pragma unroll
        for (int p = 0; p < 8; p++) {
            const uint4 wv = wbuf[p];
            if (pre) wbuf[p] = ldg_nc_v4(pwn + p * 512);
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
        for (int c = 0; c < 4; c++) d[c] = (dj[0][c] + dj[1][c]) + (dj[2][c] + dj[3][c]);
        const uint4 sv = sbuf;
        if (pre) sbuf = ldg_nc_v4(a.sb8 + (i0 + k + RB_WARPS) * 512 + lane * 16);
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
        float *ps = pool + (size_t)unit * ipu * 16;
        if (t == 0) {
            ps[iu * 16 + gq] = y0;
            ps[iu * 16 + gq + 8] = y1;
        }
        __syncwarp();
        int done = 0;
        if (lane == 0) {
            __threadfence_block();
            done = atomicAdd(&s_cnt[unit], 1) + 1 == ipu;
        }
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done) {
            __threadfence_block();
            rb_epilogue<EPI>(a, ps, nbk, u0 + unit, lane, best);
        }
    }
    if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) s_key[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long m = 0ull;
            for (int w = 0; w < RB_WARPS; w++) m = s_key[w] > m ? s_key[w] : m;
            if (m) atomicMax(a.amax, m);
        }
    }
#ifdef MLXD_TRACE
    __syncthreads();
    MLXD_TRACE_END(0x40 + EPI)
#endif
}

// ---------------------------------------------- integer-MMA decode GEMV
//
// mlx's qmv computes, per output row, sum over groups of
//     scale * sum_k(x_k * q_k) + bias * sum_k(x_k)
// in f32 (src/engine/forward.c:17-32). Here sum_k(x_k * q_k) runs on the
// integer tensor pipe: x is written once per launch as a fixed-point vector
// X_k = round(x_k * 2^(20-E)) with E the exponent of max|x|, so |X_k| < 2^21,
// and X_k is split into three int8 digits X = d0 + 128 d1 + 16384 d2
// (d0, d1 in [0, 127], d2 signed). A bf16 x_k within 13 binades of the
// largest is exact in X; smaller ones round at 2^(E-21), below the rounding
// of an f32 sum of the products. mma.m16n8k32 (u8 weights x s8 digits, s32
// accumulate, exact) then takes 32 columns of 16 rows per instruction with
// its 8 N columns holding (group parity, digit): the two groups of a pair
// share one accumulator, each confined to its own columns. Per pair, a
// lane holds two digit columns of one group for rows g and g+8; it
// recombines them in f32 and applies that group's scale, and lanes with
// even t also add bias * sum(x over the group). The exponent factor is
// applied once per item, and the quad sum gives the item's 16 partials.
// Two MMAs and about twenty instructions per 512-byte tile, against four
// bf16 MMAs and ~67 instructions for the bf16 fragment kernel above.
// smem: raw x (bf16 [cols]), then B fragments xb[group][digit][t] (16 B:
// b0, b1 of the low-nibble MMA, b0, b1 of the high-nibble MMA), then per
// block of 8 groups the bias multipliers xsum4[t][j] (the group sum for even
// t, 0 for odd t), a 16-byte zero entry, the item partials and the counters
struct I8Smem {
    size_t xb, xsum, zero, pool, cnt, res, ring, total;
};
// res: the residual rows of the CTA's units (16 bf16 per unit);
// ring: one 4.6 KB item slot per warp (ring_warps of them) for the item
// requested with cp.async before the producer is waited for
static __host__ __device__ inline I8Smem i8_layout(int cols, int pool_items, int pool_units, int ring_warps = 0) {
    I8Smem L;
    const int ng = cols / 64;
    L.xb = (((size_t)cols * 2 + 15) / 16) * 16;
    L.xsum = L.xb + (size_t)ng * I8_ENT * 16;
    L.zero = L.xsum + (size_t)(ng / 8) * 64;
    L.pool = L.zero + 16;
    L.cnt = L.pool + (size_t)pool_items * 64;
    L.res = ((L.cnt + (size_t)pool_units * 4 + 15) / 16) * 16;
    L.ring = L.res + (size_t)pool_units * 32;
    L.total = L.ring + (size_t)ring_warps * 4608;
    return L;
}

// Whole row blocks per CTA, as qgemv8r_kernel: warp w of the NW warps takes
// items w, w+NW, ... of the CTA's units and keeps the next DEPTH items
// (4 KB of tiles + two 16-byte scale/bias words each) in registers while
// computing the current one, the first DEPTH of them requested before the
// PDL wait.
// SM2: each warp's second item goes to a shared-memory slot by cp.async
// before the wait (DEPTH 1), so two items per warp stream during the wait and
// the staging of x without costing registers
template <int PRO, int EPI, int NW, int DEPTH, bool SM2>
__global__ void __launch_bounds__(NW * 32, 1) qgemv_i8_kernel(GemvArgs a, int pool_items) {
    MLXD_TRACE_START
    constexpr int NT = NW * 32;
    constexpr int UNIT_RB = EPI == EPI_SWIGLU ? 2 : 1;
    static_assert(DEPTH == 1 || DEPTH == 2, "register item buffers");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(16) float s_red[NW];
    __shared__ __align__(16) unsigned s_max[NW];
    __shared__ unsigned long long s_key[NW];
    const int nbk = a.cols / 512;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3, gq = lane >> 2;
    const int n_units = a.rows / 16 / UNIT_RB;
    const int u0 = (int)((long long)n_units * blockIdx.x / gridDim.x);
    const int u1 = (int)((long long)n_units * (blockIdx.x + 1) / gridDim.x);
    const int ipu = nbk * UNIT_RB;
    const int n = (u1 - u0) * ipu;
    const long long i0 = (long long)u0 * ipu;
    static_assert(!SM2 || DEPTH == 1, "the shared-memory item follows one register item");
    const I8Smem L = i8_layout(a.cols, pool_items, (u1 - u0), SM2 ? NW : 0);
    float *pool = reinterpret_cast<float *>(smem_raw + L.pool);
    int *s_cnt = reinterpret_cast<int *>(smem_raw + L.cnt);
    for (int i = tid; i < u1 - u0; i += NT) s_cnt[i] = 0;
    // residual rows complete before the producer started: requested now, 16
    // bytes (8 rows) per thread, waited for by their threads before the
    // staging's last barrier
    uint16_t *s_res = reinterpret_cast<uint16_t *>(smem_raw + L.res);
    const bool res_s = EPI == EPI_RESIDUAL && a.res_early && (reinterpret_cast<uintptr_t>(a.residual) & 15) == 0;
    const bool res_mine = res_s && tid < 2 * (u1 - u0);
    if (res_mine) {
        cp_async16(s_res + 8 * tid, a.residual + (size_t)u0 * 16 + 8 * tid);
        cp_async_commit();
    }

    // the warp's first items stream while the previous kernel finishes
    const uint64_t pol = l2_policy_evict_first();
    const uint8_t *sbl = a.sbi + (gq * 2 + (t >> 1)) * 32;
    uint4 wb[DEPTH][8];
    uint4 sb[DEPTH][2];
    auto load = [&](int d, int k) {
        if (k < n) {
            const uint8_t *pw = a.ti8 + (i0 + k) * 4096 + lane * 16;
#pragma unroll
            for (int p = 0; p < 8; p++) wb[d][p] = ldg_nc_v4_ef(pw + p * 512, pol);
            sb[d][0] = ldg_nc_v4_ef(sbl + (i0 + k) * 512, pol);
            sb[d][1] = ldg_nc_v4_ef(sbl + (i0 + k) * 512 + 16, pol);
        }
    };
#pragma unroll
    for (int d = 0; d < DEPTH; d++) load(d, warp + d * NW);
    unsigned char *slot = smem_raw + L.ring + (size_t)warp * 4608;
    if constexpr (SM2) {
        if (warp + NW < n) {
            const uint8_t *pw = a.ti8 + (i0 + warp + NW) * 4096 + lane * 16;
#pragma unroll
            for (int p = 0; p < 8; p++) cp_async16(slot + p * 512 + lane * 16, pw + p * 512);
            cp_async16(slot + 4096 + lane * 16, a.sbi + (i0 + warp + NW) * 512 + lane * 16);
        }
        cp_async_commit();
    }
    l2_prefetch_share(a.pf);
    I8Pre<NT> pre;
    i8_stage_pre<NT>(pre, PRO == PRO_RMSNORM ? a.norm_w : nullptr, a.cols);
    pdl_wait();
    MLXD_TRACE_WAITED
    if (res_mine) cp_async_wait<0>();
    uint16_t *xraw = reinterpret_cast<uint16_t *>(smem_raw);
    uint32_t *xbw = reinterpret_cast<uint32_t *>(smem_raw + L.xb);
    float *xsum4 = reinterpret_cast<float *>(smem_raw + L.xsum);
    uint32_t *zero16 = reinterpret_cast<uint32_t *>(smem_raw + L.zero);
    const float lscale = i8_stage<NT>(a.x, PRO == PRO_RMSNORM ? a.norm_w : nullptr, a.cols, a.eps, xraw, xbw,
                                      xsum4, zero16, s_red, s_max, pre);
    pdl_trigger();
#ifdef MLXD_TRACE
    const unsigned long long tr_staged_ = gtime();
#endif
    const I8Lane IL = i8_lane(xbw, xsum4, zero16, lscale);

    unsigned long long best = 0ull;
    // the item's 16 partial sums to the pool; the warp completing a unit
    // adds the unit's partials in item order and runs the epilogue
    auto finish = [&](int k, float y0, float y1) {
        const int unit = k / ipu;
        const int iu = k - unit * ipu;
        float *ps = pool + (size_t)unit * ipu * 16;
        if (t == 0) {
            ps[iu * 16 + gq] = y0;
            ps[iu * 16 + gq + 8] = y1;
        }
        __syncwarp();
        int done = 0;
        if (lane == 0) {
            __threadfence_block();
            done = atomicAdd(&s_cnt[unit], 1) + 1 == ipu;
        }
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done) {
            __threadfence_block();
            rb_epilogue<EPI>(a, ps, nbk, u0 + unit, lane, best, res_s ? s_res + unit * 16 : nullptr);
        }
    };
    // item k from register buffer d, refilled with item kn as it is read
    auto process = [&](int d, int k, int kn) {
        const bool more = kn < n;
        const uint8_t *pwn = a.ti8 + (i0 + kn) * 4096 + lane * 16;
        const int bk = (k % ipu) % nbk;
        const uint4 sA = sb[d][0], sB = sb[d][1];
        if (more) {
            sb[d][0] = ldg_nc_v4_ef(sbl + (i0 + kn) * 512, pol);
            sb[d][1] = ldg_nc_v4_ef(sbl + (i0 + kn) * 512 + 16, pol);
        }
        float y0, y1;
        i8_item(wb[d], sA, sB, IL, bk, y0, y1, [&](int p) {
            if (more) wb[d][p] = ldg_nc_v4_ef(pwn + p * 512, pol);
        });
        finish(k, y0, y1);
    };
    if constexpr (SM2) {
        const int cnt = warp < n ? (n - warp + NW - 1) / NW : 0;
        if (cnt > 0) process(0, warp, warp + 2 * NW);
        if (cnt > 1) {
            // the item in the shared-memory slot (the lanes' copies seen by all)
            cp_async_wait<0>();
            __syncwarp();
            uint4 w[8];
#pragma unroll
            for (int p = 0; p < 8; p++) w[p] = *reinterpret_cast<const uint4 *>(slot + p * 512 + lane * 16);
            const unsigned char *rec = slot + 4096 + (gq * 2 + (t >> 1)) * 32;
            const uint4 sA = *reinterpret_cast<const uint4 *>(rec), sB = *reinterpret_cast<const uint4 *>(rec + 16);
            const int k = warp + NW;
            float y0, y1;
            i8_item(w, sA, sB, IL, (k % ipu) % nbk, y0, y1, I8NoRefill{});
            finish(k, y0, y1);
        }
        for (int i = 2; i < cnt; i++) process(0, warp + i * NW, warp + (i + 1) * NW);
    } else {
        for (int k = warp; k < n; k += DEPTH * NW) {
            process(0, k, k + DEPTH * NW);
            if (DEPTH == 2 && k + NW < n) process(DEPTH - 1, k + NW, k + NW + DEPTH * NW);
        }
    }
    if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) s_key[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long m = 0ull;
            for (int w = 0; w < NW; w++) m = s_key[w] > m ? s_key[w] : m;
            if (m) atomicMax(a.amax, m);
        }
    }
#ifdef MLXD_TRACE
    const unsigned long long tr_loop_ = gtime();
    __syncthreads();
    MLXD_TRACE_REC(tid == 0, 0x60 + EPI, tr_staged_, tr_loop_, gtime())
    MLXD_TRACE_END(0x50 + EPI)
#endif
}

// grid and workspace slots of one launch
static bool fast8_shape(int cols, int G) { return G == 64 && (cols / 64) % 8 == 0; }

static void gemv_plan(int rows, int cols, int G, int epi, int sms, int *grid, int *slots,
                      bool fast) {
    const int ipr = fast ? cols / G / 8 : cols / G;   // items per row block
    const long long T = (long long)(rows / 16) * ipr;
    const long long min_items = fast ? 1 : 4;          // per warp
    long long g = (T + GEMV_WARPS * min_items - 1) / (GEMV_WARPS * min_items);
    if (g > sms) g = sms;
    if (g < 1) g = 1;
    *grid = (int)g;
    long long TW = g * GEMV_WARPS < T ? g * GEMV_WARPS : T;
    int unit_tiles = ipr * (epi == EPI_SWIGLU ? 2 : 1);
    long long per_warp = T / TW;   // floor, >= 1 unless T < TW
    long long s = per_warp > 0 ? (unit_tiles + per_warp - 1) / per_warp + 2 : unit_tiles + 1;
    if (s > unit_tiles + 1) s = unit_tiles + 1;
    *slots = (int)s;
}

size_t gemv_workspace_floats(int rows, int cols, int G, int epi, int sms, int *units_out) {
    int grid, slots, g2, s2;
    gemv_plan(rows, cols, G, epi, sms, &grid, &slots, false);
    if (fast8_shape(cols, G)) {
        gemv_plan(rows, cols, G, epi, sms, &g2, &s2, true);
        if (s2 > slots) slots = s2;
    }
    int unit_rb = epi == EPI_SWIGLU ? 2 : 1;
    int units = rows / 16 / unit_rb;
    if (units_out) *units_out = units;
    return (size_t)units * slots * 16 * unit_rb;
}

static int g_sms = 0;
int num_sms() {
    if (!g_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms <= 0) g_sms = 148;
    }
    return g_sms;
}

template <int G, bool SBF32, int PRO, int EPI>
static int launch_gemv(GemvArgs a, cudaStream_t st, bool pdl) {
    auto kern = qgemv_kernel<G, SBF32, PRO, EPI>;
    int ng = a.cols / G;
    size_t smem = xraw_offset(ng, G / 8) + (size_t)a.cols * 2;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    int grid, slots;
    gemv_plan(a.rows, a.cols, G, EPI, num_sms(), &grid, &slots, false);
    a.ws_slots = slots;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
    return 0;
}

template <int PRO, int EPI>
static int launch_gemv8(GemvArgs a, cudaStream_t st, bool pdl) {
    auto kern = qgemv8_kernel<PRO, EPI>;
    int ng = a.cols / 64;
    size_t smem = xraw_offset(ng, 8) + (size_t)a.cols * 2;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    int grid, slots;
    gemv_plan(a.rows, a.cols, 64, EPI, num_sms(), &grid, &slots, true);
    a.ws_slots = slots;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
    return 0;
}


template <int PRO, int EPI>
static int launch_gemv8r(GemvArgs a, cudaStream_t st, bool pdl) {
    auto kern = qgemv8r_kernel<PRO, EPI>;
    const int ng = a.cols / 64;
    const int unit_rb = EPI == EPI_SWIGLU ? 2 : 1;
    const int n_units = a.rows / 16 / unit_rb;
    int grid = num_sms();
    if (grid > n_units) grid = n_units;
    const int per = (n_units + grid - 1) / grid;
    const int pool_items = per * unit_rb * (a.cols / 512);
    const size_t smem = ((xraw_offset(ng, 8) + (size_t)a.cols * 2 + 15) / 16) * 16 + (size_t)pool_items * 64 +
                        (size_t)per * 4;
    if (smem > 200 * 1024) {
        set_error("qgemv: %d x %d needs %zu bytes of shared memory", a.rows, a.cols, smem);
        return -1;
    }
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(RB_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, kern, a, pool_items));
    return 0;
}

template <int PRO, int EPI, int NW, int DEPTH, bool SM2>
static int launch_gemv_i8_cfg(GemvArgs a, cudaStream_t st, bool pdl) {
    auto kern = qgemv_i8_kernel<PRO, EPI, NW, DEPTH, SM2>;
    const int unit_rb = EPI == EPI_SWIGLU ? 2 : 1;
    const int n_units = a.rows / 16 / unit_rb;
    int grid = num_sms();
    if (a.grid_cap > 0 && grid > a.grid_cap) grid = a.grid_cap;
    if (grid > n_units) grid = n_units;
    const int per = (n_units + grid - 1) / grid;
    const int pool_items = per * unit_rb * (a.cols / 512);
    const size_t smem = i8_layout(a.cols, pool_items, per, SM2 ? NW : 0).total;
    if (smem > 220 * 1024) {
        set_error("qgemv: %d x %d needs %zu bytes of shared memory", a.rows, a.cols, smem);
        return -1;
    }
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MLXD_CHECK(cudaLaunchKernelEx(&cfg, kern, a, pool_items));
    return 0;
}

// 16 warps with one item in registers ahead: on Qwen3-8B 608 tokens/s,
// against 582 for 12 warps x 2 items and 479 for 16 x 2 (register spills).
// A launch without programmatic dependent launch (a projection on its own)
// also streams each warp's second item into shared memory before staging x:
// gate|up 15.8 -> 14.4 us, lm_head at 6.43 TB/s. Inside the PDL-chained
// decode graph the same early traffic slows the previous kernel's tail
// (646 -> 614 tokens/s), so chained launches keep one item; loading even that
// one after the wait instead of before it costs 636 -> 589 tokens/s.
// A launch capped to the SMs that the running attention kernel leaves free
// (the o projection) streams two items per warp too: its CTAs are resident
// and idle for the whole attention step.
template <int PRO, int EPI>
static int launch_gemv_i8(GemvArgs a, cudaStream_t st, bool pdl) {
    if (!pdl || a.grid_cap > 0) return launch_gemv_i8_cfg<PRO, EPI, 16, 1, true>(a, st, pdl);
    return launch_gemv_i8_cfg<PRO, EPI, 16, 1, false>(a, st, pdl);
}

static int dispatch_gemv_i8(int pro, int epi, const GemvArgs &a, cudaStream_t st, bool pdl) {
#define MLXD_GEMVI_CASE(P, E) \
    if (pro == P && epi == E) return launch_gemv_i8<P, E>(a, st, pdl);
    MLXD_GEMVI_CASE(PRO_PLAIN, EPI_STORE)
    MLXD_GEMVI_CASE(PRO_PLAIN, EPI_RESIDUAL)
    MLXD_GEMVI_CASE(PRO_PLAIN, EPI_SWIGLU)
    MLXD_GEMVI_CASE(PRO_PLAIN, EPI_ARGMAX)
    MLXD_GEMVI_CASE(PRO_PLAIN, EPI_PARTIAL_F32)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_STORE)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_RESIDUAL)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_SWIGLU)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_ARGMAX)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_PARTIAL_F32)
#undef MLXD_GEMVI_CASE
    set_error("qgemv: bad prologue/epilogue");
    return -1;
}

static int dispatch_gemv8r(int pro, int epi, const GemvArgs &a, cudaStream_t st, bool pdl) {
#define MLXD_GEMVR_CASE(P, E) \
    if (pro == P && epi == E) return launch_gemv8r<P, E>(a, st, pdl);
    MLXD_GEMVR_CASE(PRO_PLAIN, EPI_STORE)
    MLXD_GEMVR_CASE(PRO_PLAIN, EPI_RESIDUAL)
    MLXD_GEMVR_CASE(PRO_PLAIN, EPI_SWIGLU)
    MLXD_GEMVR_CASE(PRO_PLAIN, EPI_ARGMAX)
    MLXD_GEMVR_CASE(PRO_PLAIN, EPI_PARTIAL_F32)
    MLXD_GEMVR_CASE(PRO_RMSNORM, EPI_STORE)
    MLXD_GEMVR_CASE(PRO_RMSNORM, EPI_RESIDUAL)
    MLXD_GEMVR_CASE(PRO_RMSNORM, EPI_SWIGLU)
    MLXD_GEMVR_CASE(PRO_RMSNORM, EPI_ARGMAX)
    MLXD_GEMVR_CASE(PRO_RMSNORM, EPI_PARTIAL_F32)
#undef MLXD_GEMVR_CASE
    set_error("qgemv: bad prologue/epilogue");
    return -1;
}

static int dispatch_gemv8(int pro, int epi, const GemvArgs &a, cudaStream_t st, bool pdl) {
#define MLXD_GEMV8_CASE(P, E) \
    if (pro == P && epi == E) return launch_gemv8<P, E>(a, st, pdl);
    MLXD_GEMV8_CASE(PRO_PLAIN, EPI_STORE)
    MLXD_GEMV8_CASE(PRO_PLAIN, EPI_RESIDUAL)
    MLXD_GEMV8_CASE(PRO_PLAIN, EPI_SWIGLU)
    MLXD_GEMV8_CASE(PRO_PLAIN, EPI_ARGMAX)
    MLXD_GEMV8_CASE(PRO_PLAIN, EPI_PARTIAL_F32)
    MLXD_GEMV8_CASE(PRO_RMSNORM, EPI_STORE)
    MLXD_GEMV8_CASE(PRO_RMSNORM, EPI_RESIDUAL)
    MLXD_GEMV8_CASE(PRO_RMSNORM, EPI_SWIGLU)
    MLXD_GEMV8_CASE(PRO_RMSNORM, EPI_ARGMAX)
    MLXD_GEMV8_CASE(PRO_RMSNORM, EPI_PARTIAL_F32)
#undef MLXD_GEMV8_CASE
    set_error("qgemv: bad prologue/epilogue");
    return -1;
}

template <int G, bool SBF32>
static int dispatch_gemv(int pro, int epi, const GemvArgs &a, cudaStream_t st, bool pdl) {
#define MLXD_GEMV_CASE(P, E) \
    if (pro == P && epi == E) return launch_gemv<G, SBF32, P, E>(a, st, pdl);
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_STORE)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_RESIDUAL)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_SWIGLU)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_ARGMAX)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_PARTIAL_F32)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_PARTIAL_F32)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_STORE)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_RESIDUAL)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_SWIGLU)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_ARGMAX)
#undef MLXD_GEMV_CASE
    set_error("qgemv: bad prologue/epilogue");
    return -1;
}

// decode kernel for the group-64 fast layout: the integer-MMA kernel over the
// ti8/sbi layout (default, 3), the bf16-fragment kernel with whole row blocks
// per CTA (MLXD_GEMV_KIND=2) or its stream-K split over warps (0)
static int g_gemv_kind = [] {
    const char *e = getenv("MLXD_GEMV_KIND");
    return e ? atoi(e) : 3;
}();

int qgemv(const QMat &W, int pro, int epi, GemvArgs a, cudaStream_t st, bool pdl) {
    if (!W.quant) {
        set_error("qgemv: matrix is not quantized");
        return -1;
    }
    a.tiles = W.tiles;
    a.sb = W.sb;
    a.rows = W.rows;
    a.cols = W.cols;
    if (!a.ws || !a.cnt) {
        set_error("qgemv: no workspace");
        return -1;
    }
    if (((uintptr_t)a.x | (uintptr_t)a.norm_w) & 15) {
        set_error("qgemv: x and the norm weights must be 16-byte aligned");
        return -1;
    }
    if (W.rows % (epi == EPI_SWIGLU ? 32 : 16)) {
        set_error("qgemv: rows %d not a multiple of the row block", W.rows);
        return -1;
    }
    if (W.ti8 && W.sbi && W.fast8() && g_gemv_kind == 3) {
        a.ti8 = W.ti8;
        a.sbi = W.sbi;
        return dispatch_gemv_i8(pro, epi, a, st, pdl);
    }
    if (W.sb8 && W.fast8()) {
        a.sb8 = W.sb8;
        if (g_gemv_kind != 0) return dispatch_gemv8r(pro, epi, a, st, pdl);
        return dispatch_gemv8(pro, epi, a, st, pdl);
    }
    bool f32 = W.sdtype == MLXD_F32;
    if (W.group == 64) return f32 ? dispatch_gemv<64, true>(pro, epi, a, st, pdl)
                                  : dispatch_gemv<64, false>(pro, epi, a, st, pdl);
    if (W.group == 32) return f32 ? dispatch_gemv<32, true>(pro, epi, a, st, pdl)
                                  : dispatch_gemv<32, false>(pro, epi, a, st, pdl);
    set_error("qgemv: group size %d not supported", W.group);
    return -1;
}

void qgemv_stream(const QMat &W, std::vector<std::pair<const unsigned char *, size_t>> &out) {
    if (!W.quant) return;
    if (W.ti8 && W.sbi && W.fast8() && g_gemv_kind == 3) {
        out.emplace_back(W.ti8, W.tile_bytes());
        out.emplace_back(W.sbi, W.sb_bytes());
    } else if (W.sb8 && W.fast8()) {
        out.emplace_back(W.tiles, W.tile_bytes());
        out.emplace_back(W.sb8, W.sb_bytes() * 2);
    } else {
        out.emplace_back(W.tiles, W.tile_bytes());
        out.emplace_back(W.sb, W.sb_bytes());
    }
}

// ------------------------------------------ decode GEMV on static scratch
//
// The same decode GEMV for callers that cannot allocate device memory at the
// time they call it: code running inside a caching allocator's callback or
// out-of-memory handler (allocating there re-enters the allocator), and a
// serving loop that owns all device memory up front under a fixed plan (a
// cudaMalloc mid-loop can fail once the plan has taken the HBM, and its
// implicit device synchronisation stalls every stream). Instead of the per-matrix workspace that mlxd_cuda_linear_create allocates,
// the split row-block partial sums and their arrival counters live in one
// fixed array of device memory below: STATIC_WS_FLOATS f32 partials (2 MiB)
// followed by STATIC_WS_UNITS counters, which bounds a matrix at 262144 rows
// and at 2^19 workspace floats (gemv_workspace_floats). Every call on a device
// shares the array, and it keeps what the last call left there: the counters
// are cleared on the caller's stream before each launch (the partial sums are
// always written before they are read). Two calls whose kernels can overlap
// on the GPU, i.e. on streams with no ordering between them, race on the
// array and give wrong results.
constexpr size_t STATIC_WS_FLOATS = (size_t)1 << 19;
constexpr int STATIC_WS_UNITS = 1 << 14;
constexpr int STATIC_MAX_DEVICES = 64;
static __device__ __align__(256) float g_gemv_static_scratch[STATIC_WS_FLOATS + STATIC_WS_UNITS];

// Address of the array on the current device. Looked up once per device, on
// that device's first call (the lookup can load the module, so that first
// call belongs before any stream capture); later calls read the table.
static float *static_scratch_on_current_device() {
    static std::mutex mu;
    static float *addr[STATIC_MAX_DEVICES] = {};
    int dev = 0;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return nullptr;
    if (dev < 0 || dev >= STATIC_MAX_DEVICES) {
        set_error("linear_noalloc: device %d beyond the %d supported", dev, STATIC_MAX_DEVICES);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        if (!cuda_ok(cudaGetSymbolAddress(&p, g_gemv_static_scratch), "cudaGetSymbolAddress"))
            return nullptr;
        addr[dev] = (float *)p;
    }
    return addr[dev];
}

int qgemv_static_scratch(const QMat &W, const uint16_t *x, uint16_t *y, cudaStream_t st) {
    if (!W.quant) {
        set_error("linear_noalloc: matrix is not quantized");
        return -1;
    }
    int units = 0;
    size_t wsf = gemv_workspace_floats(W.rows, W.cols, W.group, EPI_STORE, num_sms(), &units);
    if (wsf > STATIC_WS_FLOATS || units > STATIC_WS_UNITS) {
        set_error("linear_noalloc: a %d x %d matrix needs %zu workspace floats and %d counters; "
                  "the static scratch holds %zu and %d",
                  W.rows, W.cols, wsf, units, STATIC_WS_FLOATS, STATIC_WS_UNITS);
        return -1;
    }
    float *base = static_scratch_on_current_device();
    if (!base) return -1;
    int *cnt = (int *)(base + STATIC_WS_FLOATS);
    MLXD_CHECK(cudaMemsetAsync(cnt, 0, (size_t)units * sizeof(int), st));
    GemvArgs a = {};
    a.x = x;
    a.y = y;
    a.ws = base;
    a.cnt = cnt;
    return qgemv(W, PRO_PLAIN, EPI_STORE, a, st, false);
}

}  // namespace mlxd
