// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMEM),
// in the library's group-exact arithmetic (gemv_i8.cuh).
//
// y[S][rows] = x[S][cols] . deq(W)^T for a chunk of prompt tokens
// (mlx_quantized_matmul at S > 1, src/engine/forward.c:17-32), W 4-bit with
// group 64 and bf16 scales/biases. Each token's input is first written in
// per-group fixed point (xq_kernel: three int8 digits per input, the group
// exponents and T_g * 2^(E_g - 20)); then per CTA tile of 128 weight rows x
// 64 tokens the tensor cores form the exact integer digit sums of every
// group and the epilogue warps turn each group's sums into its f64 terms:
//
//   warp 0, one lane   TMA: the digit tile (192 rows: token t, digit d at
//                      row 3t + d; 128 columns = two groups, 128B swizzle)
//                      and the two groups' table entries of the 64 tokens
//                      into stage s;
//   warps 1-2          the weight tile of the stage: 128 rows x 128 columns
//                      of nibbles from the MLX array, widened to u8 in the
//                      K-major 128B-swizzled layout, and the rows' scale and
//                      bias of the two groups;
//   warp 3, one lane   per group: two tcgen05.mma.kind::i8 (M 128, N 192,
//                      K 32; u8 weights x s8 digits -> s32 in TMEM) into one
//                      of two TMEM buffers, then tcgen05.commit;
//   warps 4-11         per group: tcgen05.ld of the buffer (warpgroup w: its
//                      32 tokens), P = d0 + 128 d1 + 16384 d2 per (row,
//                      token), acc += s * P * 2^(E - 20) + b * tf in f64; at
//                      the end the epilogue (store / +residual / SwiGLU / f64
//                      partial) rounds each value once.
// Every mbarrier wait gives up after 0.5 s and sets an error word the host
// reads; TMEM is released on every path.
#include <cuda.h>
#include <mutex>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

constexpr int XG_BM = 128, XG_TOK = 64, XG_BN = 3 * XG_TOK, XG_BK = 128, XG_NS = 3;
constexpr int XG_THREADS = 640;   // 4 warps (TMA, 2 producers, MMA) + 16 epilogue warps
constexpr int XG_ABYTES = XG_BM * XG_BK;             // 16 KB of u8 weights
constexpr int XG_BBYTES = XG_BN * XG_BK;             // 24 KB of digits
constexpr int XG_TBYTES = 2 * XG_TOK * 16;           // 2 KB of table entries
constexpr int XG_SBYTES = 2 * XG_BM * 4;             // 1 KB of (scale, bias)
constexpr int XG_STAGE = XG_ABYTES + XG_BBYTES + XG_TBYTES + XG_SBYTES;
constexpr size_t XG_SMEM = 1024 + (size_t)XG_NS * XG_STAGE + 256 + (size_t)XG_BM * XG_TOK / 2 * 8;

static __device__ int g_xgemm_err;

// per (group, token) entry of the GEMM's input table: tf = T_g * 2^(E_g - 20)
// (NaN for a non-finite group), E_g, and the high word 0x43300000 +
// (E_g - 20) << 20 that scales a group sum by 2^(E_g - 20) (int_times_pow2),
// made once here instead of per output row
struct XTab {
    double tf;
    int e;
    int hi;
};

// v * 2^(E_g - 20) for |v| < 2^31, exactly: int_times_pow2 with the table's
// high word
MLXD_DEV double int_times_pow2_hi(int v, int hi) {
    return __hiloint2double(hi, v ^ (int)0x80000000) - __hiloint2double(hi, (int)0x80000000);
}

// K-major operand with 128-byte rows in the 128B swizzle: 8-row atoms of
// 1024 B (stride byte offset), leading offset unused (1), descriptor version 1
MLXD_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                      // leading byte offset (16 B units)
    d |= (uint64_t)(1024 >> 4) << 32;            // stride byte offset
    d |= (uint64_t)1 << 46;                      // version
    d |= (uint64_t)2 << 61;                      // SWIZZLE_128B
    return d;
}
// kind::i8 instruction descriptor: s32 accumulator (2 at bit 4), A u8 (0 at
// bit 7), B s8 (1 at bit 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t umma_idesc_u8s8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

MLXD_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MLXD_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MLXD_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

MLXD_DEV void tmem_ld16(uint32_t (&v)[16], uint32_t ta) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(ta));
}
MLXD_DEV void tmem_ld8(uint32_t (&v)[8], uint32_t ta) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(ta));
}

// 8 nibbles (elements 0..7, LSB first) of one MLX word widened to 8 bytes
MLXD_DEV uint2 widen_nibbles(uint32_t w) {
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
    return make_uint2(__byte_perm(lo, hi, 0x5140), __byte_perm(lo, hi, 0x7362));
}

// Inputs in per-group fixed point for the GEMM: one warp per (token, group);
// xd [S_pad][3][cols] int8 digits (rows past S are zero), tab [ng][S_pad]
__global__ void xq_kernel(const uint16_t *__restrict__ x, int S, int S_pad, int cols, int8_t *__restrict__ xd,
                          XTab *__restrict__ tab) {
    const int ng = cols / 64;
    const int wg = (int)(((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (wg >= ng * S_pad) return;
    const int s = wg / ng, g = wg % ng;
    uint32_t v = 0u;   // two bf16 inputs
    if (s < S) v = *reinterpret_cast<const uint32_t *>(x + (size_t)s * cols + (size_t)g * 64 + 2 * lane);
    unsigned mx = max(v & 0x7fffu, (v >> 16) & 0x7fffu);
    mx = __reduce_max_sync(0xffffffffu, mx);
    const int eb = (int)(mx >> 7);
    const bool bad = eb == 0xff;
    int E = bad ? 0 : eb - 127;
    if (E < -100) E = -100;
    const float sc = __int_as_float((127 + 20 - E) << 23);
    constexpr float MAGIC = 12582912.0f;
    int X[2], tsum = 0;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const float xf = j ? hi_bf(v) : lo_bf(v);
        X[j] = bad ? 0 : (int)__float_as_uint(__fmaf_rn(xf, sc, MAGIC)) - 0x4B400000;
        tsum += X[j];
    }
    tsum = __reduce_add_sync(0xffffffffu, tsum);
#pragma unroll
    for (int d = 0; d < 3; d++) {
        uint32_t b2 = 0;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const uint32_t u = (uint32_t)X[j];
            const uint32_t digit = d == 0 ? (u & 0x7fu) : d == 1 ? ((u >> 7) & 0x7fu) : ((u >> 14) & 0xffu);
            b2 |= digit << (8 * j);
        }
        *reinterpret_cast<uint16_t *>(xd + ((size_t)s * 3 + d) * cols + (size_t)g * 64 + 2 * lane) = (uint16_t)b2;
    }
    if (lane == 0) {
        XTab e;
        e.tf = bad ? __longlong_as_double(0x7ff8000000000000ll) : int_times_pow2(tsum, E - 20);
        e.e = E;
        e.hi = 0x43300000 + (E - 20) * (1 << 20);
        tab[(size_t)g * S_pad + s] = e;
    }
}

template <int EPI>
__global__ void __launch_bounds__(XG_THREADS, 1)
    qgemm_x_kernel(const __grid_constant__ CUtensorMap tmd, const uint32_t *__restrict__ w, const uint16_t *__restrict__ sg,
                   const uint16_t *__restrict__ bg, const XTab *__restrict__ tab, int rows, int cols, int S, int S_pad,
                   uint16_t *__restrict__ y, const uint16_t *__restrict__ residual, double *__restrict__ yf) {
    extern __shared__ __align__(1024) unsigned char xsm_raw[];
    unsigned char *xsm = reinterpret_cast<unsigned char *>(((uintptr_t)xsm_raw + 1023) & ~(uintptr_t)1023);
    // stage s: [A 16 KB][B 24 KB][tables 2 KB][scale/bias 1 KB]
    auto stA = [&](int s) { return xsm + (size_t)s * XG_STAGE; };
    auto stB = [&](int s) { return xsm + (size_t)s * XG_STAGE + XG_ABYTES; };
    auto stT = [&](int s) { return reinterpret_cast<XTab *>(xsm + (size_t)s * XG_STAGE + XG_ABYTES + XG_BBYTES); };
    auto stS = [&](int s) {
        return reinterpret_cast<uint32_t *>(xsm + (size_t)s * XG_STAGE + XG_ABYTES + XG_BBYTES + XG_TBYTES);
    };
    uint64_t *full = reinterpret_cast<uint64_t *>(xsm + (size_t)XG_NS * XG_STAGE);
    uint64_t *empty = full + XG_NS;
    uint64_t *accf = empty + XG_NS;   // [2] a TMEM buffer holds a finished group
    uint64_t *acce = accf + 2;        // [2] the epilogue has read a TMEM buffer
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);
    double *xch = reinterpret_cast<double *>(xsm + (size_t)XG_NS * XG_STAGE + 256);   // SwiGLU exchange
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ng = cols / 64, nkb = cols / XG_BK;
    const int row0 = blockIdx.x * XG_BM, tok0 = blockIdx.y * XG_TOK;
    if (tid == 0) {
        for (int s = 0; s < XG_NS; s++) {
            mbar_init(&full[s], 1 + 64);
            mbar_init(&empty[s], 1 + 16);   // the MMAs done and the 16 epilogue warps' reads of the stage
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 16);
        }
        s_fail = 0;
        fence_mbar_init();
    }
    if (warp == 3) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t tmap = reinterpret_cast<uint64_t>(&tmd);
            for (int kb = 0; kb < nkb; kb++) {
                const int s = kb % XG_NS, u = kb / XG_NS;
                if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                mbar_expect_tx(&full[s], XG_BBYTES + XG_TBYTES);
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(stB(s))), "l"(tmap), "r"(kb * XG_BK), "r"(blockIdx.y * XG_BN), "r"(smem_u32(&full[s]))
                    : "memory");
                for (int h = 0; h < 2; h++)
                    bulk_g2s(stT(s) + h * XG_TOK, tab + (size_t)(2 * kb + h) * S_pad + tok0, XG_TOK * 16, &full[s]);
            }
        }
    } else if (warp == 1 || warp == 2) {
        // thread i of 64: rows i and i + 64 of the tile; the global loads of
        // stage kb + 2 are issued while stage kb is written (two register sets)
        const int i = tid - 32;
        uint4 wv0[2][4], wv1[2][4];
        uint32_t sb0[2][2], sb1[2][2];
        auto fetch = [&](int kb, uint4 (&wv)[2][4], uint32_t (&sb)[2][2]) {
            if (kb >= nkb) return;
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int r = row0 + i + 64 * rr;
                const uint4 *src = reinterpret_cast<const uint4 *>(w + (size_t)r * (cols / 8) + (size_t)kb * 16);
#pragma unroll
                for (int q = 0; q < 4; q++) wv[rr][q] = ldg_nc_v4(src + q);
                const size_t gi = (size_t)r * ng + 2 * kb;
                const uint32_t s2 = *reinterpret_cast<const uint32_t *>(sg + gi);   // groups 2kb, 2kb+1
                const uint32_t b2 = *reinterpret_cast<const uint32_t *>(bg + gi);
                sb[rr][0] = (s2 & 0xffffu) | (b2 << 16);
                sb[rr][1] = (s2 >> 16) | (b2 & 0xffff0000u);
            }
        };
        // stage kb from one register set, then that set refilled with kb + 2
        auto put = [&](int kb, uint4 (&wv)[2][4], uint32_t (&sb)[2][2]) -> bool {
            const int s = kb % XG_NS, u = kb / XG_NS;
            if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1)) {
                s_fail = 1;
                return false;
            }
            unsigned char *A = stA(s);
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int r = i + 64 * rr;
                unsigned char *rowp = A + (r >> 3) * 1024 + (r & 7) * 128;
                const uint32_t wd[16] = {wv[rr][0].x, wv[rr][0].y, wv[rr][0].z, wv[rr][0].w,
                                         wv[rr][1].x, wv[rr][1].y, wv[rr][1].z, wv[rr][1].w,
                                         wv[rr][2].x, wv[rr][2].y, wv[rr][2].z, wv[rr][2].w,
                                         wv[rr][3].x, wv[rr][3].y, wv[rr][3].z, wv[rr][3].w};
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const uint2 e0 = widen_nibbles(wd[2 * c]), e1 = widen_nibbles(wd[2 * c + 1]);
                    *reinterpret_cast<uint4 *>(rowp + ((c ^ (r & 7)) << 4)) = make_uint4(e0.x, e0.y, e1.x, e1.y);
                }
#pragma unroll
                for (int h = 0; h < 2; h++) stS(s)[h * XG_BM + r] = sb[rr][h];
            }
            fence_proxy_async();
            mbar_arrive(&full[s]);
            fetch(kb + 2, wv, sb);
            return true;
        };
        fetch(0, wv0, sb0);
        fetch(1, wv1, sb1);
        for (int kb = 0; kb < nkb; kb += 2) {
            if (!put(kb, wv0, sb0)) break;
            if (kb + 1 < nkb && !put(kb + 1, wv1, sb1)) break;
        }
    } else if (warp == 3) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_u8s8(XG_BM, XG_BN);
            for (int g = 0; g < ng; g++) {
                const int kb = g >> 1, s = kb % XG_NS, u = kb / XG_NS, b = g & 1, ub = g >> 1;
                if ((g & 1) == 0 && !mbar_wait(&full[s], u & 1)) {
                    s_fail = 1;
                    break;
                }
                if (ub > 0 && !mbar_wait(&acce[b], (ub - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(stA(s)) + (g & 1) * 64, b0 = smem_u32(stB(s)) + (g & 1) * 64;
                const uint32_t dt = tmem + (uint32_t)(b * 256);
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const uint64_t ad = umma_desc_sw128(a0 + k * 32), bd = umma_desc_sw128(b0 + k * 32);
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(dt),
                        "l"(ad), "l"(bd), "r"(idesc), "r"(k)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&accf[b]))
                             : "memory");
                if ((g & 1) == 1 || g == ng - 1)
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                     smem_u32(&empty[s]))
                                 : "memory");
            }
        }
    } else {
        // epilogue warps 4-19: rows 32 (warp % 4) .. + 31, tokens 16 tq .. + 15
        const int q = warp & 3, tq = (warp - 4) >> 2;
        const int trow = q * 32 + lane;
        double acc[16];
#pragma unroll
        for (int t = 0; t < 16; t++) acc[t] = 0.0;
        bool ok = true;
        for (int g = 0; g < ng; g++) {
            const int kb = g >> 1, s = kb % XG_NS, b = g & 1, ub = g >> 1;
            if (!mbar_wait(&accf[b], ub & 1)) {
                s_fail = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sbw = stS(s)[(g & 1) * XG_BM + trow];
            const double sc = (double)lo_bf(sbw), bi = (double)hi_bf(sbw);
            const XTab *tb = stT(s) + (g & 1) * XG_TOK + tq * 16;
            const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 256 + tq * 48);
#pragma unroll
            for (int tp = 0; tp < 2; tp++) {
                // 8 tokens (24 columns) per TMEM round trip
                uint32_t v[24];
                {
                    uint32_t a16[16], a8[8];
                    tmem_ld16(a16, ta + tp * 24);
                    tmem_ld8(a8, ta + tp * 24 + 16);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int k = 0; k < 16; k++) v[k] = a16[k];
#pragma unroll
                    for (int k = 0; k < 8; k++) v[16 + k] = a8[k];
                }
                if (tp == 1) {
                    // the buffer is read: the MMA warp may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acce[b]);
                }
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const int t = tp * 8 + k;
                    const int P = (int)v[3 * k] + ((int)v[3 * k + 1] << 7) + ((int)v[3 * k + 2] << 14);
                    const XTab e = tb[t];
                    acc[t] = fma(sc, int_times_pow2_hi(P, e.hi), acc[t]);
                    acc[t] = fma(bi, e.tf, acc[t]);
                }
            }
            // the stage's tables and scales are read: after its last group,
            // each epilogue warp releases it (with the MMA warp's commit)
            if ((g & 1) == 1 || g == ng - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }
        if (ok) {
            const int row = row0 + trow;
            if constexpr (EPI == EPI_SWIGLU) {
                // rows 0-63 of the tile are gate rows, 64-127 the up rows of
                // the same 64 outputs (alternating 64-row blocks)
                if (q >= 2) {
#pragma unroll
                    for (int t = 0; t < 16; t++) xch[(size_t)(tq * 16 + t) * 64 + (trow - 64)] = acc[t];
                }
                asm volatile("bar.sync 1, 512;" ::: "memory");
                if (q < 2) {
                    const int pairs = rows / 2, pr = (row0 / 128) * 64 + trow;
#pragma unroll
                    for (int t = 0; t < 16; t++) {
                        const int tok = tok0 + tq * 16 + t;
                        if (tok < S) {
                            const double up = xch[(size_t)(tq * 16 + t) * 64 + trow];
                            y[(size_t)tok * pairs + pr] = f2bf(swiglu_bf16(bf2f(d2bf(acc[t])), bf2f(d2bf(up))));
                        }
                    }
                }
            } else {
#pragma unroll
                for (int t = 0; t < 16; t++) {
                    const int tok = tok0 + tq * 16 + t;
                    if (tok >= S) continue;
                    const size_t o = (size_t)tok * rows + row;
                    if constexpr (EPI == EPI_RESIDUAL) y[o] = f2bf(__fadd_rn(bf2f(residual[o]), bf2f(d2bf(acc[t]))));
                    else if constexpr (EPI == EPI_PARTIAL) yf[o] = acc[t];
                    else y[o] = d2bf(acc[t]);
                }
            }
        } else if (EPI == EPI_SWIGLU) {
            asm volatile("bar.sync 1, 512;" ::: "memory");
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 3) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
    if (tid == 0 && s_fail) atomicExch(&g_xgemm_err, 1);
}

// ------------------------------------------------------------------ host

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return (EncodeTiledFn)p;
    }();
    return fn;
}

// digits [S_pad * 3][cols] int8 as a 2-D tensor map: box 128 columns x 192 rows, 128B swizzle
static int make_digit_map(CUtensorMap *m, const int8_t *xd, int S_pad, int cols) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("prefill GEMM: cuTensorMapEncodeTiled unavailable");
        return -1;
    }
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)S_pad * 3};
    cuuint64_t strides[1] = {(cuuint64_t)cols};
    cuuint32_t box[2] = {(cuuint32_t)XG_BK, (cuuint32_t)XG_BN};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(xd), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("prefill GEMM: tensor map encode failed (%d)", (int)r);
        return -1;
    }
    return 0;
}

bool qgemm_tc_eligible(const QMat &W, int S, int epi) {
    (void)epi;
    return S >= 2 && W.quant && W.group == 64 && W.sdtype == MLXD_BF16 && W.w && W.rows % XG_BM == 0 &&
           W.cols % XG_BK == 0;
}

size_t qgemm_tc_ws_bytes(int S, int cols) {
    const size_t S_pad = ((size_t)S + XG_TOK - 1) / XG_TOK * XG_TOK;
    return ((S_pad * 3 * cols + 255) / 256) * 256 + S_pad * (cols / 64) * sizeof(XTab) + 256;
}

template <int EPI>
static int launch_x(const QMat &W, const CUtensorMap &m, const XTab *tab, int S, int S_pad, uint16_t *y,
                    const uint16_t *res, double *yf, cudaStream_t st) {
    auto kern = qgemm_x_kernel<EPI>;
    if (!smem_allowed((const void *)kern, XG_SMEM)) return -1;
    dim3 grid(W.rows / XG_BM, S_pad / XG_TOK);
    kern<<<grid, XG_THREADS, XG_SMEM, st>>>(m, W.w, (const uint16_t *)W.s, (const uint16_t *)W.b, tab, W.rows, W.cols, S,
                                            S_pad, y, res, yf);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

int qgemm_tc(const QMat &W, const uint16_t *x, int S, int epi, const uint16_t *res, uint16_t *y, double *yf, void *ws,
             size_t ws_bytes, cudaStream_t st) {
    if (!qgemm_tc_eligible(W, S, epi)) {
        set_error("prefill GEMM: matrix not eligible");
        return -1;
    }
    if (ws_bytes < qgemm_tc_ws_bytes(S, W.cols) || ((uintptr_t)ws & 255) || ((uintptr_t)x & 3)) {
        set_error("prefill GEMM: workspace too small or misaligned");
        return -1;
    }
    const int S_pad = (S + XG_TOK - 1) / XG_TOK * XG_TOK;
    int8_t *xd = (int8_t *)ws;
    XTab *tab = reinterpret_cast<XTab *>((unsigned char *)ws + (((size_t)S_pad * 3 * W.cols + 255) / 256) * 256);
    const int ng = W.cols / 64;
    const size_t warps = (size_t)ng * S_pad;
    xq_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(x, S, S_pad, W.cols, xd, tab);
    MLXD_CHECK(cudaGetLastError());
    CUtensorMap m;
    if (make_digit_map(&m, xd, S_pad, W.cols)) return -1;
    switch (epi) {
    case EPI_STORE: return launch_x<EPI_STORE>(W, m, tab, S, S_pad, y, res, yf, st);
    case EPI_RESIDUAL: return launch_x<EPI_RESIDUAL>(W, m, tab, S, S_pad, y, res, yf, st);
    case EPI_SWIGLU: return launch_x<EPI_SWIGLU>(W, m, tab, S, S_pad, y, res, yf, st);
    case EPI_PARTIAL: return launch_x<EPI_PARTIAL>(W, m, tab, S, S_pad, y, res, yf, st);
    }
    set_error("prefill GEMM: bad epilogue");
    return -1;
}

// nonzero once a launch gave up on a wait (read and cleared)
int qgemm_tc_timeouts() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_xgemm_err, sizeof v) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_xgemm_err, &z, sizeof z);
    return v;
}

}  // namespace mlxd
