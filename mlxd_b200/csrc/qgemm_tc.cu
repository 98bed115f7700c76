// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// y[S][rows] = x[S][cols] . deq(W)^T for a chunk of prompt tokens
// (mlx_quantized_matmul at S > 1, src/engine/forward.c:17-32), W 4-bit with
// group 64 and bf16 scales/biases. mlx's qmm dequantizes a weight tile to the
// compute type, bf16(scale*q + bias) (one rounding, bf16 fma), and multiplies
// it with bf16 x accumulating in f32; this kernel does the same with the
// dequantized tile in shared memory and the accumulator in tensor memory.
//
// CTA tile: 128 weight rows (M) x 256 tokens (N), K in steps of one group
// (64 columns), TC_NS-deep pipeline of shared-memory stages:
//   warp 0, one lane   TMA: the x tile [256 tokens][64] bf16, 128-byte
//                      swizzle (K-major canonical layout), into stage s;
//   warps 2-5          dequantize the 128 x 64 weight tile of the stage from
//                      the integer-MMA tile layout (ti8) and the scale/bias
//                      records (sb) into the same K-major 128B-swizzled form,
//                      then fence.proxy.async and arrive;
//   warp 1, one lane   tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16,
//                      bf16 x bf16 -> f32 in TMEM) x 4 per stage, then
//                      tcgen05.commit releases the stage; after the last
//                      stage a commit signals the epilogue;
//   warps 2-5          tcgen05.ld the 128 x 256 f32 accumulator (each warp
//                      its 32 TMEM lanes = 32 rows) and apply the epilogue
//                      (store / +residual / SwiGLU / f32 partial).
// Every mbarrier wait gives up after 0.5 s and sets an error word the host
// reads; TMEM is released on every path.
#include <cuda.h>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"

namespace mlxd {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64, TC_NS = 4, TC_GTHREADS = 192;
constexpr int TC_ABYTES = TC_BM * TC_BK * 2;   // 16 KB
constexpr int TC_BBYTES = TC_BN * TC_BK * 2;   // 32 KB
constexpr size_t TC_SMEM = 1024 + (size_t)TC_NS * (TC_ABYTES + TC_BBYTES) + 256;

static __device__ int g_tcgemm_err;

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
// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

MLXD_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MLXD_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MLXD_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// the weight tile of stage kb: record rec (0..255) = lane L of row block
// rb_local of this CTA; 8 words of bf16 pairs per row go to the swizzled rows
MLXD_DEV void deq_store_record(unsigned char *A, int rb_local, int L, uint4 w, uint2 sbv) {
    const int gq = L >> 2, t = L & 3;
    const uint32_t sA2 = (sbv.x & 0xffffu) * 0x10001u, bA2 = (sbv.x >> 16) * 0x10001u;
    const uint32_t sB2 = (sbv.y & 0xffffu) * 0x10001u, bB2 = (sbv.y >> 16) * 0x10001u;
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = rb_local * 16 + gq + 8 * (i & 1);
        const uint32_t s2 = (i & 1) ? sB2 : sA2, b2 = (i & 1) ? bB2 : bA2;
        const int kb0 = 16 * (i >> 1) + 4 * t;   // low nibbles: k = kb0..kb0+3, high: +32
        // bytes (j, j+1) into the two halves, then the nibbles into 128.0's mantissa
        const uint32_t p01 = __byte_perm(wv[i], 0u, 0x4140), p23 = __byte_perm(wv[i], 0u, 0x4342);
        uint32_t q[4];
        q[0] = (p01 & 0x000F000Fu) | 0x43004300u;          // k0, k0+1
        q[1] = (p23 & 0x000F000Fu) | 0x43004300u;          // k0+2, k0+3
        q[2] = ((p01 >> 4) & 0x000F000Fu) | 0x43004300u;   // k0+32, +33
        q[3] = ((p23 >> 4) & 0x000F000Fu) | 0x43004300u;   // k0+34, +35
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            __nv_bfloat162 qq = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&q[e]),
                                        __floats2bfloat162_rn(128.f, 128.f));
            __nv_bfloat162 r = __hfma2(*reinterpret_cast<const __nv_bfloat162 *>(&s2), qq,
                                       *reinterpret_cast<const __nv_bfloat162 *>(&b2));
            o[e] = *reinterpret_cast<uint32_t *>(&r);
        }
        unsigned char *rowp = A + (row >> 3) * 1024 + (row & 7) * 128;
        const int sw = row & 7;
        // k0..k0+3: chunk k0/8, byte (k0 % 8) * 2; k0 + 32: chunk + 4
        const int c0 = kb0 >> 3, off = (kb0 & 7) * 2;
        *reinterpret_cast<uint2 *>(rowp + ((c0 ^ sw) << 4) + off) = make_uint2(o[0], o[1]);
        *reinterpret_cast<uint2 *>(rowp + (((c0 + 4) ^ sw) << 4) + off) = make_uint2(o[2], o[3]);
    }
}

template <int EPI>
__global__ void __launch_bounds__(TC_GTHREADS, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmx, const uint8_t *__restrict__ ti8,
                    const uint8_t *__restrict__ sb, int rows, int cols, int S, uint16_t *__restrict__ y,
                    const uint16_t *__restrict__ residual, float *__restrict__ yf) {
    extern __shared__ __align__(1024) unsigned char tsm_raw[];
    unsigned char *tsm = reinterpret_cast<unsigned char *>(((uintptr_t)tsm_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *Abuf = tsm;
    unsigned char *Bbuf = tsm + (size_t)TC_NS * TC_ABYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(Bbuf + (size_t)TC_NS * TC_BBYTES);
    uint64_t *empty = full + TC_NS;
    uint64_t *accf = empty + TC_NS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nk = cols / TC_BK, ng = cols / 64;
    const int n0 = blockIdx.y * TC_BN;
    if (tid == 0) {
        for (int s = 0; s < TC_NS; s++) {
            mbar_init(&full[s], 1 + 128);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        s_fail = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // x tiles by TMA
            const uint64_t tmap = reinterpret_cast<uint64_t>(&tmx);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % TC_NS, u = kb / TC_NS;
                if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                mbar_expect_tx(&full[s], TC_BBYTES);
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(Bbuf + (size_t)s * TC_BBYTES)), "l"(tmap), "r"(kb * TC_BK), "r"(n0),
                      "r"(smem_u32(&full[s]))
                    : "memory");
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(TC_BM, TC_BN);
            for (int kb = 0; kb < nk; kb++) {
                const int s = kb % TC_NS, u = kb / TC_NS;
                if (!mbar_wait(&full[s], u & 1)) {
                    s_fail = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(Abuf + (size_t)s * TC_ABYTES), b0 = smem_u32(Bbuf + (size_t)s * TC_BBYTES);
#pragma unroll
                for (int k = 0; k < TC_BK / 16; k++) {
                    const uint64_t ad = umma_desc_sw128(a0 + k * 32), bd = umma_desc_sw128(b0 + k * 32);
                    const uint32_t acc = (kb | k) != 0;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem),
                        "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(0u)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&empty[s]))
                             : "memory");
            }
            // the accumulator is complete once every issued MMA is
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(accf))
                         : "memory");
        }
    } else {
        // dequantize: thread i of 128 takes records i and i + 128 of the
        // stage (record = lane L of row block rb_local)
        const int i = tid - 64;
        const int rbA = i >> 5, rbB = (i + 128) >> 5, L = i & 31, gq = L >> 2;
        const int rb0 = blockIdx.x * (TC_BM / 16);
        auto ldrec = [&](int rbl, int g, uint4 &w, uint2 &sv) {
            const size_t tile = (size_t)(rb0 + rbl) * ng + g;
            w = ldg_nc_v4(ti8 + (tile * 32 + L) * 16);
            sv = ldg_nc_v2(sb + (tile * 8 + gq) * 8);
        };
        // the records of the next TC_NS stages in registers (loop unrolled by
        // TC_NS so that the ring index is a constant)
        uint4 wA[TC_NS], wB[TC_NS];
        uint2 sA[TC_NS], sB[TC_NS];
#pragma unroll
        for (int j = 0; j < TC_NS; j++)
            if (j < nk) {
                ldrec(rbA, j, wA[j], sA[j]);
                ldrec(rbB, j, wB[j], sB[j]);
            }
        bool failed = false;
        for (int kb0 = 0; kb0 < nk && !failed; kb0 += TC_NS) {
#pragma unroll
            for (int j = 0; j < TC_NS; j++) {
                const int kb = kb0 + j;
                if (kb >= nk || failed) break;
                const int u = kb / TC_NS;   // stage j, use u
                const uint4 cA = wA[j], cB = wB[j];
                const uint2 dA = sA[j], dB = sB[j];
                if (kb + TC_NS < nk) {
                    ldrec(rbA, kb + TC_NS, wA[j], sA[j]);
                    ldrec(rbB, kb + TC_NS, wB[j], sB[j]);
                }
                if (u > 0 && !mbar_wait(&empty[j], (u - 1) & 1)) {
                    s_fail = 1;
                    failed = true;
                    break;
                }
                unsigned char *A = Abuf + (size_t)j * TC_ABYTES;
                deq_store_record(A, rbA, L, cA, dA);
                deq_store_record(A, rbB, L, cB, dB);
                fence_proxy_async();
                mbar_arrive(&full[j]);
            }
        }
        // epilogue: warp w reads TMEM lanes 32*(w%4).. (rows of the tile)
        const bool ok = mbar_wait(accf, 0);
        if (!ok) s_fail = 1;
        tc_fence_after();
        const int q = warp & 3;
        const int trow = q * 32 + lane;                 // row within the tile
        const int row = blockIdx.x * TC_BM + trow;
        if (ok) {
            for (int c0 = 0; c0 < TC_BN; c0 += 32) {
                uint32_t v[32];
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                      "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                      "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
                      "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
                      "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int tok = n0 + c0 + j;
                    const float acc = __uint_as_float(v[j]);
                    if constexpr (EPI == EPI_SWIGLU) {
                        // rows 16p..16p+15 gate, 16p+16.. up of the same pair
                        const float up = __shfl_down_sync(0xffffffffu, acc, 16);
                        if ((lane & 16) == 0 && tok < S) {
                            const int pair = (blockIdx.x * TC_BM + q * 32) / 32;
                            y[(size_t)tok * (rows / 2) + pair * 16 + (lane & 15)] =
                                f2bf(swiglu_bf16(rbf(acc), rbf(up)));
                        }
                    } else if (tok < S) {
                        const size_t o = (size_t)tok * rows + row;
                        if constexpr (EPI == EPI_RESIDUAL) y[o] = f2bf(__fadd_rn(bf2f(residual[o]), rbf(acc)));
                        else if constexpr (EPI == EPI_PARTIAL_F32) yf[o] = acc;
                        else y[o] = f2bf(acc);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_BN));
    }
    if (tid == 0 && s_fail) atomicExch(&g_tcgemm_err, 1);
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

// x [S][cols] bf16 as a 2-D tensor map: box 64 columns x 256 tokens, 128B swizzle
static int make_x_map(CUtensorMap *m, const uint16_t *x, int S, int cols) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("qgemm_tc: cuTensorMapEncodeTiled unavailable");
        return -1;
    }
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)S};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BN};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("qgemm_tc: tensor map encode failed (%d)", (int)r);
        return -1;
    }
    return 0;
}

template <int EPI>
static int launch_tc(const QMat &W, const CUtensorMap &m, int S, uint16_t *y, const uint16_t *res, float *yf,
                     cudaStream_t st) {
    auto kern = qgemm_tc_kernel<EPI>;
    static bool configured = false;
    if (!configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
        configured = true;
    }
    dim3 grid(W.rows / TC_BM, (S + TC_BN - 1) / TC_BN);
    kern<<<grid, TC_GTHREADS, TC_SMEM, st>>>(m, W.ti8, W.sb, W.rows, W.cols, S, y, res, yf);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

bool qgemm_tc_eligible(const QMat &W, int S) {
    static const bool on = [] {
        const char *e = getenv("MLXD_GEMM_TC");
        return !e || atoi(e) != 0;
    }();
    return on && S >= 2 && W.quant && W.fast8() && W.ti8 && W.sb && W.rows % TC_BM == 0 && W.cols % TC_BK == 0;
}

int qgemm_tc(const QMat &W, const uint16_t *x, int S, uint16_t *y, int epi, const uint16_t *res, float *yf,
             cudaStream_t st) {
    if (((uintptr_t)x & 15) || (W.cols * 2) % 16) {
        set_error("qgemm_tc: x must be 16-byte aligned");
        return -1;
    }
    CUtensorMap m;
    if (make_x_map(&m, x, S, W.cols)) return -1;
    switch (epi) {
    case EPI_STORE: return launch_tc<EPI_STORE>(W, m, S, y, res, yf, st);
    case EPI_RESIDUAL: return launch_tc<EPI_RESIDUAL>(W, m, S, y, res, yf, st);
    case EPI_SWIGLU: return launch_tc<EPI_SWIGLU>(W, m, S, y, res, yf, st);
    case EPI_PARTIAL_F32: return launch_tc<EPI_PARTIAL_F32>(W, m, S, y, res, yf, st);
    }
    set_error("qgemm_tc: bad epilogue");
    return -1;
}

// nonzero once a launch gave up on a wait (read and cleared)
int qgemm_tc_timeouts() {
    int v = 0, z = 0;
    if (cudaMemcpyFromSymbol(&v, g_tcgemm_err, sizeof v) != cudaSuccess) return -1;
    if (v) cudaMemcpyToSymbol(g_tcgemm_err, &z, sizeof z);
    return v;
}

}  // namespace mlxd
