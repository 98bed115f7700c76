// Prefill projections (S > 1 tokens) and dense bf16 projections.
//
// qgemm: y[S][rows] = x[S][cols] . deq(W)^T for a chunk of prompt tokens
// (mlx_quantized_matmul at S > 1, forward.c:17-32). Weights stay in the
// decode tile layout; each warp owns a 16-row block and builds its A
// fragments in registers, dequantising with one fused multiply-add per pair
// (bf16(scale*q + bias), the mlx qmm tile semantics); the token tile of x is
// staged in shared memory by cp.async and read with ldmatrix. 8 warps = 128
// rows x 64 tokens per CTA, f32 accumulation across all groups.
//
// dense_linear: bf16 weights (unquantized checkpoints, forward.c:33-44),
// one thread per output with the same fixed 8-way association as the oracle.
#include "common.cuh"
#include "kernels.h"

namespace mlxd {

constexpr int GM_TOK = 64;     // tokens per CTA
constexpr int GM_WARPS = 8;

MLXD_DEV uint32_t deq_pair_bf16(uint32_t nib, uint32_t s2, uint32_t b2) {
    // nib holds bf16 (128+q_lo, 128+q_hi); subtract 128 exactly, then s*q+b
    __nv_bfloat162 q = __hsub2(*reinterpret_cast<__nv_bfloat162 *>(&nib),
                               __floats2bfloat162_rn(128.f, 128.f));
    __nv_bfloat162 r = __hfma2(*reinterpret_cast<__nv_bfloat162 *>(&s2), q,
                               *reinterpret_cast<__nv_bfloat162 *>(&b2));
    return *reinterpret_cast<uint32_t *>(&r);
}
MLXD_DEV uint32_t deq_pair_f32(uint32_t nib, float s, float b) {
    float qlo = lo_bf(nib) - 128.f, qhi = hi_bf(nib) - 128.f;
    return pack_bf2(__fmaf_rn(s, qlo, b), __fmaf_rn(s, qhi, b));
}

template <int G, bool SBF32, int EPI>
__global__ void __launch_bounds__(GM_WARPS * 32) qgemm_kernel(
    const uint8_t *__restrict__ tiles, const uint8_t *__restrict__ sb, int rows, int cols,
    const uint16_t *__restrict__ x, int S, uint16_t *__restrict__ y,
    const uint16_t *__restrict__ residual, float *__restrict__ yf) {
    constexpr int LD = G + 8;
    constexpr int KJ = G / 16;
    __shared__ __align__(16) uint16_t sx[2][GM_TOK * LD];
    __shared__ uint16_t sred[EPI == EPI_SWIGLU ? GM_WARPS * 16 * GM_TOK : 1];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int ng = cols / G, nrb = rows / 16;
    const int rb = blockIdx.x * GM_WARPS + warp;
    const bool active = rb < nrb;
    const int n0 = blockIdx.y * GM_TOK;
    const int ntok = min(GM_TOK, S - n0);

    auto load_x = [&](int gi, int buf) {
        constexpr int CH = G / 8;   // 16-byte chunks per token row
        for (int c = tid; c < GM_TOK * CH; c += GM_WARPS * 32) {
            int r = c / CH, cc = c % CH;
            bool ok = r < ntok;
            const uint16_t *src = x + (size_t)(n0 + (ok ? r : 0)) * cols + gi * G + cc * 8;
            cp_async16_zfill(&sx[buf][r * LD + cc * 8], src, ok);
        }
        cp_async_commit();
    };

    float acc[GM_TOK / 8][4];
#pragma unroll
    for (int n = 0; n < GM_TOK / 8; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

    using WT = typename std::conditional<G == 64, uint4, uint2>::type;
    using ST = typename std::conditional<SBF32, uint4, uint2>::type;
    auto ldw = [&](int gi) -> WT {
        size_t tile = (size_t)rb * ng + gi;
        if constexpr (G == 64) return ldg_nc_v4(tiles + (tile * 32 + lane) * 16);
        else return ldg_nc_v2(tiles + (tile * 32 + lane) * 8);
    };
    auto lds = [&](int gi) -> ST {
        size_t tile = (size_t)rb * ng + gi;
        if constexpr (SBF32) return ldg_nc_v4(sb + (tile * 8 + g) * 16);
        else return ldg_nc_v2(sb + (tile * 8 + g) * 8);
    };

    WT wv{};
    ST sv{};
    if (active) {
        wv = ldw(0);
        sv = lds(0);
    }
    load_x(0, 0);
    for (int gi = 0; gi < ng; gi++) {
        int buf = gi & 1;
        if (gi + 1 < ng) {
            load_x(gi + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        WT wc = wv;
        ST sc = sv;
        if (active && gi + 1 < ng) {
            wv = ldw(gi + 1);
            sv = lds(gi + 1);
        }
        if (active) {
            // dequantised A fragments for the KJ k16 steps of this group
            uint32_t af[KJ][4];
            if constexpr (SBF32) {
                float sA = __uint_as_float(sc.x), bA = __uint_as_float(sc.y);
                float sB = __uint_as_float(sc.z), bB = __uint_as_float(sc.w);
                if constexpr (G == 64) {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        af[j][0] = deq_pair_f32(nib_pair(wc.x, j), sA, bA);
                        af[j][1] = deq_pair_f32(nib_pair(wc.z, j), sB, bB);
                        af[j][2] = deq_pair_f32(nib_pair(wc.y, j), sA, bA);
                        af[j][3] = deq_pair_f32(nib_pair(wc.w, j), sB, bB);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        af[j][0] = deq_pair_f32(nib_pair(wc.x, 2 * j), sA, bA);
                        af[j][1] = deq_pair_f32(nib_pair(wc.y, 2 * j), sB, bB);
                        af[j][2] = deq_pair_f32(nib_pair(wc.x, 2 * j + 1), sA, bA);
                        af[j][3] = deq_pair_f32(nib_pair(wc.y, 2 * j + 1), sB, bB);
                    }
                }
            } else {
                uint32_t sA2 = (sc.x & 0xffffu) * 0x10001u, bA2 = (sc.x >> 16) * 0x10001u;
                uint32_t sB2 = (sc.y & 0xffffu) * 0x10001u, bB2 = (sc.y >> 16) * 0x10001u;
                if constexpr (G == 64) {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        af[j][0] = deq_pair_bf16(nib_pair(wc.x, j), sA2, bA2);
                        af[j][1] = deq_pair_bf16(nib_pair(wc.z, j), sB2, bB2);
                        af[j][2] = deq_pair_bf16(nib_pair(wc.y, j), sA2, bA2);
                        af[j][3] = deq_pair_bf16(nib_pair(wc.w, j), sB2, bB2);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        af[j][0] = deq_pair_bf16(nib_pair(wc.x, 2 * j), sA2, bA2);
                        af[j][1] = deq_pair_bf16(nib_pair(wc.y, 2 * j), sB2, bB2);
                        af[j][2] = deq_pair_bf16(nib_pair(wc.x, 2 * j + 1), sA2, bA2);
                        af[j][3] = deq_pair_bf16(nib_pair(wc.y, 2 * j + 1), sB2, bB2);
                    }
                }
            }
            const uint16_t *xs = sx[buf];
#pragma unroll
            for (int j = 0; j < KJ; j++) {
#pragma unroll
                for (int n = 0; n < GM_TOK / 8; n += 2) {
                    uint32_t b[4];
                    int r = n * 8 + (lane & 7) + ((lane >> 4) << 3);
                    int c = j * 16 + ((lane >> 3) & 1) * 8;
                    ldmatrix_x4(b, xs + r * LD + c);
                    mma_bf16_16816(acc[n], af[j], b[0], b[1]);
                    mma_bf16_16816(acc[n + 1], af[j], b[2], b[3]);
                }
            }
        }
        __syncthreads();
    }

    // epilogue. acc[n][0..1]: row g, tokens 8n+2t(+1); acc[n][2..3]: row g+8
    if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
        for (int n = 0; n < GM_TOK / 8; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                int r = g + (e >= 2 ? 8 : 0), tok = n * 8 + 2 * t + (e & 1);
                sred[(warp * 16 + r) * GM_TOK + tok] = f2bf(acc[n][e]);
            }
        __syncthreads();
        // warp pairs (2i gate, 2i+1 up) -> 16 activations per token
        for (int idx = tid; idx < (GM_WARPS / 2) * 16 * GM_TOK; idx += GM_WARPS * 32) {
            int pr = idx / (16 * GM_TOK), rem = idx % (16 * GM_TOK);
            int r = rem / GM_TOK, tok = rem % GM_TOK;
            int rbg = blockIdx.x * GM_WARPS + 2 * pr;
            if (rbg >= nrb || tok >= ntok) continue;
            float gv = bf2f(sred[((2 * pr) * 16 + r) * GM_TOK + tok]);
            float uv = bf2f(sred[((2 * pr + 1) * 16 + r) * GM_TOK + tok]);
            int out_row = (rbg / 2) * 16 + r;
            y[(size_t)(n0 + tok) * (rows / 2) + out_row] = f2bf(swiglu_bf16(gv, uv));
        }
        return;
    }
    if (!active) return;
#pragma unroll
    for (int n = 0; n < GM_TOK / 8; n++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            int r = rb * 16 + g + (e >= 2 ? 8 : 0);
            int tok = n * 8 + 2 * t + (e & 1);
            if (tok >= ntok) continue;
            size_t o = (size_t)(n0 + tok) * rows + r;
            if constexpr (EPI == EPI_RESIDUAL) y[o] = f2bf(__fadd_rn(bf2f(residual[o]), rbf(acc[n][e])));
            else if constexpr (EPI == EPI_PARTIAL_F32) yf[o] = acc[n][e];
            else y[o] = f2bf(acc[n][e]);
        }
}

// f32 dot product, fixed association: eight interleaved partial sums (lane
// i takes elements i, i+8, ...) combined pairwise; identical to the oracle.
MLXD_DEV float dot8(const uint16_t *a, const uint16_t *b, int n) {
    float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j + 8 <= n; j += 8)
#pragma unroll
        for (int t = 0; t < 8; t++) p[t] = __fadd_rn(p[t], __fmul_rn(bf2f(a[j + t]), bf2f(b[j + t])));
    for (int t = 0; j < n; j++, t++) p[t] = __fadd_rn(p[t], __fmul_rn(bf2f(a[j]), bf2f(b[j])));
    return __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[1]), __fadd_rn(p[2], p[3])),
                     __fadd_rn(__fadd_rn(p[4], p[5]), __fadd_rn(p[6], p[7])));
}

template <int EPI>
__global__ void dense_linear_kernel(const uint16_t *__restrict__ w, int rows, int cols,
                                    const uint16_t *__restrict__ x, int S, uint16_t *__restrict__ y,
                                    const uint16_t *__restrict__ residual, int gate_rows,
                                    float *__restrict__ yf) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    int out_rows = EPI == EPI_SWIGLU ? gate_rows : rows;
    if (idx >= (size_t)S * out_rows) return;
    int s = (int)(idx / out_rows), r = (int)(idx % out_rows);
    const uint16_t *xv = x + (size_t)s * cols;
    if constexpr (EPI == EPI_SWIGLU) {
        // dense gate/up stacked as [gate rows; up rows]
        float gv = rbf(dot8(xv, w + (size_t)r * cols, cols));
        float uv = rbf(dot8(xv, w + (size_t)(gate_rows + r) * cols, cols));
        y[(size_t)s * gate_rows + r] = f2bf(swiglu_bf16(gv, uv));
    } else {
        float a = dot8(xv, w + (size_t)r * cols, cols);
        size_t o = (size_t)s * rows + r;
        if constexpr (EPI == EPI_RESIDUAL) y[o] = f2bf(__fadd_rn(bf2f(residual[o]), rbf(a)));
        else if constexpr (EPI == EPI_PARTIAL_F32) yf[o] = a;
        else y[o] = f2bf(a);
    }
}

template <int G, bool F32, int EPI>
static int launch_qgemm(const QMat &W, const uint16_t *x, int S, uint16_t *y, const uint16_t *res,
                        float *yf, cudaStream_t st) {
    dim3 grid((W.rows / 16 + GM_WARPS - 1) / GM_WARPS, (S + GM_TOK - 1) / GM_TOK);
    qgemm_kernel<G, F32, EPI><<<grid, GM_WARPS * 32, 0, st>>>(W.tiles, W.sb, W.rows, W.cols, x, S, y, res, yf);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

template <int G, bool F32>
static int dispatch_qgemm(const QMat &W, const uint16_t *x, int S, uint16_t *y, int epi,
                          const uint16_t *res, float *yf, cudaStream_t st) {
    if (epi == EPI_STORE) return launch_qgemm<G, F32, EPI_STORE>(W, x, S, y, res, yf, st);
    if (epi == EPI_RESIDUAL) return launch_qgemm<G, F32, EPI_RESIDUAL>(W, x, S, y, res, yf, st);
    if (epi == EPI_SWIGLU) return launch_qgemm<G, F32, EPI_SWIGLU>(W, x, S, y, res, yf, st);
    if (epi == EPI_PARTIAL_F32) return launch_qgemm<G, F32, EPI_PARTIAL_F32>(W, x, S, y, res, yf, st);
    set_error("qgemm: bad epilogue");
    return -1;
}

int linear_multi(const QMat &W, const uint16_t *x, int S, uint16_t *y, int epi,
                 const uint16_t *residual, float *yf, cudaStream_t st) {
    if (S <= 0) return 0;
    if (!W.quant) {
        int out_rows = epi == EPI_SWIGLU ? W.rows / 2 : W.rows;
        size_t n = (size_t)S * out_rows;
        unsigned blocks = (unsigned)((n + 127) / 128);
        if (epi == EPI_STORE) dense_linear_kernel<EPI_STORE><<<blocks, 128, 0, st>>>(W.dense, W.rows, W.cols, x, S, y, residual, 0, yf);
        else if (epi == EPI_RESIDUAL) dense_linear_kernel<EPI_RESIDUAL><<<blocks, 128, 0, st>>>(W.dense, W.rows, W.cols, x, S, y, residual, 0, yf);
        else if (epi == EPI_PARTIAL_F32) dense_linear_kernel<EPI_PARTIAL_F32><<<blocks, 128, 0, st>>>(W.dense, W.rows, W.cols, x, S, y, residual, 0, yf);
        else dense_linear_kernel<EPI_SWIGLU><<<blocks, 128, 0, st>>>(W.dense, W.rows, W.cols, x, S, y, residual, W.rows / 2, yf);
        MLXD_CHECK(cudaGetLastError());
        return 0;
    }
    if (epi == EPI_SWIGLU && W.rows % 32) {
        set_error("qgemm: gate/up rows must pair 16-row blocks");
        return -1;
    }
    if (qgemm_tc_eligible(W, S)) return qgemm_tc(W, x, S, y, epi, residual, yf, st);
    bool f32 = W.sdtype == MLXD_F32;
    if (W.group == 64) return f32 ? dispatch_qgemm<64, true>(W, x, S, y, epi, residual, yf, st)
                                  : dispatch_qgemm<64, false>(W, x, S, y, epi, residual, yf, st);
    if (W.group == 32) return f32 ? dispatch_qgemm<32, true>(W, x, S, y, epi, residual, yf, st)
                                  : dispatch_qgemm<32, false>(W, x, S, y, epi, residual, yf, st);
    set_error("qgemm: group size %d not supported", W.group);
    return -1;
}

}  // namespace mlxd
