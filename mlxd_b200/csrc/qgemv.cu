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
#include "common.cuh"
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

MLXD_DEV unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)k << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

constexpr int GEMV_THREADS = 256;

template <int G, bool SBF32, int PRO, int EPI, int RB>
__global__ void __launch_bounds__(GEMV_THREADS, 2) qgemv_kernel(GemvArgs a) {
    constexpr int XW = G / 8;           // x words per (group, t)
    constexpr int P = (G == 64) ? 8 : 8; // prefetch depth (items)
    constexpr int WB = G / 4;           // tile bytes per lane
    constexpr int SBB = SBF32 ? 16 : 8; // sb bytes per record
    using WT = typename Ld<G, false>::W;
    using ST = typename std::conditional<SBF32, uint4, uint2>::type;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int ng = a.cols / G;
    uint32_t *xp = reinterpret_cast<uint32_t *>(smem_raw);
    float *xs = reinterpret_cast<float *>(xp + (size_t)ng * 4 * XW);
    float *red = xs + ng;                // [8][RB][16]
    __shared__ float s_red[8];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = lane & 3;
    const int rb0 = blockIdx.x * RB;
    const int g0 = (warp * ng) / 8, g1 = ((warp + 1) * ng) / 8;
    const int nper = g1 - g0;
    const int n_items = RB * nper;

    WT wbuf[P];
    ST sbuf[P];
#pragma unroll
    for (int p = 0; p < P; p++) {
        if (p < n_items) {
            int rb = p / nper, g = g0 + p % nper;
            size_t tile = (size_t)(rb0 + rb) * ng + g;
            wbuf[p] = load_w<G>(a.tiles + (tile * 32 + lane) * WB);
            sbuf[p] = load_sb<SBF32>(a.sb + (tile * 8 + (lane >> 2)) * SBB);
        }
    }

    // ---- prologue: x (optionally RMS-normalised) into the fragment order
    pdl_wait();
    const uint32_t *x2 = reinterpret_cast<const uint32_t *>(a.x);
    const int npairs = a.cols / 2;
    float inv = 1.0f;
    if (PRO == PRO_RMSNORM) {
        float acc = 0.f;
        for (int p = tid; p < npairs; p += GEMV_THREADS) {
            uint32_t v = x2[p];
            float lo = lo_bf(v), hi = hi_bf(v);
            acc = fmaf(lo, lo, acc);
            acc = fmaf(hi, hi, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) s_red[warp] = acc;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) tot += s_red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.cols), a.eps)));
    }
    const uint32_t *nw2 = reinterpret_cast<const uint32_t *>(a.norm_w);
    for (int p = tid; p < npairs; p += GEMV_THREADS) {
        uint32_t v = x2[p];
        if (PRO == PRO_RMSNORM) {
            uint32_t wv = nw2[p];
            float lo = rbf(__fmul_rn(lo_bf(wv), rbf(__fmul_rn(lo_bf(v), inv))));
            float hi = rbf(__fmul_rn(hi_bf(wv), rbf(__fmul_rn(hi_bf(v), inv))));
            v = pack_bf2(lo, hi);
        }
        int k = 2 * p;
        int gi = k / G, kk = k % G;
        int j = kk >> 4, w16 = kk & 15;
        int hi = w16 >= 8, tt = (w16 & 7) >> 1;
        xp[(gi * 4 + tt) * XW + j * 2 + hi] = v;
    }
    __syncthreads();
    for (int gi = warp; gi < ng; gi += 8) {
        float s = 0.f;
        if (lane < 4 * XW) {
            uint32_t v = xp[gi * 4 * XW + lane];
            s = lo_bf(v) + hi_bf(v);
        }
        s = warp_sum(s);
        if (lane == 0) xs[gi] = s;
    }
    __syncthreads();
    pdl_trigger();

    // ---- main loop over (row block, group) items of this warp
    float y0 = 0.f, y1 = 0.f;
    for (int base = 0; base < n_items; base += P) {
#pragma unroll
        for (int p = 0; p < P; p++) {
            int i = base + p;
            if (i < n_items) {
                int rb = i / nper, g = g0 + i % nper;
                WT wv = wbuf[p];
                ST sv = sbuf[p];
                int nx = i + P;
                if (nx < n_items) {
                    int nrb = nx / nper, ngg = g0 + nx % nper;
                    size_t tile = (size_t)(rb0 + nrb) * ng + ngg;
                    wbuf[p] = load_w<G>(a.tiles + (tile * 32 + lane) * WB);
                    sbuf[p] = load_sb<SBF32>(a.sb + (tile * 8 + (lane >> 2)) * SBB);
                }
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                const uint4 *xq = reinterpret_cast<const uint4 *>(xp + (g * 4 + t) * XW);
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
                float xsg = xs[g];
                y0 = fmaf(sA, d[0], y0);
                y0 = fmaf(fmaf(-128.f, sA, bA), xsg, y0);
                y1 = fmaf(sB, d[2], y1);
                y1 = fmaf(fmaf(-128.f, sB, bB), xsg, y1);
                if (i % nper == nper - 1) {
                    if (t == 0) {
                        red[(warp * RB + rb) * 16 + (lane >> 2)] = y0;
                        red[(warp * RB + rb) * 16 + (lane >> 2) + 8] = y1;
                    }
                    y0 = 0.f;
                    y1 = 0.f;
                }
            }
        }
    }
    if (nper == 0 && lane < 16)
        for (int rb = 0; rb < RB; rb++) red[(warp * RB + rb) * 16 + lane] = 0.f;
    __syncthreads();

    // ---- cross-warp reduction (fixed order) and epilogue
    if (tid < RB * 16) {
        int rb = tid >> 4, r = tid & 15;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) acc += red[(w * RB + rb) * 16 + r];
        int row = (rb0 + rb) * 16 + r;
        if constexpr (EPI == EPI_STORE) {
            a.y[row] = f2bf(acc);
        } else if constexpr (EPI == EPI_RESIDUAL) {
            a.y[row] = f2bf(__fadd_rn(bf2f(a.residual[row]), rbf(acc)));
        } else if constexpr (EPI == EPI_SWIGLU) {
            red[rb * 16 + r] = acc;  // warp 0 slots reused after the reduction
        } else if constexpr (EPI == EPI_PARTIAL_F32) {
            a.yf[row] = acc;
        } else {
            float v = rbf(acc);
            a.y[row] = f2bf(acc);
            unsigned long long key = argmax_key(v, a.row_offset + row);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                unsigned long long other = __shfl_xor_sync(0xffffu, key, o, 16);
                key = other > key ? other : key;
            }
            if (r == 0) atomicMax(a.amax, key);
        }
    }
    if constexpr (EPI == EPI_SWIGLU) {
        __syncthreads();
        if (tid < RB * 8) {
            int pair = tid >> 4, r = tid & 15;
            float g = rbf(red[(2 * pair) * 16 + r]);
            float u = rbf(red[(2 * pair + 1) * 16 + r]);
            a.y[(blockIdx.x * (RB / 2) + pair) * 16 + r] = f2bf(swiglu_bf16(g, u));
        }
    }
}

template <int G, bool SBF32, int PRO, int EPI>
static int launch_gemv(const GemvArgs &a, cudaStream_t st, bool pdl) {
    constexpr int RB = EPI == EPI_SWIGLU ? 2 : 1;
    auto kern = qgemv_kernel<G, SBF32, PRO, EPI, RB>;
    int ng = a.cols / G;
    size_t smem = (size_t)ng * 4 * (G / 8) * 4 + (size_t)ng * 4 + 8 * RB * 16 * 4;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        MLXD_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        configured = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.rows / 16 / RB);
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

template <int G, bool SBF32>
static int dispatch_gemv(int pro, int epi, const GemvArgs &a, cudaStream_t st, bool pdl) {
#define MLXD_GEMV_CASE(P, E) \
    if (pro == P && epi == E) return launch_gemv<G, SBF32, P, E>(a, st, pdl);
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_STORE)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_RESIDUAL)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_SWIGLU)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_ARGMAX)
    MLXD_GEMV_CASE(PRO_PLAIN, EPI_PARTIAL_F32)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_STORE)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_RESIDUAL)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_SWIGLU)
    MLXD_GEMV_CASE(PRO_RMSNORM, EPI_ARGMAX)
#undef MLXD_GEMV_CASE
    set_error("qgemv: bad prologue/epilogue");
    return -1;
}

int qgemv(const QMat &W, int pro, int epi, GemvArgs a, cudaStream_t st, bool pdl) {
    if (!W.quant) {
        set_error("qgemv: matrix is not quantized");
        return -1;
    }
    a.tiles = W.tiles;
    a.sb = W.sb;
    a.rows = W.rows;
    a.cols = W.cols;
    if (W.rows % (epi == EPI_SWIGLU ? 32 : 16)) {
        set_error("qgemv: rows %d not a multiple of the row block", W.rows);
        return -1;
    }
    bool f32 = W.sdtype == MLXD_F32;
    if (W.group == 64) return f32 ? dispatch_gemv<64, true>(pro, epi, a, st, pdl)
                                  : dispatch_gemv<64, false>(pro, epi, a, st, pdl);
    if (W.group == 32) return f32 ? dispatch_gemv<32, true>(pro, epi, a, st, pdl)
                                  : dispatch_gemv<32, false>(pro, epi, a, st, pdl);
    set_error("qgemv: group size %d not supported", W.group);
    return -1;
}

}  // namespace mlxd
