// Small per-token ops: embedding gather, RMSNorm rows, prefill q/k norm +
// RoPE + KV append, residual add.
#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

// fwd_embed (forward.c:65-147): gather rows of the MLX-format table,
// dequantise scale*q + bias (one rounding), bf16 out.
template <bool QUANT, bool SF32>
__global__ void embed_kernel(Embed e, int H, int G, int V, const int32_t *__restrict__ ids,
                             uint16_t *__restrict__ h) {
    int s = blockIdx.x;
    int id = ids[s];
    // an invalid id (a failed draw reports -1) reads row 0; the host rejects
    // the step when it reads the token back
    if (id < 0 || id >= V) id = 0;
    uint16_t *out = h + (size_t)s * H;
    if (QUANT) {
        const uint32_t *w = e.w + (size_t)id * (H / 8);
        int ng = H / G;
        for (int wd = threadIdx.x; wd < H / 8; wd += blockDim.x) {
            uint32_t v = w[wd];
            int g = (wd * 8) / G;
            float sc, bi;
            if (SF32) {
                sc = ((const float *)e.s)[(size_t)id * ng + g];
                bi = ((const float *)e.b)[(size_t)id * ng + g];
            } else {
                sc = bf2f(((const uint16_t *)e.s)[(size_t)id * ng + g]);
                bi = bf2f(((const uint16_t *)e.b)[(size_t)id * ng + g]);
            }
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float a = __fmaf_rn(sc, (float)((v >> (8 * i)) & 0xF), bi);
                float b = __fmaf_rn(sc, (float)((v >> (8 * i + 4)) & 0xF), bi);
                o[i] = pack_bf2(a, b);
            }
            *reinterpret_cast<uint4 *>(out + wd * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {
        const uint16_t *src = e.dense + (size_t)id * H;
        for (int i = threadIdx.x; i < H; i += blockDim.x) out[i] = src[i];
    }
}

int embed_rows(const Embed &e, int H, int G, int V, const int32_t *ids, int S, uint16_t *h,
               cudaStream_t st) {
    if (e.quant) {
        if (e.sdtype == MLXD_F32) embed_kernel<true, true><<<S, 128, 0, st>>>(e, H, G, V, ids, h);
        else embed_kernel<true, false><<<S, 128, 0, st>>>(e, H, G, V, ids, h);
    } else {
        embed_kernel<false, false><<<S, 128, 0, st>>>(e, H, G, V, ids, h);
    }
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

// fwd_rmsnorm (forward.c:186-219), mlx_fast_rms_norm numerics: f32 sum of
// squares, 1/sqrt(mean + eps), normalised value rounded to bf16, times the
// bf16 weight, rounded again.
__global__ void rmsnorm_kernel(const uint16_t *__restrict__ x, int n, const uint16_t *__restrict__ w,
                               float eps, uint16_t *__restrict__ y) {
    const uint16_t *xr = x + (size_t)blockIdx.x * n;
    uint16_t *yr = y + (size_t)blockIdx.x * n;
    __shared__ float red[32];
    float acc = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = bf2f(xr[i]);
        acc = fmaf(v, v, acc);
    }
    acc = warp_sum(acc);
    int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = acc;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < nw; i++) tot += red[i];
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        yr[i] = f2bf(__fmul_rn(bf2f(w[i]), rbf(__fmul_rn(bf2f(xr[i]), inv))));
}

int rmsnorm_rows(const uint16_t *x, int rows, int n, const uint16_t *w, float eps, uint16_t *y,
                 cudaStream_t st) {
    if (rows <= 0) return 0;
    int threads = n >= 1024 ? 256 : (n >= 256 ? 128 : 32);
    rmsnorm_kernel<<<rows, threads, 0, st>>>(x, n, w, eps, y);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

// Prefill: per token s and head, q/k norm + RoPE at pos0+s, then write q to
// q_out [S][hq][D] and k, v into the cache slot (pos % cap).
__global__ void qk_rope_append_kernel(const uint16_t *__restrict__ qkv, int qdim, int hq, int hkv,
                                      int gate, int D, const uint16_t *qn, const uint16_t *kn,
                                      float eps, const float *cs, int rope_dims, int pos0,
                                      uint16_t *q_out, uint16_t *kc, uint16_t *vc, int cap) {
    extern __shared__ float sv[];
    int s = blockIdx.x;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float *v = sv + warp * D;
    const uint16_t *row = qkv + (size_t)s * (qdim + 2 * hkv * D);
    int pos = pos0 + s;
    int slot = pos % cap;
    for (int hv = warp; hv < hq + 2 * hkv; hv += nw) {
        if (hv < hq) {
            const uint16_t *src = row + (size_t)hv * D * (gate ? 2 : 1);
            for (int d = lane; d < D; d += 32) v[d] = bf2f(src[d]);
            __syncwarp();
            head_norm_rope(v, D, qn, eps, cs, rope_dims, pos);
            uint16_t *dst = q_out + ((size_t)s * hq + hv) * D;
            for (int d = lane; d < D; d += 32) dst[d] = f2bf(v[d]);
        } else if (hv < hq + hkv) {
            int kh = hv - hq;
            const uint16_t *src = row + qdim + (size_t)kh * D;
            for (int d = lane; d < D; d += 32) v[d] = bf2f(src[d]);
            __syncwarp();
            head_norm_rope(v, D, kn, eps, cs, rope_dims, pos);
            uint16_t *dst = kc + ((size_t)kh * cap + slot) * D;
            for (int d = lane; d < D; d += 32) dst[d] = f2bf(v[d]);
        } else {
            int kh = hv - hq - hkv;
            const uint16_t *src = row + qdim + (size_t)(hkv + kh) * D;
            uint16_t *dst = vc + ((size_t)kh * cap + slot) * D;
            for (int d = lane; d < D; d += 32) dst[d] = src[d];
        }
        __syncwarp();
    }
}

int qk_rope_append(const uint16_t *qkv, int S, int qdim, int hq, int hkv, int gate,
                   const uint16_t *qn, const uint16_t *kn, float eps, RopeArgs r, int pos0,
                   uint16_t *q_out, uint16_t *kc, uint16_t *vc, int cap, cudaStream_t st) {
    int threads = 256;
    size_t smem = (size_t)(threads / 32) * r.D * sizeof(float);
    qk_rope_append_kernel<<<S, threads, smem, st>>>(qkv, qdim, hq, hkv, gate, r.D, qn, kn, eps,
                                                    r.cs, r.rope_dims, pos0, q_out, kc, vc, cap);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

// tensor parallelism: the row-parallel projection's value is the sum of the
// ranks' f64 partials (exact terms of the group-exact arithmetic, added in
// rank order), rounded once to bf16, then added to the residual in bf16
__global__ void add_partials_kernel(uint16_t *h_out, const uint16_t *h_in, const double *part, int nranks,
                                    size_t stride, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    double v = 0.0;
    for (int r = 0; r < nranks; r++) v += part[(size_t)r * stride + i];
    h_out[i] = f2bf(__fadd_rn(bf2f(h_in[i]), bf2f(d2bf(v))));
}

int add_partials(uint16_t *h_out, const uint16_t *h_in, const double *part, int nranks, size_t stride, size_t n,
                 cudaStream_t st) {
    add_partials_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(h_out, h_in, part, nranks, stride, n);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace mlxd
