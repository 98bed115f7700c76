// Synthetic MLX-format weights for benchmarks and tests.
//
// Values: N(0, std) approximated by the Irwin-Hall sum of 12 uniforms
// (each 24 bits from SplitMix64, Steele/Lea/Flood 2014), every step an IEEE
// operation, so the host and device generators produce identical bits.
// Quantisation: MLX affine 4-bit (mlx ops.cpp affine_quantize): per group the
// larger-magnitude edge maps exactly to a level, scale = (max-min)/15 signed,
// bias = edge, q = clip(round((w - bias)/scale), 0, 15), nibble j%8 of word
// j/8 (LSB first); scales and biases stored as bf16.
#include "common.cuh"
#include "kernels.h"

#include <math.h>
#include <string.h>

namespace mlxd {

__host__ __device__ static inline uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

#ifdef __CUDA_ARCH__
#define MUL(a, b) __fmul_rn(a, b)
#define SUB(a, b) __fsub_rn(a, b)
#define DIV(a, b) __fdiv_rn(a, b)
#else
#define MUL(a, b) ((a) * (b))
#define SUB(a, b) ((a) - (b))
#define DIV(a, b) ((a) / (b))
#endif

__host__ __device__ static inline uint16_t f2bf_hd(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__host__ __device__ static inline float bf2f_hd(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// value of element e of a stream keyed by seed, as the bf16 bits of N(0,std)
__host__ __device__ static inline uint16_t synth_value(uint64_t seed, uint64_t e, float std) {
    uint64_t base = sm64(seed ^ 0x5EED5EED5EEDull) + e * 6ull;
    uint32_t sum = 0;
    for (int i = 0; i < 6; i++) {
        uint64_t r = sm64(base + (uint64_t)i);
        sum += (uint32_t)(r >> 40);
        sum += (uint32_t)((r >> 16) & 0xFFFFFFu);
    }
    float z = SUB(MUL((float)sum, 1.0f / 16777216.0f), 6.0f);
    return f2bf_hd(MUL(z, std));
}

__host__ __device__ static inline float rint_hd(float x) {
#ifdef __CUDA_ARCH__
    return rintf(x);
#else
    return nearbyintf(x);
#endif
}

// one group: G values -> G/8 words, scale and bias (bf16)
__host__ __device__ static inline void synth_group(uint64_t seed, int row, int col0, int cols, int G,
                                                   float std, uint32_t *wout, uint16_t *sout,
                                                   uint16_t *bout) {
    float v[64];
    float mx = -INFINITY, mn = INFINITY;
    for (int j = 0; j < G; j++) {
        v[j] = bf2f_hd(synth_value(seed, (uint64_t)row * cols + col0 + j, std));
        mx = v[j] > mx ? v[j] : mx;
        mn = v[j] < mn ? v[j] : mn;
    }
    const float n_bins = 15.0f, eps = 1e-7f;
    bool mask = fabsf(mn) > fabsf(mx);
    float sc = DIV(SUB(mx, mn), n_bins);
    if (sc < eps) sc = eps;
    if (!mask) sc = -sc;
    float edge = mask ? mn : mx;
    float q0 = rint_hd(DIV(edge, sc));
    if (q0 != 0.0f) sc = DIV(edge, q0);
    float bi = q0 == 0.0f ? 0.0f : edge;
    for (int w = 0; w < G / 8; w++) {
        uint32_t word = 0;
        for (int k = 0; k < 8; k++) {
            float q = rint_hd(DIV(SUB(v[w * 8 + k], bi), sc));
            q = q < 0.f ? 0.f : (q > n_bins ? n_bins : q);
            word |= ((uint32_t)q & 0xFu) << (4 * k);
        }
        wout[w] = word;
    }
    *sout = f2bf_hd(sc);
    *bout = f2bf_hd(bi);
}

__global__ void synth_q_kernel(uint32_t *w, uint16_t *s, uint16_t *b, int rows, int cols, int G,
                               uint64_t seed, float std) {
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    int ng = cols / G;
    if (idx >= (size_t)rows * ng) return;
    int r = (int)(idx / ng), g = (int)(idx % ng);
    synth_group(seed, r, g * G, cols, G, std, w + (size_t)r * (cols / 8) + g * (G / 8),
                s + (size_t)r * ng + g, b + (size_t)r * ng + g);
}

__global__ void synth_bf16_kernel(uint16_t *out, size_t n, uint64_t seed, float std, float constant) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    out[i] = std > 0.f ? synth_value(seed, i, std) : f2bf_hd(constant);
}

}  // namespace mlxd

extern "C" {

int mlxd_cuda_synth_quantized(uint32_t *w, uint16_t *scales, uint16_t *biases, int rows, int cols,
                              int group, uint64_t seed, float std, void *stream) {
    if (group != 32 && group != 64) {
        mlxd::set_error("synth: group must be 32 or 64");
        return -1;
    }
    if (cols % group) {
        mlxd::set_error("synth: cols %d not a multiple of group %d", cols, group);
        return -1;
    }
    size_t n = (size_t)rows * (cols / group);
    mlxd::synth_q_kernel<<<(unsigned)((n + 127) / 128), 128, 0, (cudaStream_t)stream>>>(
        w, scales, biases, rows, cols, group, seed, std);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

int mlxd_cuda_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float std, float constant,
                         void *stream) {
    mlxd::synth_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        out, n, seed, std, constant);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

void mlxd_host_synth_quantized(uint32_t *w, uint16_t *scales, uint16_t *biases, int rows, int cols,
                               int group, uint64_t seed, float std) {
    int ng = cols / group;
    for (int r = 0; r < rows; r++)
        for (int g = 0; g < ng; g++)
            mlxd::synth_group(seed, r, g * group, cols, group, std,
                              w + (size_t)r * (cols / 8) + g * (group / 8),
                              scales + (size_t)r * ng + g, biases + (size_t)r * ng + g);
}

void mlxd_host_synth_bf16(uint16_t *out, size_t n, uint64_t seed, float std, float constant) {
    for (size_t i = 0; i < n; i++)
        out[i] = std > 0.f ? mlxd::synth_value(seed, i, std) : mlxd::f2bf_hd(constant);
}

}  // extern "C"
