// Shared device helpers for libmlxd_cuda (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "internal.h"

#ifndef __CUDACC__
#error "common.cuh is CUDA-only"
#endif

#define MLXD_DEV __device__ __forceinline__

// ---------------------------------------------------------------- bf16 bits
MLXD_DEV float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
MLXD_DEV uint16_t f2bf(float f) {  // round to nearest even, NaN kept quiet
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
MLXD_DEV float rbf(float f) { return bf2f(f2bf(f)); }
MLXD_DEV uint32_t pack_bf2(float lo, float hi) {
    return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}
MLXD_DEV float lo_bf(uint32_t v) { return __uint_as_float(v << 16); }
MLXD_DEV float hi_bf(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Cody-Waite exp with a degree-7 Taylor polynomial; the CPU oracle evaluates
// the identical expression (same constants, same fused multiply-adds), so the
// two produce identical bits. Valid on [-104, 88.72]; 0 below, +inf above.
MLXD_DEV float own_expf(float x) {
    if (!(x > -104.0f)) return 0.0f;
    if (x > 88.72f) return __int_as_float(0x7f800000);
    float n = rintf(__fmul_rn(x, 1.44269504f));
    float r = __fmaf_rn(n, -0.693145751953125f, x);
    r = __fmaf_rn(n, -1.428606765330187e-06f, r);
    float p = 1.0f / 5040.0f;
    p = __fmaf_rn(p, r, 1.0f / 720.0f);
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = (int)n;
    int a = ni / 2, b = ni - a;
    float sa = __int_as_float((a + 127) << 23), sb = __int_as_float((b + 127) << 23);
    return __fmul_rn(__fmul_rn(p, sa), sb);
}

// mlx Sigmoid on bf16 data: y = 1/(1+exp(|x|)); x<0 -> y, else 1-y; every
// intermediate rounded to bf16 (bfloat16 arithmetic).
MLXD_DEV float sigmoid_bf16(float g) {
    float e = rbf(own_expf(fabsf(g)));
    float y = rbf(__fdiv_rn(1.0f, rbf(__fadd_rn(1.0f, e))));
    return g < 0.0f ? y : rbf(__fsub_rn(1.0f, y));
}

// silu(g)*u with the reference's three rounding points (forward.c:926-935)
MLXD_DEV float swiglu_bf16(float g, float u) {
    float sg = sigmoid_bf16(g);
    float si = rbf(__fmul_rn(g, sg));
    return rbf(__fmul_rn(si, u));
}

// ---------------------------------------------------------------- PTX bits
MLXD_DEV uint4 ldg_nc_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
MLXD_DEV uint2 ldg_nc_v2(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// weight loads marked first for eviction from L2 once read (each byte of the
// weight stream is read once per step)
MLXD_DEV uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
MLXD_DEV uint4 ldg_nc_v4_ef(const void *p, uint64_t pol) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(pol));
    return r;
}

// greedy key: order-preserving float bits over the first-index tie rule
// (a larger key wins; equal values keep the smaller index)
MLXD_DEV unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)k << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

// x pair (k, k+1) of a decode-GEMV input into the fragment order of its
// group: xp[(gi*4 + tt)*XW + j*2 + hi], XW = G/8 words per (group, t)
MLXD_DEV void put_pair(uint32_t *xp, int G, int XW, int k, uint32_t v) {
    const int gi = k / G, kk = k % G;
    const int j = kk >> 4, w16 = kk & 15;
    const int hi = w16 >= 8, tt = (w16 & 7) >> 1;
    xp[(gi * 4 + tt) * XW + j * 2 + hi] = v;
}

// ---- bulk copies (cp.async.bulk into this CTA's own shared memory) and mbarriers
MLXD_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
MLXD_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
MLXD_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// order this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same bytes
MLXD_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
MLXD_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// global -> shared copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) completing on `bar`
MLXD_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// A 16-byte line {a, b, c, d} written by one vector store / read by one
// vector load, bypassing L1 (the tensor-parallel exchange lines)
MLXD_DEV void st_line(uint32_t *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}
MLXD_DEV uint4 ld_line(const uint32_t *p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
MLXD_DEV unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
MLXD_DEV bool mbar_try(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
    return ok != 0;
}
// wait for phase `parity` of `bar`; false after half a second
MLXD_DEV bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    if (mbar_try(addr, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (unsigned i = 1;; i++) {
        if (mbar_try(addr, parity)) return true;
        if ((i & 63u) == 0 && global_ns() - t0 > 500000000ull) return false;
    }
}

// ---- optional timeline trace (compiled in with -DMLXD_TRACE only): thread 0
// of every CTA of a traced kernel appends {tag<<32 | cta, start, waited, end}
// (%globaltimer ns) to a device buffer whose word 0 counts the records.
#ifdef MLXD_TRACE
static __device__ unsigned long long *g_trace;
MLXD_DEV unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
#define MLXD_TRACE_START unsigned long long tr_t0_ = gtime(), tr_t1_ = 0;
#define MLXD_TRACE_WAITED tr_t1_ = gtime();
#define MLXD_TRACE_RESTART tr_t0_ = gtime();
MLXD_DEV unsigned smid_() {
    unsigned r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}
#define MLXD_TRACE_END(tag)                                                                  \
    if (g_trace && threadIdx.x == 0) {                                                       \
        unsigned long long i_ = atomicAdd(g_trace, 1ull);                                    \
        if (i_ < (1ull << 20)) {                                                             \
            unsigned long long *r_ = g_trace + 4 + i_ * 4;                                   \
            r_[0] = ((unsigned long long)(tag) << 32) | ((unsigned long long)smid_() << 20) |  \
                    (blockIdx.x + blockIdx.y * gridDim.x);                                   \
            r_[1] = tr_t0_;                                                                  \
            r_[2] = tr_t1_;                                                                  \
            r_[3] = gtime();                                                                 \
        }                                                                                    \
    }
#define MLXD_TRACE_REC(cond, tag, v1, v2, v3)                                            \
    if (g_trace && (cond)) {                                                                 \
        unsigned long long i_ = atomicAdd(g_trace, 1ull);                                    \
        if (i_ < (1ull << 20)) {                                                             \
            unsigned long long *r_ = g_trace + 4 + i_ * 4;                                   \
            r_[0] = ((unsigned long long)(tag) << 32) | (blockIdx.x + blockIdx.y * gridDim.x); \
            r_[1] = (v1);                                                                    \
            r_[2] = (v2);                                                                    \
            r_[3] = (v3);                                                                    \
        }                                                                                    \
    }
#define MLXD_TRACE_T(var) const unsigned long long var = gtime();
#define MLXD_TRACE_BINDER(name) \
    void trace_bind_##name(unsigned long long *p) { cudaMemcpyToSymbol(g_trace, &p, sizeof p); }
#else
#define MLXD_TRACE_START
#define MLXD_TRACE_RESTART
#define MLXD_TRACE_WAITED
#define MLXD_TRACE_END(tag)
#define MLXD_TRACE_REC(cond, tag, v1, v2, v3)
#define MLXD_TRACE_BINDER(name)
#define MLXD_TRACE_T(var)
#endif

// Programmatic dependent launch: wait for the producer grid / let the
// consumer grid be scheduled. No-ops when the launch has no PDL attribute.
MLXD_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MLXD_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, f32 accumulate
MLXD_DEV void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

MLXD_DEV void ldmatrix_x4(uint32_t (&r)[4], const void *smem) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
MLXD_DEV void ldmatrix_x2(uint32_t (&r)[2], const void *smem) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1]) : "r"(a));
}
MLXD_DEV void ldmatrix_x4_trans(uint32_t (&r)[4], const void *smem) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
MLXD_DEV void cp_async16_zfill(void *smem, const void *gmem, bool valid) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
    int src = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(a), "l"(gmem), "r"(src));
}
MLXD_DEV void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
MLXD_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MLXD_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// 4-bit nibble pair -> bf16x2 of (128 + q_lo, 128 + q_hi): nibbles i and i+4
// of the word land in the low mantissa bits of 128.0 (0x4300), exact.
MLXD_DEV uint32_t nib_pair(uint32_t w, int i) {
    uint32_t v = w >> (4 * i);
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "r"(0x000F000Fu), "r"(0x43004300u));
    return r;  // (v & mask) | magic
}

MLXD_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
MLXD_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One head vector in a warp: optional RMSNorm, then RoPE (rotate-half on the
// first rope_dims features) at absolute position pos with the host-built
// cos/sin table. v: smem staging of D floats. Returns through v (bf16 values).
MLXD_DEV void head_norm_rope(float *v, int D, const uint16_t *nw, float eps, const float *cs,
                               int rope_dims, int pos) {
    int lane = threadIdx.x & 31;
    if (nw) {
        float acc = 0.f;
        for (int d = lane; d < D; d += 32) acc = fmaf(v[d], v[d], acc);
        acc = warp_sum(acc);
        float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), eps)));
        __syncwarp();
        for (int d = lane; d < D; d += 32) v[d] = rbf(__fmul_rn(bf2f(nw[d]), rbf(__fmul_rn(v[d], inv))));
        __syncwarp();
    }
    int half = rope_dims / 2;
    const float *c = cs + (size_t)pos * half * 2;
    float a[4], b[4];
    int cnt = 0;
    for (int i = lane; i < half; i += 32, cnt++) {
        float x1 = v[i], x2 = v[i + half];
        float co = c[2 * i], si = c[2 * i + 1];
        a[cnt] = rbf(__fsub_rn(__fmul_rn(x1, co), __fmul_rn(x2, si)));
        b[cnt] = rbf(__fadd_rn(__fmul_rn(x1, si), __fmul_rn(x2, co)));
    }
    __syncwarp();
    cnt = 0;
    for (int i = lane; i < half; i += 32, cnt++) {
        v[i] = a[cnt];
        v[i + half] = b[cnt];
    }
    __syncwarp();
}
