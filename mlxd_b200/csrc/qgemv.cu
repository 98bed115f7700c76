// Quantized projections: y = x . deq(W)^T for decode (one token) and for
// prompt chunks on the generic path, and the repack into the decode layout.
//
// Replaces mlx_quantized_matmul(transpose=true, group, 4, "affine") (and the
// dense bf16 matmul) of fwd_linear (src/engine/forward.c:11-63, cast to bf16
// :46-54). Every kernel here computes the same value for an output: the
// group-exact arithmetic of gemv_i8.cuh (per-group fixed-point input, exact
// integer group sums, f64 combination, one rounding to bf16), so decode,
// prefill and tensor-parallel shards agree bit for bit with each other and
// with the oracle.
//
// Layouts (QMat, internal.h): every quantized matrix keeps the MLX arrays
// (w u32 [rows][cols/8], scales/biases [rows][cols/G]); gate|up is stored as
// alternating 64-row blocks of gate and up rows. Matrices with group 64,
// bf16 scales and cols a multiple of 512 also get the decode layout (ti8:
// tiles of 16 rows x 64 columns whose lane words are the u8 A fragments of
// mma.m16n8k32; sbi: per 16 rows x 8 groups, one 32-byte scale/bias record
// per (row pair, group parity)).
#include <mutex>
#include <stdlib.h>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(qgemv)

// ------------------------------------------------------------------ repack

// Integer-MMA tile layout (group 64): lane L = 4g + t of tile (rb, grp) holds
// four words; word i covers row g + 8(i&1) and group columns
// k = 16(i>>1) + 4t + j (j = 0..3, byte j): its low nibble is q(row, k), its
// high nibble q(row, k + 32). Masking the low nibbles gives the u8 A fragment
// of mma.m16n8k32 for columns 0-31 of the group, shifting and masking the
// high nibbles the one for columns 32-63.
__global__ void repack_i8_kernel(const uint32_t *__restrict__ w, int ldw, int nrb, int ng,
                                 uint8_t *__restrict__ tiles) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)nrb * ng * 32) return;
    const int lane = (int)(idx & 31);
    const int g = (int)((idx >> 5) % ng);
    const int rb = (int)((idx >> 5) / ng);
    const int gq = lane >> 2, t = lane & 3;
    auto q = [&](int row, int k) -> uint32_t {
        const int col = g * 64 + k;
        return (w[(size_t)row * ldw + (col >> 3)] >> (4 * (col & 7))) & 0xFu;
    };
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = rb * 16 + gq + 8 * (i & 1);
        const int kb = 16 * (i >> 1) + 4 * t;
        uint32_t v = 0;
        for (int j = 0; j < 4; j++) v |= (q(row, kb + j) | (q(row, kb + j + 32) << 4)) << (8 * j);
        o[i] = v;
    }
    const size_t tile = (size_t)rb * ng + g;
    *reinterpret_cast<uint4 *>(tiles + (tile * 32 + lane) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
}

// scale/bias records of the integer-MMA layout: record (rb, bk, g, h), 32 B:
// for j = 0..3, (s, b) of row g then of row g + 8 for group 8bk + 2j + h
__global__ void repack_sbi_kernel(const uint16_t *__restrict__ s, const uint16_t *__restrict__ b, int lds,
                                  int nrb, int nbk, uint8_t *__restrict__ sbi) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)nrb * nbk * 16) return;
    const int h = (int)(idx & 1);
    const int gq = (int)((idx >> 1) & 7);
    const int bk = (int)((idx >> 4) % nbk);
    const int rb = (int)((idx >> 4) / nbk);
    const int rowA = rb * 16 + gq, rowB = rowA + 8;
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const size_t grp = (size_t)bk * 8 + 2 * j + h;
        const size_t ia = (size_t)rowA * lds + grp, ib = (size_t)rowB * lds + grp;
        o[2 * j] = (uint32_t)s[ia] | ((uint32_t)b[ia] << 16);
        o[2 * j + 1] = (uint32_t)s[ib] | ((uint32_t)b[ib] << 16);
    }
    const size_t rec = ((size_t)rb * nbk + bk) * 16 + gq * 2 + h;
    uint4 *dst = reinterpret_cast<uint4 *>(sbi + rec * 32);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// decode layout of a whole matrix from its MLX arrays (already in device
// memory, rows in the matrix's own order: for gate|up the decode row block p
// holds gate rows 8p..8p+7 then up rows 8p..8p+7, so that one row block is
// a whole SwiGLU unit; the MLX arrays alternate 64 gate and 64 up rows)
__global__ void gateup_rows_kernel(int inter, int *map) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;   // decode row
    if (r >= 2 * inter) return;
    const int rb = r / 16, within = r % 16, up = within >> 3;
    const int logical = rb * 8 + (within & 7);              // gate/up row index
    map[r] = (logical / 64) * 128 + up * 64 + logical % 64;
}

__global__ void gather_rows_u32(const uint32_t *src, int ld, const int *map, int rows, uint32_t *dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)rows * ld) return;
    const int r = (int)(i / ld), c = (int)(i % ld);
    dst[i] = src[(size_t)map[r] * ld + c];
}
__global__ void gather_rows_u16(const uint16_t *src, int ld, const int *map, int rows, uint16_t *dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)rows * ld) return;
    const int r = (int)(i / ld), c = (int)(i % ld);
    dst[i] = src[(size_t)map[r] * ld + c];
}

int build_decode_layout(QMat &M, bool gateup, cudaStream_t st) {
    if (!M.fast()) return 0;
    const int nrb = M.rows / 16, ng = M.cols / 64, nbk = ng / 8;
    M.ti8 = (uint8_t *)dev_alloc(M.ti8_bytes());
    M.sbi = (uint8_t *)dev_alloc(M.sbi_bytes());
    if (!M.ti8 || !M.sbi) return -1;
    const uint32_t *w = M.w;
    const uint16_t *s = (const uint16_t *)M.s, *b = (const uint16_t *)M.b;
    uint32_t *tw = nullptr;
    uint16_t *ts = nullptr, *tb = nullptr;
    int *map = nullptr;
    if (gateup) {
        // the decode layout interleaves 16-row blocks; regroup the rows first
        const int ldw = M.cols / 8;
        map = (int *)dev_alloc((size_t)M.rows * 4);
        tw = (uint32_t *)dev_alloc((size_t)M.rows * ldw * 4);
        ts = (uint16_t *)dev_alloc((size_t)M.rows * ng * 2);
        tb = (uint16_t *)dev_alloc((size_t)M.rows * ng * 2);
        if (!map || !tw || !ts || !tb) {
            dev_free(map); dev_free(tw); dev_free(ts); dev_free(tb);
            return -1;
        }
        gateup_rows_kernel<<<(M.rows + 255) / 256, 256, 0, st>>>(M.rows / 2, map);
        const size_t nw = (size_t)M.rows * ldw, ns = (size_t)M.rows * ng;
        gather_rows_u32<<<(unsigned)((nw + 255) / 256), 256, 0, st>>>(M.w, ldw, map, M.rows, tw);
        gather_rows_u16<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(s, ng, map, M.rows, ts);
        gather_rows_u16<<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(b, ng, map, M.rows, tb);
        w = tw;
        s = ts;
        b = tb;
    }
    const size_t nt = (size_t)nrb * ng * 32;
    repack_i8_kernel<<<(unsigned)((nt + 255) / 256), 256, 0, st>>>(w, M.cols / 8, nrb, ng, M.ti8);
    const size_t ni = (size_t)nrb * nbk * 16;
    repack_sbi_kernel<<<(unsigned)((ni + 255) / 256), 256, 0, st>>>(s, b, ng, nrb, nbk, M.sbi);
    const bool ok = cuda_ok(cudaGetLastError(), "repack");
    if (gateup) {
        cudaStreamSynchronize(st);
        dev_free(map); dev_free(tw); dev_free(ts); dev_free(tb);
    }
    return ok ? 0 : -1;
}

// ------------------------------------------------------------- epilogues

// the value of output row `row` (f64, one rounding here); EPI_SWIGLU: row is
// the gate/up pair index, v the gate value and vu the up value
template <int EPI>
MLXD_DEV void epi_out(const GemvArgs &a, int row, double v, double vu, const uint16_t *res_s,
                      unsigned long long &best) {
    if constexpr (EPI == EPI_SWIGLU) {
        a.y[row] = f2bf(swiglu_bf16(bf2f(d2bf(v)), bf2f(d2bf(vu))));
    } else if constexpr (EPI == EPI_ARGMAX) {
        const uint16_t h = d2bf(v);
        a.y[row] = h;
        const unsigned long long key = argmax_key(bf2f(h), a.row_offset + row);
        best = key > best ? key : best;
    } else if constexpr (EPI == EPI_RESIDUAL) {
        const float r = bf2f(res_s ? *res_s : a.residual[row]);
        a.y[row] = f2bf(__fadd_rn(r, bf2f(d2bf(v))));
    } else if constexpr (EPI == EPI_PARTIAL) {
        if (a.tp_n > 0) {
            const unsigned epoch = *a.tp_seq * a.tp_mul + a.tp_add;
            const unsigned long long bits = (unsigned long long)__double_as_longlong(v);
            for (int p = 0; p < a.tp_n; p++)
                st_line(a.tp_line[p] + (size_t)row * 4, (uint32_t)bits, epoch, (uint32_t)(bits >> 32), epoch);
        } else {
            a.yf[row] = v;
        }
    } else {
        a.y[row] = d2bf(v);
    }
}

// ---------------------------------------------- integer-MMA decode GEMV
//
// One token, group 64, bf16 scales, cols a multiple of 512. A work item is a
// block of 8 consecutive groups of one row block (8 tiles, 4 KB of weights
// plus two 16-byte scale/bias words per lane). Per item, two mma.m16n8k32
// per tile give the exact digit sums; the 8 N columns hold (group parity,
// digit), so a lane holds two digit columns of one group for rows g and g+8
// and turns them into that group's exact f64 terms (gemv_i8.cuh i8_item).
// smem: B fragments xb[group][digit][t], the group table, a 16-byte zero
// entry, the f64 item partials and the counters, the residual rows and the
// cp.async item slots.
struct I8Smem {
    size_t xb, gt, zero, pool, cnt, res, ring, total;
};
// res: the residual rows of the CTA's units (16 bf16 per unit);
// ring: one 4.6 KB item slot per warp (ring_warps of them) for the item
// requested with cp.async before the producer is waited for
static __host__ __device__ inline I8Smem i8_layout(int cols, int pool_items, int pool_units, int ring_warps = 0) {
    I8Smem L;
    const int ng = cols / 64;
    L.xb = 0;
    L.gt = L.xb + (size_t)ng * I8_ENT * 16;
    L.zero = L.gt + (size_t)ng * sizeof(GTab);
    L.pool = L.zero + 16;
    L.cnt = L.pool + (size_t)pool_items * 16 * sizeof(double);
    L.res = ((L.cnt + (size_t)pool_units * 4 + 15) / 16) * 16;
    L.ring = L.res + (size_t)pool_units * 32;
    L.total = L.ring + (size_t)ring_warps * 4608;
    return L;
}

// CTA c owns units [c*U/G, (c+1)*U/G) (a unit is a row block: for SwiGLU
// 8 gate rows and their 8 up rows); warp w of the NW warps takes items w, w+NW,
// ... of that range and keeps the next DEPTH items in registers while
// computing the current one, the first DEPTH of them requested before the
// PDL wait. Each item's 16 f64 partials go to their own place in shared
// memory and the warp that completes a unit adds them and runs the epilogue:
// no global workspace, no grid-wide atomics.
// SM2: each warp's second item goes to a shared-memory slot by cp.async
// before the wait (DEPTH 1), so two items per warp stream during the wait and
// the staging of x without costing registers
template <int PRO, int EPI, int NW, int DEPTH, bool SM2>
__global__ void __launch_bounds__(NW * 32, 1) qgemv_i8_kernel(GemvArgs a, int pool_items) {
    constexpr int NT = NW * 32;
    constexpr int UNIT_RB = 1;
    static_assert(DEPTH == 1 || DEPTH == 2, "register item buffers");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(16) float s_red[NW];
    __shared__ unsigned long long s_key[NW];
    MLXD_TRACE_START
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
    double *pool = reinterpret_cast<double *>(smem_raw + L.pool);
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
    I8Pre<NT> pre;
    i8_stage_pre<NT>(pre, PRO == PRO_RMSNORM ? a.norm_w : nullptr, a.cols);
    pdl_wait();
    MLXD_TRACE_WAITED
    if (res_mine) cp_async_wait<0>();
    uint32_t *xbw = reinterpret_cast<uint32_t *>(smem_raw + L.xb);
    GTab *gt = reinterpret_cast<GTab *>(smem_raw + L.gt);
    uint32_t *zero16 = reinterpret_cast<uint32_t *>(smem_raw + L.zero);
    i8_stage<NT>(a.x, PRO == PRO_RMSNORM ? a.norm_w : nullptr, a.cols, a.eps, xbw, gt, zero16, s_red, pre);
    pdl_trigger();
    const I8Lane IL = i8_lane(xbw, gt, zero16);

    unsigned long long best = 0ull;
    // the item's 16 partial sums to the pool; the warp completing a unit
    // adds the unit's partials in item order and runs the epilogue
    auto finish = [&](int k, double y0, double y1) {
        const int unit = k / ipu;
        const int iu = k - unit * ipu;
        double *ps = pool + (size_t)unit * ipu * 16;
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
        if (done && lane < 16) {
            __threadfence_block();
            double acc = 0.0;
            for (int i = 0; i < nbk; i++) acc += ps[i * 16 + lane];
            if constexpr (EPI == EPI_SWIGLU) {
                // lane l < 8: gate row l of the block; its up row is lane l + 8
                const double up = __shfl_sync(0x0000ffffu, acc, (lane & 7) + 8);
                if (lane < 8) epi_out<EPI>(a, (u0 + unit) * 8 + lane, acc, up, nullptr, best);
            } else {
                const int row = (u0 + unit) * 16 + lane;
                epi_out<EPI>(a, row, acc, acc, res_s ? s_res + unit * 16 + lane : nullptr, best);
            }
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
        double y0, y1;
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
            double y0, y1;
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
    MLXD_TRACE_END(0x10 + EPI + 8 * PRO)
}

int num_sms() {
    static int sms[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!sms[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = v > 0 ? v : 148;
    }
    return sms[dev];
}

// cudaFuncSetAttribute is per device: remember, per kernel and device, the
// largest dynamic shared-memory size already allowed
bool smem_allowed(const void *kern, size_t bytes) {
    static std::mutex mu;
    static std::vector<std::pair<std::pair<const void *, int>, size_t>> done;
    if (bytes <= 48 * 1024) return true;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (auto &e : done)
        if (e.first.first == kern && e.first.second == dev) {
            if (e.second >= bytes) return true;
            if (!cuda_ok(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                         "cudaFuncSetAttribute"))
                return false;
            e.second = bytes;
            return true;
        }
    if (!cuda_ok(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                 "cudaFuncSetAttribute"))
        return false;
    done.push_back({{kern, dev}, bytes});
    return true;
}

template <int PRO, int EPI, int NW, int DEPTH, bool SM2>
static int launch_gemv_i8_cfg(GemvArgs a, cudaStream_t st, bool pdl) {
    auto kern = qgemv_i8_kernel<PRO, EPI, NW, DEPTH, SM2>;
    const int unit_rb = 1;
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
    if (!smem_allowed((const void *)kern, smem)) return -1;
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

// 16 warps with one item in registers ahead. A launch without programmatic
// dependent launch (a projection on its own) also streams each warp's second
// item into shared memory before staging x; inside the PDL-chained decode
// graph the same early traffic slows the previous kernel's tail, so chained
// launches keep one item. A launch capped to the SMs that the running
// attention kernel leaves free (the o projection) streams two items per warp
// too: its CTAs are resident and idle for the whole attention step.
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
    MLXD_GEMVI_CASE(PRO_PLAIN, EPI_PARTIAL)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_STORE)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_RESIDUAL)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_SWIGLU)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_ARGMAX)
    MLXD_GEMVI_CASE(PRO_RMSNORM, EPI_PARTIAL)
#undef MLXD_GEMVI_CASE
    set_error("qgemv: bad prologue/epilogue");
    return -1;
}

// --------------------------------------------------- generic exact path
//
// Any group size (32, 64), f32 or bf16 scales, any width, any number of
// tokens, and dense bf16 weights. Two launches: xfix_kernel writes each
// token's input in the per-group fixed point (X [S][cols] int32 and the group
// table [S][ng]) into the caller's workspace; gemv_generic_kernel then gives
// one warp to each (output, token): lane l takes groups l, l+32, ..., forms
// P_g = sum_k q_k X_k as an integer and adds the group's exact f64 terms; the
// warp's f64 partials are summed by a butterfly and rounded once.

// one warp per (group, token)
__global__ void xfix_kernel(const uint16_t *__restrict__ x, int cols, int G, int S, int32_t *__restrict__ X,
                            GTab *__restrict__ gt) {
    const int ng = cols / G;
    const int wg = (int)(((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (wg >= ng * S) return;
    const int s = wg / ng, g = wg % ng;
    const uint16_t *xg = x + (size_t)s * cols + (size_t)g * G;
    unsigned mx = 0u;
    for (int k = lane; k < G; k += 32) mx = max(mx, (unsigned)(xg[k] & 0x7fffu));
    mx = __reduce_max_sync(0xffffffffu, mx);
    const int eb = (int)(mx >> 7);
    const bool bad = eb == 0xff;
    int E = bad ? 0 : eb - 127;
    if (E < -100) E = -100;
    const float sc = __int_as_float((127 + 20 - E) << 23);
    constexpr float MAGIC = 12582912.0f;
    int tsum = 0;
    for (int k = lane; k < G; k += 32) {
        const int v = bad ? 0 : (int)__float_as_uint(__fmaf_rn(bf2f(xg[k]), sc, MAGIC)) - 0x4B400000;
        X[(size_t)s * cols + (size_t)g * G + k] = v;
        tsum += v;
    }
    tsum = __reduce_add_sync(0xffffffffu, tsum);
    if (lane == 0) {
        GTab e;
        e.tf = bad ? __longlong_as_double(0x7ff8000000000000ll) : int_times_pow2(tsum, E - 20);
        e.e = E;
        e.pad = 0;
        gt[(size_t)s * ng + g] = e;
    }
}

// the f64 value of row r for token s (warp-wide; every lane returns it)
template <bool SF32>
MLXD_DEV double generic_row(const QMat &W, int r, const int32_t *X, const GTab *gt) {
    const int lane = threadIdx.x & 31;
    const int G = W.group, ng = W.cols / G;
    double acc = 0.0;
    const uint32_t *wr = W.w + (size_t)r * (W.cols / 8);
    for (int g = lane; g < ng; g += 32) {
        int P = 0;
        const int32_t *xg = X + (size_t)g * G;
        for (int wd = 0; wd < G / 8; wd++) {
            const uint32_t v = wr[g * (G / 8) + wd];
#pragma unroll
            for (int i = 0; i < 8; i++) P += (int)((v >> (4 * i)) & 0xFu) * xg[wd * 8 + i];
        }
        double sc, bi;
        if constexpr (SF32) {
            sc = (double)((const float *)W.s)[(size_t)r * ng + g];
            bi = (double)((const float *)W.b)[(size_t)r * ng + g];
        } else {
            sc = (double)bf2f(((const uint16_t *)W.s)[(size_t)r * ng + g]);
            bi = (double)bf2f(((const uint16_t *)W.b)[(size_t)r * ng + g]);
        }
        const GTab e = gt[g];
        acc = fma(sc, int_times_pow2(P, e.e - 20), acc);
        acc = fma(bi, e.tf, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

MLXD_DEV double dense_row(const QMat &W, int r, const uint16_t *x) {
    const int lane = threadIdx.x & 31;
    double acc = 0.0;
    const uint16_t *wr = W.dense + (size_t)r * W.cols;
    for (int k = lane; k < W.cols; k += 32) acc = fma((double)bf2f(x[k]), (double)bf2f(wr[k]), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

// grid.x: outputs in groups of 8 (one per warp), grid.y: tokens. Outputs
// are rows, or gate/up pairs for SwiGLU (rows 128p + i and 128p + 64 + i).
// y / yf / residual are [S][outputs].
template <int EPI, int KIND>   // KIND 0: quantized bf16 scales, 1: quantized f32, 2: dense
__global__ void __launch_bounds__(256) gemv_generic_kernel(QMat W, GemvArgs a, const int32_t *X, const GTab *gt,
                                                            int outs) {
    const int o = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int s = blockIdx.y;
    if (o >= outs) return;
    const int ng = W.quant ? W.cols / W.group : 0;
    const int32_t *Xs = X + (size_t)s * W.cols;
    const GTab *gs = gt + (size_t)s * ng;
    const uint16_t *xs = a.x + (size_t)s * W.cols;
    auto row = [&](int r) -> double {
        if constexpr (KIND == 2) return dense_row(W, r, xs);
        else return generic_row<KIND == 1>(W, r, Xs, gs);
    };
    double v, vu = 0.0;
    if constexpr (EPI == EPI_SWIGLU) {
        const int r = (o / 64) * 128 + o % 64;
        v = row(r);
        vu = row(r + 64);
    } else {
        v = row(o);
    }
    if ((threadIdx.x & 31) != 0) return;
    GemvArgs b = a;
    b.y = a.y ? a.y + (size_t)s * outs : nullptr;
    b.yf = a.yf ? a.yf + (size_t)s * outs : nullptr;
    b.residual = a.residual ? a.residual + (size_t)s * outs : nullptr;
    unsigned long long best = 0ull;
    epi_out<EPI>(b, o, v, vu, nullptr, best);
    if constexpr (EPI == EPI_ARGMAX) atomicMax(a.amax, best);
}

size_t generic_ws_bytes(const QMat &W, int S, int pro) {
    size_t b = 0;
    if (pro == PRO_RMSNORM) b += (((size_t)S * W.cols * 2 + 255) / 256) * 256;
    if (W.quant) b += (size_t)S * W.cols * 4 + (size_t)S * (W.cols / W.group) * sizeof(GTab);
    return b + 256;
}

template <int EPI>
static int launch_generic(const QMat &W, GemvArgs a, int S, unsigned char *ws, cudaStream_t st) {
    int32_t *X = nullptr;
    GTab *gt = nullptr;
    if (W.quant) {
        const int ng = W.cols / W.group;
        X = reinterpret_cast<int32_t *>(ws);
        gt = reinterpret_cast<GTab *>(ws + (((size_t)S * W.cols * 4 + 15) / 16) * 16);
        const size_t warps = (size_t)ng * S;
        xfix_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(a.x, W.cols, W.group, S, X, gt);
        MLXD_CHECK(cudaGetLastError());
    }
    const int outs = EPI == EPI_SWIGLU ? W.rows / 2 : W.rows;
    dim3 grid((outs + 7) / 8, S);
    if (!W.quant) gemv_generic_kernel<EPI, 2><<<grid, 256, 0, st>>>(W, a, X, gt, outs);
    else if (W.sdtype == MLXD_F32) gemv_generic_kernel<EPI, 1><<<grid, 256, 0, st>>>(W, a, X, gt, outs);
    else gemv_generic_kernel<EPI, 0><<<grid, 256, 0, st>>>(W, a, X, gt, outs);
    MLXD_CHECK(cudaGetLastError());
    return 0;
}

int qgemm_generic(const QMat &W, int pro, int epi, GemvArgs a, int S, void *ws, size_t ws_bytes, cudaStream_t st) {
    if (S <= 0) return 0;
    if (ws_bytes < generic_ws_bytes(W, S, pro) || !ws) {
        set_error("linear: workspace of %zu bytes too small (%zu needed)", ws_bytes, generic_ws_bytes(W, S, pro));
        return -1;
    }
    if (epi == EPI_SWIGLU && W.rows % 128) {
        set_error("linear: gate|up rows %d not a multiple of 128", W.rows);
        return -1;
    }
    unsigned char *p = (unsigned char *)ws;
    if (pro == PRO_RMSNORM) {
        uint16_t *xn = (uint16_t *)p;
        if (rmsnorm_rows(a.x, S, W.cols, a.norm_w, a.eps, xn, st)) return -1;
        a.x = xn;
        p += (((size_t)S * W.cols * 2 + 255) / 256) * 256;
    }
    switch (epi) {
    case EPI_STORE: return launch_generic<EPI_STORE>(W, a, S, p, st);
    case EPI_RESIDUAL: return launch_generic<EPI_RESIDUAL>(W, a, S, p, st);
    case EPI_SWIGLU: return launch_generic<EPI_SWIGLU>(W, a, S, p, st);
    case EPI_ARGMAX: return launch_generic<EPI_ARGMAX>(W, a, S, p, st);
    case EPI_PARTIAL: return launch_generic<EPI_PARTIAL>(W, a, S, p, st);
    }
    set_error("linear: bad epilogue");
    return -1;
}

// ------------------------------------------------------------ dispatch

int qgemv(const QMat &W, int pro, int epi, GemvArgs a, cudaStream_t st, bool pdl) {
    a.rows = W.rows;
    a.cols = W.cols;
    if (((uintptr_t)a.x | (uintptr_t)a.norm_w) & 15) {
        set_error("qgemv: x and the norm weights must be 16-byte aligned");
        return -1;
    }
    if (a.tp_n > 0 && !(W.ti8 && W.sbi && W.fast() && epi == EPI_PARTIAL)) {
        set_error("qgemv: the tensor-parallel send needs a decode-layout partial projection");
        return -1;
    }
    if (W.ti8 && W.sbi && W.fast()) {
        if (W.rows % 16) {
            set_error("qgemv: rows %d not a multiple of the row block", W.rows);
            return -1;
        }
        a.ti8 = W.ti8;
        a.sbi = W.sbi;
        return dispatch_gemv_i8(pro, epi, a, st, pdl);
    }
    return qgemm_generic(W, pro, epi, a, 1, a.gws, a.gws_bytes, st);
}

// ------------------------------------------ decode GEMV on static scratch
//
// The same one-token projection for callers that cannot allocate device
// memory at the time they call it: code running inside a caching allocator's
// callback or out-of-memory handler (allocating there re-enters the
// allocator), and a serving loop that owns all device memory up front under
// a fixed plan (a cudaMalloc mid-loop can fail once the plan has taken the
// HBM, and its implicit device synchronisation stalls every stream). The
// generic path's per-call workspace (the input in per-group fixed point,
// 4 bytes per column, and a 16-byte entry per group) lives in one fixed array
// of device memory below, 2 MiB + 64 KiB, which bounds the input at 262144
// columns (the integer-MMA layout stages its input in shared memory and needs
// none of it). Every call on a device shares the array and it keeps what the
// last call left there; each call writes all the workspace it reads before
// reading it. Two calls whose kernels can overlap on the GPU, i.e. on streams
// with no ordering between them, race on the array and give wrong results.
constexpr size_t STATIC_SCRATCH_BYTES = ((size_t)2 << 20) + ((size_t)64 << 10);
constexpr int STATIC_MAX_COLS = 1 << 18;
constexpr int STATIC_MAX_DEVICES = 64;
static __device__ __align__(256) unsigned char g_gemv_static_scratch[STATIC_SCRATCH_BYTES];

// Address of the array on the current device. Looked up once per device, on
// that device's first call (the lookup can load the module, so that first
// call belongs before any stream capture); later calls read the table.
static unsigned char *static_scratch_on_current_device() {
    static std::mutex mu;
    static unsigned char *addr[STATIC_MAX_DEVICES] = {};
    int dev = 0;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return nullptr;
    if (dev < 0 || dev >= STATIC_MAX_DEVICES) {
        set_error("linear_noalloc: device %d beyond the %d supported", dev, STATIC_MAX_DEVICES);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        if (!cuda_ok(cudaGetSymbolAddress(&p, g_gemv_static_scratch), "cudaGetSymbolAddress")) return nullptr;
        addr[dev] = (unsigned char *)p;
    }
    return addr[dev];
}

int qgemv_static_scratch(const QMat &W, const uint16_t *x, uint16_t *y, cudaStream_t st) {
    if (!W.quant) {
        set_error("linear_noalloc: matrix is not quantized");
        return -1;
    }
    const size_t need = generic_ws_bytes(W, 1, PRO_PLAIN);
    if (W.cols > STATIC_MAX_COLS || need > STATIC_SCRATCH_BYTES) {
        set_error("linear_noalloc: a %d x %d matrix needs %zu bytes of workspace; the static scratch holds %zu "
                  "(at most %d columns)",
                  W.rows, W.cols, need, STATIC_SCRATCH_BYTES, STATIC_MAX_COLS);
        return -1;
    }
    unsigned char *base = static_scratch_on_current_device();
    if (!base) return -1;
    GemvArgs a = {};
    a.x = x;
    a.y = y;
    a.gws = base;
    a.gws_bytes = STATIC_SCRATCH_BYTES;
    return qgemv(W, PRO_PLAIN, EPI_STORE, a, st, false);
}

}  // namespace mlxd
