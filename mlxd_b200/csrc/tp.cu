// Tensor parallelism: the exchanges of one decode step over NVLink, without
// NCCL inside the step.
//
// The reference has no multi-GPU path (one mlx stream, src/engine/engine.c:
// 360-602). Each row-parallel projection (o_proj, down_proj) leaves on every
// rank an f64 partial of each output row: the exact terms of its own groups
// in the library's projection arithmetic. The step needs, on every rank,
// bf16(h + bf16(sum of the partials)), which equals the one-GPU result. A
// mailbox per rank (cudaMalloc'd, mapped into every peer with cudaIpc) holds,
// per exchange parity, one slot of rows per source rank. A row travels as one
// 16-byte line {low word, epoch, high word, epoch} written by a single vector
// store (plain st.global over NVLink, no bulk or TMA copy): each 8-byte half
// is written at once, so a reader that sees the epoch in both halves has the
// whole value, and no fence or separate flag is needed (the LL protocol of
// NCCL's low-latency kernels):
//
//   thread r of CTA c of every rank stores row c*128 + r of its partial into
//   slot [rank] of every rank's mailbox; then it polls (bounded) slots
//   [0..N) of its own mailbox until each holds the epoch, adds the N values in
//   rank order and the residual.
//
// Every rank keeps a device step counter s, advanced once at the end of
// every one-token step (all ranks run the same steps). The epoch of exchange
// idx of step s is s * 2L + idx + 1, read on the device, so a captured graph
// replays it, and no epoch repeats across generations or caches.
// Exchanges alternate between two buffers: when a rank writes exchange e + 2
// into a peer's buffer, it has seen every peer's rows of exchange e + 1, which
// each peer stored after finishing exchange e (its reads included). A wait that exceeds its limit
// sets the error word and returns; the host reports it (no hang, no trap).
// The greedy argmax keys and, for sampled decoding, the vocabulary shards of
// the logits travel the same way in mailboxes of their own.
#include <cuda_runtime.h>
#include <nccl.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "gemv_i8.cuh"
#include "kernels.h"

namespace mlxd {

MLXD_TRACE_BINDER(tp)

constexpr int TP_SLICE = 128;      // rows per CTA (and per flag)
constexpr int TP_MAX = 8;          // ranks
static_assert(TP_MAX <= (int)(sizeof(GemvArgs::tp_line) / sizeof(GemvArgs::tp_line[0])),
              "the GEMV's send half addresses every rank's mailbox");

struct TpPeers {
    unsigned char *mb[TP_MAX];     // every rank's mailbox (own included), mapped here
};

struct TpState {
    int n = 1, rank = 0, H = 0, slices = 0, L2 = 0, V = 0, vslices = 0;
    size_t off_vec, off_key, off_kflag, off_log, off_lflag, bytes;
    unsigned char *mine = nullptr;             // this rank's mailbox
    std::vector<void *> opened;                // peers' mappings (cudaIpcCloseMemHandle)
    TpPeers peers = {};
    int *err = nullptr;                        // device error word
    unsigned *seq = nullptr;                   // device step counter
};

// layout of a mailbox: vector lines, key slots, key flags, logits row,
// logits flags
static void tp_layout(TpState &t) {
    const size_t N = (size_t)t.n;
    t.off_vec = 0;
    t.off_key = t.off_vec + 2 * N * t.H * 16;
    t.off_kflag = t.off_key + 2 * N * 8;
    t.off_log = t.off_kflag + 256;
    t.off_lflag = t.off_log + (((size_t)t.V * 2 + 255) / 256) * 256;
    t.bytes = t.off_lflag + ((N * t.vslices * 4 + 255) / 256) * 256;
}

MLXD_DEV unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
MLXD_DEV void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// wait until *p == v; false (error word set) after about one second
MLXD_DEV bool wait_flag(const unsigned *p, unsigned v, int *err) {
    if (ld_acquire_sys(p) == v) return true;
    const unsigned long long t0 = global_ns();
    for (unsigned i = 1;; i++) {
        if (ld_acquire_sys(p) == v) return true;
        if ((i & 255u) == 0 && global_ns() - t0 > 1000000000ull) {
            atomicExch(err, 1);
            return false;
        }
    }
}

// the line at p once both halves hold the epoch; false (error word set)
// after about one second
MLXD_DEV bool wait_line(const uint32_t *p, unsigned epoch, uint4 &v, int *err) {
    v = ld_line(p);
    if (v.y == epoch && v.w == epoch) return true;
    const unsigned long long t0 = global_ns();
    for (unsigned i = 1;; i++) {
        v = ld_line(p);
        if (v.y == epoch && v.w == epoch) return true;
        if ((i & 255u) == 0 && global_ns() - t0 > 1000000000ull) {
            atomicExch(err, 1);
            return false;
        }
    }
}

// out = bf16(res + bf16(sum over ranks of part)), one row per thread
__global__ void __launch_bounds__(TP_SLICE) tp_sum_kernel(TpPeers peers, unsigned char *mine, size_t off_vec, int n,
                                                          int rank, int H, const double *part, const uint16_t *res,
                                                          uint16_t *out, const unsigned *seq, int L2, int idx,
                                                          int *err) {
    MLXD_TRACE_START
    pdl_wait();
    MLXD_TRACE_WAITED
    const int row = blockIdx.x * TP_SLICE + threadIdx.x;
    const unsigned epoch = *seq * (unsigned)L2 + (unsigned)idx + 1u;
    const int buf = idx & 1;
    if (row < H) {
        const unsigned long long bits = (unsigned long long)__double_as_longlong(part[row]);
        const uint32_t lo = (uint32_t)bits, hi = (uint32_t)(bits >> 32);
        for (int p = 0; p < n; p++) {
            uint32_t *line = reinterpret_cast<uint32_t *>(peers.mb[p] + off_vec) + (((size_t)buf * n + rank) * H + row) * 4;
            st_line(line, lo, epoch, hi, epoch);
        }
    }
    // the next projection's CTAs may start loading weights during the wait
    pdl_trigger();
    if (row < H) {
        double s = 0.0;
        bool ok = true;
        for (int src = 0; src < n && ok; src++) {
            const uint32_t *line = reinterpret_cast<const uint32_t *>(mine + off_vec) + (((size_t)buf * n + src) * H + row) * 4;
            uint4 v;
            ok = wait_line(line, epoch, v, err);
            s += __longlong_as_double((long long)(((unsigned long long)v.z << 32) | v.x));
        }
        out[row] = f2bf(__fadd_rn(bf2f(res[row]), bf2f(d2bf(s))));
    }
    MLXD_TRACE_END(0x30)
}

// the receive half alone, for a projection whose GEMV epilogue stored its
// rows' lines itself: out = bf16(res + bf16(sum over ranks)), one row per
// thread
__global__ void __launch_bounds__(TP_SLICE) tp_recv_kernel(const unsigned char *mine, size_t off_vec, int n, int H,
                                                           const uint16_t *res, uint16_t *out, const unsigned *seq,
                                                           int L2, int idx, int *err) {
    MLXD_TRACE_START
    pdl_wait();
    MLXD_TRACE_WAITED
    pdl_trigger();
    const int row = blockIdx.x * TP_SLICE + threadIdx.x;
    if (row >= H) return;
    const unsigned epoch = *seq * (unsigned)L2 + (unsigned)idx + 1u;
    const int buf = idx & 1;
    double s = 0.0;
    bool ok = true;
    for (int src = 0; src < n && ok; src++) {
        const uint32_t *line = reinterpret_cast<const uint32_t *>(mine + off_vec) + (((size_t)buf * n + src) * H + row) * 4;
        uint4 v;
        ok = wait_line(line, epoch, v, err);
        s += __longlong_as_double((long long)(((unsigned long long)v.z << 32) | v.x));
    }
    out[row] = f2bf(__fadd_rn(bf2f(res[row]), bf2f(d2bf(s))));
    MLXD_TRACE_END(0x31)
}

// greedy: the ranks' argmax keys; every rank takes the largest and ends the
// step (position + 1, step counter + 1, token, key cleared)
__global__ void tp_argmax_kernel(TpPeers peers, unsigned char *mine, size_t off_key, size_t off_kflag, int n, int rank,
                                 unsigned long long *amax, int32_t *d_pos, int32_t *token, unsigned *seq, int *err) {
    pdl_wait();
    const unsigned epoch = *seq + 1u;
    const int buf = (int)(*seq & 1u);
    const int tid = threadIdx.x;
    if (tid < n) {
        unsigned long long *slot = reinterpret_cast<unsigned long long *>(peers.mb[tid] + off_key) + (size_t)buf * n + rank;
        *slot = *amax;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        for (int p = 0; p < n; p++) {
            unsigned *fl = reinterpret_cast<unsigned *>(peers.mb[p] + off_kflag) + (size_t)buf * n + rank;
            st_release_sys(fl, epoch);
        }
    }
    __shared__ unsigned long long keys[TP_MAX];
    if (tid < n) {
        const unsigned *fl = reinterpret_cast<const unsigned *>(mine + off_kflag) + (size_t)buf * n + tid;
        wait_flag(fl, epoch, err);
        keys[tid] = __ldcv(reinterpret_cast<const unsigned long long *>(mine + off_key) + (size_t)buf * n + tid);
    }
    __syncthreads();
    if (tid == 0) {
        unsigned long long m = 0ull;
        for (int p = 0; p < n; p++) m = keys[p] > m ? keys[p] : m;
        *token = (int32_t)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFull));
        *amax = 0ull;
        *d_pos += 1;
        *seq += 1u;
    }
}

// sampled decoding: every rank's vocabulary shard of the logits into every
// rank's full row (the sampler then runs on the whole row on each rank, with
// the same inputs and stream: the same token everywhere). Runs after the
// step's end advanced the counter: epoch s + 1 of the next value.
__global__ void __launch_bounds__(256) tp_gather_logits_kernel(TpPeers peers, unsigned char *mine, size_t off_log,
                                                               size_t off_lflag, int n, int rank, int Vl, int vslices,
                                                               const uint16_t *logits, const unsigned *seq, int *err) {
    pdl_wait();
    const int c = blockIdx.x, tid = threadIdx.x;
    const unsigned epoch = *seq + 1u;
    const int per = (Vl + vslices - 1) / vslices;
    const int i0 = c * per, i1 = min(Vl, i0 + per);
    for (int p = 0; p < n; p++) {
        uint16_t *row = reinterpret_cast<uint16_t *>(peers.mb[p] + off_log) + (size_t)rank * Vl;
        for (int i = i0 + tid; i < i1; i += blockDim.x) row[i] = logits[i];
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        for (int p = 0; p < n; p++) {
            unsigned *fl = reinterpret_cast<unsigned *>(peers.mb[p] + off_lflag) + (size_t)rank * vslices + c;
            st_release_sys(fl, epoch);
        }
    }
    // every slice of every rank must have arrived before the sampler runs:
    // CTA c waits for slice c of all ranks; the sampler's first launch waits
    // for this whole grid
    if (tid < n) {
        const unsigned *fl = reinterpret_cast<const unsigned *>(mine + off_lflag) + (size_t)tid * vslices + c;
        wait_flag(fl, epoch, err);
    }
    __syncthreads();
}

}  // namespace mlxd

using namespace mlxd;

// ------------------------------------------------------------------ host

namespace mlxd {

void tp_free(mlxd_model *m) {
    TpState *t = (TpState *)m->tp;
    if (!t) return;
    cudaDeviceSynchronize();
    for (void *p : t->opened) cudaIpcCloseMemHandle(p);
    dev_free(t->mine);
    dev_free(t->err);
    dev_free(t->seq);
    delete t;
    m->tp = nullptr;
}

// mailboxes and their peer mappings; collective over the model's NCCL
// communicator (every rank calls it once, after the communicator exists)
int tp_setup(mlxd_model *m) {
    if (m->c.tp_size <= 1) return 0;
    if (m->c.tp_size > TP_MAX) {
        set_error("tensor parallelism over %d GPUs: at most %d", m->c.tp_size, TP_MAX);
        return -1;
    }
    TpState *t = new TpState();
    m->tp = t;
    t->n = m->c.tp_size;
    t->rank = m->c.tp_rank;
    t->H = m->c.hidden;
    t->slices = (t->H + TP_SLICE - 1) / TP_SLICE;
    t->L2 = 2 * m->c.layers;
    t->V = m->c.vocab;
    t->vslices = 64;
    tp_layout(*t);
    t->mine = (unsigned char *)dev_alloc(t->bytes);
    t->err = (int *)dev_alloc(sizeof(int));
    t->seq = (unsigned *)dev_alloc(sizeof(unsigned));
    if (!t->mine || !t->err || !t->seq) return -1;
    // flags start below any epoch (epochs start at 1)
    MLXD_CHECK(cudaMemset(t->mine, 0, t->bytes));
    MLXD_CHECK(cudaMemset(t->err, 0, sizeof(int)));
    MLXD_CHECK(cudaMemset(t->seq, 0, sizeof(unsigned)));
    cudaIpcMemHandle_t h;
    MLXD_CHECK(cudaIpcGetMemHandle(&h, t->mine));
    // every rank's handle through the communicator
    unsigned char *dh = (unsigned char *)dev_alloc(sizeof(h) * t->n);
    if (!dh) return -1;
    MLXD_CHECK(cudaMemcpy(dh + sizeof(h) * t->rank, &h, sizeof(h), cudaMemcpyHostToDevice));
    ncclResult_t r = ncclAllGather(dh + sizeof(h) * t->rank, dh, sizeof(h), ncclUint8, (ncclComm_t)m->nccl, nullptr);
    std::vector<cudaIpcMemHandle_t> all(t->n);
    const bool ok = r == ncclSuccess && cuda_ok(cudaDeviceSynchronize(), "handle exchange") &&
                    cuda_ok(cudaMemcpy(all.data(), dh, sizeof(h) * t->n, cudaMemcpyDeviceToHost), "handles");
    dev_free(dh);
    if (!ok) {
        if (r != ncclSuccess) set_error("ncclAllGather: %s", ncclGetErrorString(r));
        return -1;
    }
    for (int p = 0; p < t->n; p++) {
        if (p == t->rank) {
            t->peers.mb[p] = t->mine;
            continue;
        }
        void *ptr = nullptr;
        MLXD_CHECK(cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess));
        t->opened.push_back(ptr);
        t->peers.mb[p] = (unsigned char *)ptr;
    }
    // every rank has mapped every mailbox before any exchange runs
    MLXD_CHECK(cudaDeviceSynchronize());
    int *dummy = (int *)dev_alloc(sizeof(int));
    if (!dummy) return -1;
    r = ncclAllReduce(dummy, dummy, 1, ncclInt32, ncclSum, (ncclComm_t)m->nccl, nullptr);
    const bool ok2 = r == ncclSuccess && cuda_ok(cudaDeviceSynchronize(), "mailbox barrier");
    dev_free(dummy);
    if (!ok2) {
        if (r != ncclSuccess) set_error("ncclAllReduce: %s", ncclGetErrorString(r));
        return -1;
    }
    return 0;
}

static int launch_pdl(cudaStream_t st, bool pdl, dim3 grid, dim3 block, const void *kern, void **args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MLXD_CHECK(cudaLaunchKernelExC(&cfg, kern, args));
    return 0;
}

int tp_sum(mlxd_model *m, const double *part, const uint16_t *res, uint16_t *out, int idx, cudaStream_t st,
           bool pdl) {
    TpState *t = (TpState *)m->tp;
    if (!t) {
        set_error("tensor parallel exchange used before tp_init");
        return -1;
    }
    TpPeers peers = t->peers;
    unsigned char *mine = t->mine;
    size_t ov = t->off_vec;
    int n = t->n, rank = t->rank, H = t->H, L2 = t->L2;
    int *err = t->err;
    const unsigned *seq = t->seq;
    void *args[] = {&peers, &mine, &ov, &n, &rank, &H, (void *)&part, (void *)&res, &out, (void *)&seq, &L2, &idx, &err};
    return launch_pdl(st, pdl, dim3(t->slices), dim3(TP_SLICE), (const void *)tp_sum_kernel, args);
}

int tp_send_args(mlxd_model *m, int idx, GemvArgs &a) {
    TpState *t = (TpState *)m->tp;
    if (!t) {
        set_error("tensor parallel exchange used before tp_init");
        return -1;
    }
    const int buf = idx & 1;
    for (int p = 0; p < t->n; p++)
        a.tp_line[p] = reinterpret_cast<uint32_t *>(t->peers.mb[p] + t->off_vec) + ((size_t)buf * t->n + t->rank) * t->H * 4;
    a.tp_n = t->n;
    a.tp_seq = t->seq;
    a.tp_mul = (unsigned)t->L2;
    a.tp_add = (unsigned)idx + 1u;
    return 0;
}

int tp_recv(mlxd_model *m, const uint16_t *res, uint16_t *out, int idx, cudaStream_t st, bool pdl) {
    TpState *t = (TpState *)m->tp;
    if (!t) {
        set_error("tensor parallel exchange used before tp_init");
        return -1;
    }
    const unsigned char *mine = t->mine;
    size_t ov = t->off_vec;
    int n = t->n, H = t->H, L2 = t->L2;
    int *err = t->err;
    const unsigned *seq = t->seq;
    void *args[] = {(void *)&mine, &ov, &n, &H, (void *)&res, &out, (void *)&seq, &L2, &idx, &err};
    return launch_pdl(st, pdl, dim3(t->slices), dim3(TP_SLICE), (const void *)tp_recv_kernel, args);
}

int tp_argmax(mlxd_model *m, unsigned long long *amax, int32_t *d_pos, int32_t *token, cudaStream_t st, bool pdl) {
    TpState *t = (TpState *)m->tp;
    if (!t) {
        set_error("tensor parallel exchange used before tp_init");
        return -1;
    }
    TpPeers peers = t->peers;
    unsigned char *mine = t->mine;
    size_t ok_ = t->off_key, of = t->off_kflag;
    int n = t->n, rank = t->rank;
    int *err = t->err;
    unsigned *seq = t->seq;
    void *args[] = {&peers, &mine, &ok_, &of, &n, &rank, &amax, &d_pos, &token, &seq, &err};
    return launch_pdl(st, pdl, dim3(1), dim3(32), (const void *)tp_argmax_kernel, args);
}

// the device step counter (advanced by the step's last kernel)
unsigned *tp_seq(mlxd_model *m) {
    TpState *t = (TpState *)m->tp;
    return t ? t->seq : nullptr;
}

// the full logits row (bf16 [V]) after tp_gather_logits
uint16_t *tp_full_logits(mlxd_model *m) {
    TpState *t = (TpState *)m->tp;
    return t ? reinterpret_cast<uint16_t *>(t->mine + t->off_log) : nullptr;
}

int tp_gather_logits(mlxd_model *m, const uint16_t *logits, cudaStream_t st, bool pdl) {
    TpState *t = (TpState *)m->tp;
    if (!t) {
        set_error("tensor parallel exchange used before tp_init");
        return -1;
    }
    TpPeers peers = t->peers;
    unsigned char *mine = t->mine;
    size_t ol = t->off_log, of = t->off_lflag;
    int n = t->n, rank = t->rank, Vl = t->V / t->n, vs = t->vslices;
    int *err = t->err;
    const unsigned *seq = t->seq;
    void *args[] = {&peers, &mine, &ol, &of, &n, &rank, &Vl, &vs, (void *)&logits, (void *)&seq, &err};
    return launch_pdl(st, pdl, dim3(vs), dim3(256), (const void *)tp_gather_logits_kernel, args);
}

// nonzero once an exchange gave up waiting for a peer (read and cleared)
int tp_timeouts(mlxd_model *m) {
    TpState *t = (TpState *)m->tp;
    if (!t) return 0;
    int v = 0, z = 0;
    if (cudaMemcpy(&v, t->err, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v) cudaMemcpy(t->err, &z, sizeof z, cudaMemcpyHostToDevice);
    return v;
}

}  // namespace mlxd
