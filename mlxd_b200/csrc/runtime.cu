// Errors, tracked device memory, devices and streams (replaces
// src/mlxbridge/mlxbridge.c: gpu stream :6-8, synchronize :126-132, memory
// statistics :134-178).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <mutex>
#include <unordered_map>

#include "internal.h"

namespace mlxd {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return false;
}

static std::mutex g_mem_mu;
static std::unordered_map<void *, size_t> g_sizes;
static size_t g_active = 0, g_peak = 0;

void *dev_alloc(size_t bytes) {
    void *p = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        set_error("cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mem_mu);
    g_sizes[p] = bytes;
    g_active += bytes;
    if (g_active > g_peak) g_peak = g_active;
    return p;
}

void dev_free(void *p) {
    if (!p) return;
    {
        std::lock_guard<std::mutex> lk(g_mem_mu);
        auto it = g_sizes.find(p);
        if (it != g_sizes.end()) {
            g_active -= it->second;
            g_sizes.erase(it);
        }
    }
    cudaFree(p);
}

}  // namespace mlxd

using namespace mlxd;

#ifdef MLXD_TRACE
// timeline trace (instrumented builds only): one device buffer for every
// traced kernel, word 0 the record count, records of 4 words from word 4
namespace mlxd {
void trace_bind_sampler(unsigned long long *p);
void trace_bind_qgemv(unsigned long long *p);
void trace_bind_attention(unsigned long long *p);
void trace_bind_tp(unsigned long long *p);
}  // namespace mlxd
extern "C" void mlxd_trace_bind(unsigned long long *p) {
    mlxd::trace_bind_sampler(p);
    mlxd::trace_bind_qgemv(p);
    mlxd::trace_bind_attention(p);
    mlxd::trace_bind_tp(p);
}
#endif

extern "C" {

const char *mlxd_cuda_last_error(void) { return g_err; }

int mlxd_cuda_init(int device) {
    MLXD_CHECK(cudaSetDevice(device));
    MLXD_CHECK(cudaFree(nullptr));
    return 0;
}

int mlxd_cuda_device_count(int *n) {
    if (!n) return -1;
    int c = 0;
    MLXD_CHECK(cudaGetDeviceCount(&c));
    *n = c;
    return 0;
}

int mlxd_cuda_stream_create(void **stream) {
    if (!stream) return -1;
    cudaStream_t s;
    MLXD_CHECK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return 0;
}

int mlxd_cuda_stream_destroy(void *stream) {
    if (stream) MLXD_CHECK(cudaStreamDestroy((cudaStream_t)stream));
    return 0;
}

int mlxd_cuda_synchronize(void *stream) {
    if (stream) MLXD_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
    else MLXD_CHECK(cudaDeviceSynchronize());
    return 0;
}

int mlxd_cuda_alloc(void **dptr, size_t bytes) {
    if (!dptr) return -1;
    void *p = dev_alloc(bytes);
    if (!p) return -1;
    *dptr = p;
    return 0;
}

int mlxd_cuda_free(void *dptr) {
    dev_free(dptr);
    return 0;
}

int mlxd_cuda_upload(void *dst, const void *src, size_t bytes, void *stream) {
    MLXD_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    if (!stream) MLXD_CHECK(cudaStreamSynchronize(nullptr));
    return 0;
}

int mlxd_cuda_download(void *dst, const void *src, size_t bytes, void *stream) {
    MLXD_CHECK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    MLXD_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
    return 0;
}

int mlxd_cuda_memset(void *dst, int value, size_t bytes, void *stream) {
    MLXD_CHECK(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream));
    return 0;
}

size_t mlxd_cuda_active_memory(void) {
    std::lock_guard<std::mutex> lk(g_mem_mu);
    return g_active;
}

size_t mlxd_cuda_peak_memory(void) {
    std::lock_guard<std::mutex> lk(g_mem_mu);
    return g_peak;
}

}  // extern "C"
