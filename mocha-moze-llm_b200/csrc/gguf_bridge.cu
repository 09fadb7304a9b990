// mocha_gguf_matmul: the reference's GGUF quantised-matmul bridge
// (src/gguf-cuda.cu:110-144) on B200.
//
// Same contract as the reference: argument checks (type 8/12/14, cols % 256 == 0,
// 1 <= vectors <= 32, row bytes within 32 bits), host pointers in and out, byte
// strides, weights cached on the device keyed by (host pointer, size), one
// GGUF_CUDA_STATS line at exit, 1 on any error and no CPU fallback.  Differences: a
// B200 has room for every weight, so each matrix is uploaded once and kept resident
// in the 16-byte-aligned device layout (no 8 MiB streaming tile); the reference's
// MOCHA_GGUF_GPU_CACHE_MIB range check (0..256) is kept, and the value is reported.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <vector>

#include "gguf_kernels.cuh"
#include "mocha_gguf.h"

namespace {

struct Entry {
    const void *source;
    uint64_t bytes;
    uint8_t *device;
    gguf::DevMat mat;
};

struct Bridge {
    bool initialized = false;
    int device = 0;
    int cache_mib = 64;
    cudaStream_t stream = nullptr;
    std::vector<Entry> entries;
    float *d_x = nullptr, *d_y = nullptr, *h_x = nullptr, *h_y = nullptr;
    size_t x_cap = 0, y_cap = 0;
    uint8_t *d_raw = nullptr;
    size_t raw_cap = 0;
    unsigned long long calls = 0, uploads = 0, hits = 0, q4 = 0, q6 = 0, q8 = 0;
    uint64_t cached = 0;
    double upload_s = 0, compute_s = 0;
};

Bridge g_bridge;

double now_s()
{
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

int ck(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return 0;
    fprintf(stderr, "GGUF_CUDA_ERROR %s: %d %s\n", what, (int)e, cudaGetErrorString(e));
    return 1;
}
#define TRY(x)                          \
    do {                                \
        if (ck((x), #x)) return 1;      \
    } while (0)

void finish()
{
    Bridge &b = g_bridge;
    if (!b.initialized) return;
    fprintf(stderr,
            "GGUF_CUDA_STATS CALLS=%llu Q4_K=%llu Q6_K=%llu Q8_0=%llu CACHE_HITS=%llu UPLOAD_BYTES=%llu "
            "CACHE_BYTES=%llu TILE_BYTES=0 UPLOAD_S=%.6f COMPUTE_S=%.6f\n",
            b.calls, b.q4, b.q6, b.q8, b.hits, b.uploads, (unsigned long long)b.cached, b.upload_s, b.compute_s);
    cudaSetDevice(b.device);
    for (auto &e : b.entries) cudaFree(e.device);
    b.entries.clear();
    cudaFree(b.d_x);
    cudaFree(b.d_y);
    cudaFree(b.d_raw);
    cudaFreeHost(b.h_x);
    cudaFreeHost(b.h_y);
    if (b.stream) cudaStreamDestroy(b.stream);
    b.initialized = false;
}

int init()
{
    Bridge &b = g_bridge;
    if (b.initialized) return 0;
    const char *dev = getenv("MOCHA_DEVICE");
    b.device = dev ? atoi(dev) : 0;
    cudaDeviceProp prop;
    TRY(cudaGetDeviceProperties(&prop, b.device));
    if (prop.major != 10) {
        fprintf(stderr, "GGUF CUDA requires a compute capability 10.x (B200) device\n");
        return 1;
    }
    const char *value = getenv("MOCHA_GGUF_GPU_CACHE_MIB");
    const int mib = value ? atoi(value) : 64;
    if (mib < 0 || mib > 256) return 1;
    b.cache_mib = mib;
    TRY(cudaSetDevice(b.device));
    TRY(cudaStreamCreateWithFlags(&b.stream, cudaStreamNonBlocking));
    b.initialized = true;
    atexit(finish);
    fprintf(stderr, "GGUF_CUDA DEVICE=%s CACHE_LIMIT_MIB=%d RESIDENT_WEIGHTS=1 QUANTIZED_WEIGHTS=1\n", prop.name, mib);
    return 0;
}

template <typename T>
int reserve_dev(T **p, size_t *cap, size_t bytes)
{
    if (bytes <= *cap) return 0;
    if (*p) TRY(cudaFree(*p));
    *p = nullptr;
    *cap = 0;
    TRY(cudaMalloc((void **)p, bytes));
    *cap = bytes;
    return 0;
}

}  // namespace

extern "C" int mocha_gguf_matmul(int type, const void *w, int cols, int rows, const float *x, int vectors,
                                 unsigned x_stride, float *y, unsigned y_stride)
{
    if ((type != 8 && type != 12 && type != 14) || cols <= 0 || rows <= 0 || vectors < 1 || vectors > 32 ||
        cols % 256 || !w || !x || !y)
        return 1;
    if (init()) return 1;
    Bridge &b = g_bridge;
    TRY(cudaSetDevice(b.device));
    const unsigned row_bytes = gguf::row_bytes(type, cols);
    const uint64_t size = (uint64_t)row_bytes * rows;
    if (!row_bytes || size > 0xffffffffULL) return 1;

    const Entry *hit = nullptr;
    for (const auto &e : b.entries)
        if (e.source == w && e.bytes == size) {
            hit = &e;
            b.hits++;
            break;
        }
    double t0 = now_s();
    if (!hit) {
        uint8_t *dst = nullptr;
        TRY(cudaMalloc(&dst, size));
        int rc = 0;
        if (type == gguf::Q4_K) {
            rc = ck(cudaMemcpy(dst, w, size, cudaMemcpyHostToDevice), "cache upload");
        } else {
            rc = reserve_dev(&b.d_raw, &b.raw_cap, size) ||
                 ck(cudaMemcpy(b.d_raw, w, size, cudaMemcpyHostToDevice), "cache upload") ||
                 gguf::enqueue_repack(type, b.d_raw, rows, cols, dst, b.stream) ||
                 ck(cudaStreamSynchronize(b.stream), "repack");
        }
        if (rc) {
            cudaFree(dst);
            return 1;
        }
        b.entries.push_back(Entry{w, size, dst, gguf::make_devmat(type, rows, cols, dst)});
        b.cached += size;
        b.uploads += size;
        hit = &b.entries.back();
    }
    // stage x (strided host vectors) into pinned memory, one upload
    const size_t xb = (size_t)cols * vectors * sizeof(float), yb = (size_t)rows * vectors * sizeof(float);
    if (xb > b.x_cap) {
        if (b.h_x) cudaFreeHost(b.h_x);
        if (b.d_x) cudaFree(b.d_x);
        b.h_x = nullptr;
        b.d_x = nullptr;
        b.x_cap = 0;
        TRY(cudaMallocHost(&b.h_x, xb));
        TRY(cudaMalloc(&b.d_x, xb));
        b.x_cap = xb;
    }
    if (yb > b.y_cap) {
        if (b.h_y) cudaFreeHost(b.h_y);
        if (b.d_y) cudaFree(b.d_y);
        b.h_y = nullptr;
        b.d_y = nullptr;
        b.y_cap = 0;
        TRY(cudaMallocHost(&b.h_y, yb));
        TRY(cudaMalloc(&b.d_y, yb));
        b.y_cap = yb;
    }
    for (int v = 0; v < vectors; v++)
        memcpy(b.h_x + (size_t)v * cols, (const uint8_t *)x + (size_t)v * x_stride, (size_t)cols * 4);
    TRY(cudaMemcpyAsync(b.d_x, b.h_x, xb, cudaMemcpyHostToDevice, b.stream));
    b.upload_s += now_s() - t0;
    t0 = now_s();
    if (gguf::enqueue_gemv(hit->mat, b.d_x, vectors, cols, b.d_y, rows, b.stream)) return 1;
    TRY(cudaMemcpyAsync(b.h_y, b.d_y, yb, cudaMemcpyDeviceToHost, b.stream));
    TRY(cudaStreamSynchronize(b.stream));
    b.compute_s += now_s() - t0;
    for (int v = 0; v < vectors; v++)
        memcpy((uint8_t *)y + (size_t)v * y_stride, b.h_y + (size_t)v * rows, (size_t)rows * 4);
    b.calls++;
    if (type == gguf::Q4_K) b.q4++;
    else if (type == gguf::Q6_K) b.q6++;
    else b.q8++;
    return 0;
}

// Test hook: exact dequantisation of a cached matrix (same key as the matmul cache),
// written to a host buffer of rows*cols floats.  Not part of the reference ABI.
extern "C" int mocha_gguf_dequant(int type, const void *w, int cols, int rows, float *out)
{
    if ((type != 8 && type != 12 && type != 14) || cols <= 0 || rows <= 0 || !w || !out) return 1;
    if (init()) return 1;
    Bridge &b = g_bridge;
    TRY(cudaSetDevice(b.device));
    const unsigned row_bytes = gguf::row_bytes(type, cols);
    if (!row_bytes) return 1;
    const uint64_t size = (uint64_t)row_bytes * rows;
    uint8_t *raw = nullptr, *dst = nullptr;
    float *d_out = nullptr;
    int rc = ck(cudaMalloc(&raw, size), "malloc") || ck(cudaMalloc(&dst, size), "malloc") ||
             ck(cudaMalloc(&d_out, (size_t)rows * cols * 4), "malloc") ||
             ck(cudaMemcpy(raw, w, size, cudaMemcpyHostToDevice), "upload") ||
             gguf::enqueue_repack(type, raw, rows, cols, dst, b.stream);
    if (!rc) {
        const gguf::DevMat m = gguf::make_devmat(type, rows, cols, dst);
        rc = gguf::enqueue_dequant(m, d_out, b.stream) ||
             ck(cudaMemcpyAsync(out, d_out, (size_t)rows * cols * 4, cudaMemcpyDeviceToHost, b.stream), "copy") ||
             ck(cudaStreamSynchronize(b.stream), "sync");
    }
    cudaFree(raw);
    cudaFree(dst);
    cudaFree(d_out);
    return rc;
}
