// Self-contained check entry for the tcgen05 GEMM: one grouped-Q8 matrix times a
// batch of fp32 rows, through the same weight split, activation split, tensor maps
// and kernel the batched engine uses.  Allocates its own device buffers.
#include <stdio.h>
#include <vector>

#include "mb_common.cuh"
#include "mocha_b200.h"
#include "tc_gemm.cuh"
#include "tc_q8gemm.cuh"

namespace {

__global__ void k_split_rows(const float *__restrict__ x, size_t count, __nv_bfloat16 *hi, __nv_bfloat16 *lo)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        mb::tc::split_bf16(x[i], hi[i], lo[i]);
}

// one warp per (row, 64-group): two values per lane
__global__ void k_limbs(const float *__restrict__ x, int n, int cols, int8_t *limbs, float *scales)
{
    const int g = blockIdx.x, r = blockIdx.y, lane = threadIdx.x;
    const float v[2] = {x[(size_t)r * cols + g * 64 + 2 * lane], x[(size_t)r * cols + g * 64 + 2 * lane + 1]};
    mb::tq::store_limbs<2, 32>(v, limbs + (size_t)r * 3 * cols, cols, g * 64 + 2 * lane,
                               scales + (size_t)r * (cols / 64) + g, lane);
}

struct Buffers {
    std::vector<void *> ptrs;
    ~Buffers()
    {
        for (void *p : ptrs) cudaFree(p);
    }
    template <class T>
    T *alloc(size_t count)
    {
        void *p = nullptr;
        if (cudaMalloc(&p, count * sizeof(T) + 256) != cudaSuccess) return nullptr;
        ptrs.push_back(p);
        return (T *)p;
    }
};

}  // namespace

extern "C" int mocha_tc_gemm_check(int device, int rows, int n, int cols, const signed char *q, const float *scales,
                                   const float *x, float *y, int splits)
{
    if (rows <= 0 || rows % 128 || cols <= 0 || cols % 64 || n <= 0 || n > 1024 || !q || !scales || !x || !y) {
        fprintf(stderr, "mocha_tc_gemm_check: bad arguments\n");
        return 1;
    }
    MB_CHECK(cudaSetDevice(device));
    Buffers b;
    const size_t wn = (size_t)rows * cols, xn = (size_t)n * cols;
    int8_t *dq = b.alloc<int8_t>(wn);
    float *ds = b.alloc<float>(wn / 64), *dx = b.alloc<float>(xn);
    __nv_bfloat16 *whi = b.alloc<__nv_bfloat16>(wn), *wlo = b.alloc<__nv_bfloat16>(wn);
    __nv_bfloat16 *xhi = b.alloc<__nv_bfloat16>(xn), *xlo = b.alloc<__nv_bfloat16>(xn);
    int *err = b.alloc<int>(1);
    mb::tc::Gemm g;
    if (!dq || !ds || !dx || !whi || !wlo || !xhi || !xlo || !err) {
        fprintf(stderr, "mocha_tc_gemm_check: out of device memory\n");
        return 1;
    }
    MB_CHECK(cudaMemcpy(dq, q, wn, cudaMemcpyHostToDevice));
    MB_CHECK(cudaMemcpy(ds, scales, wn / 64 * 4, cudaMemcpyHostToDevice));
    MB_CHECK(cudaMemcpy(dx, x, xn * 4, cudaMemcpyHostToDevice));
    MB_CHECK(cudaMemset(err, 0, sizeof(int)));
    if (mb::tc::split_weights(dq, ds, wn, whi, wlo, 0)) return 1;
    k_split_rows<<<148 * 4, 256>>>(dx, xn, xhi, xlo);
    MB_CHECK(cudaGetLastError());
    // plan with the partial buffer sized after the split count is known
    if (mb::tc::gemm_plan(&g, whi, wlo, rows, cols, xhi, xlo, n, nullptr, rows, splits, err)) return 1;
    const mb::tc::Split sp = mb::tc::gemm_split(g, n);
    float *dp = b.alloc<float>((size_t)sp.splits * n * rows);
    if (!dp) return 1;
    g.p.d = dp;
    if (mb::tc::gemm_launch(g, n, 0)) return 1;
    MB_CHECK(cudaDeviceSynchronize());
    int herr = 0;
    MB_CHECK(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) {
        fprintf(stderr, "mocha_tc_gemm_check: kernel reported error %d\n", herr);
        return 1;
    }
    std::vector<float> part((size_t)sp.splits * n * rows);
    MB_CHECK(cudaMemcpy(part.data(), dp, part.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < (size_t)n * rows; i++) {
        float acc = 0.f;
        for (int s = 0; s < sp.splits; s++) acc += part[(size_t)s * n * rows + i];
        y[i] = acc;
    }
    return 0;
}

extern "C" int mocha_tq_gemm_check(int device, int rows, int n, int cols, const signed char *q, const float *scales,
                                   const float *x, float *y, int splits)
{
    if (rows <= 0 || rows % 128 || cols <= 0 || cols % 128 || n <= 0 || n > 1024 || !q || !scales || !x || !y) {
        fprintf(stderr, "mocha_tq_gemm_check: bad arguments\n");
        return 1;
    }
    MB_CHECK(cudaSetDevice(device));
    Buffers b;
    const size_t wn = (size_t)rows * cols, xn = (size_t)n * cols;
    int8_t *dq = b.alloc<int8_t>(wn), *dl = b.alloc<int8_t>(3 * xn);
    float *ds = b.alloc<float>(wn / 64), *dx = b.alloc<float>(xn), *dxs = b.alloc<float>(xn / 64);
    int *err = b.alloc<int>(1);
    if (!dq || !dl || !ds || !dx || !dxs || !err) {
        fprintf(stderr, "mocha_tq_gemm_check: out of device memory\n");
        return 1;
    }
    MB_CHECK(cudaMemcpy(dq, q, wn, cudaMemcpyHostToDevice));
    MB_CHECK(cudaMemcpy(ds, scales, wn / 64 * 4, cudaMemcpyHostToDevice));
    MB_CHECK(cudaMemcpy(dx, x, xn * 4, cudaMemcpyHostToDevice));
    MB_CHECK(cudaMemset(err, 0, sizeof(int)));
    k_limbs<<<dim3(cols / 64, n), 32>>>(dx, n, cols, dl, dxs);
    MB_CHECK(cudaGetLastError());
    mb::tq::Gemm g;
    if (mb::tq::plan(&g, dq, ds, rows, cols, dl, dxs, n, nullptr, rows, splits, err)) return 1;
    const mb::tc::Split sp = mb::tq::split_for(g, n);
    float *dp = b.alloc<float>((size_t)sp.splits * n * rows);
    if (!dp) return 1;
    g.p.d = dp;
    if (mb::tq::launch(g, n, 0)) return 1;
    MB_CHECK(cudaDeviceSynchronize());
    int herr = 0;
    MB_CHECK(cudaMemcpy(&herr, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) {
        fprintf(stderr, "mocha_tq_gemm_check: kernel reported error %d\n", herr);
        return 1;
    }
    std::vector<float> part((size_t)sp.splits * n * rows);
    MB_CHECK(cudaMemcpy(part.data(), dp, part.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < (size_t)n * rows; i++) {
        float acc = 0.f;
        for (int s = 0; s < sp.splits; s++) acc += part[(size_t)s * n * rows + i];
        y[i] = acc;
    }
    return 0;
}
