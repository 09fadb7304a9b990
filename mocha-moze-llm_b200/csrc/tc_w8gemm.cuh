// tcgen05 GEMM of grouped-Q8 weights, converted on chip, against bf16-pair activations.
//
//   D[n][m] = sum_k (q[m][k] * s[m][k/64]) * x[n][k]
//
// The reference's int8 weights and fp32 scales stay in HBM as stored (1.06 B per
// weight).  Per 64-wide K stage, TMA brings the int8 weight tile and the activation
// tile (bf16 pair x = x_hi + x_lo, ~17 significant bits) into shared memory; four
// converter warps turn each weight row into w = q*s in fp32 and its bf16 pair
// w_hi + w_lo, written in the 128-byte-swizzled K-major layout; one thread issues the
// three products w_hi*x_hi + w_hi*x_lo + w_lo*x_hi into one fp32 TMEM accumulator for
// the whole K range, so the epilogue runs once per tile.  Tiles of 128 weight rows x
// 64/128/256 activation rows; persistent CTAs, double-buffered TMEM accumulators, K
// split per launch with ordered partials [split][n][ldd].
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tc_gemm.cuh"  // Split

namespace mb {
namespace tw {

struct Params {
    CUtensorMap a;          // int8 weights [M][K], box {64, 128}, no swizzle
    CUtensorMap b_hi, b_lo; // bf16 activations [n_max][K], box {64, BN}, 128-byte swizzle
    const float *sw;        // weight scales [M][K / 64]
    float *d;               // partials [splits][n][ldd]
    long long ldd, split_stride;
    int M, N, K;            // M % 128 == 0, K % 64 == 0
    int kstages;            // 64-wide K stages per split
    int *err;
};

struct Gemm {
    Params p;
    int bn = 0, n_max = 0, fixed_splits = 0;
    size_t smem = 0;
};

int plan(Gemm *g, const int8_t *q, const float *sw, int M, int K, const __nv_bfloat16 *x_hi,
         const __nv_bfloat16 *x_lo, int n_max, float *d, long long ldd, int splits, int *err);
tc::Split split_for(const Gemm &g, int n);
size_t partial_floats(const Gemm &g);
int launch(const Gemm &g, int n, cudaStream_t s, tc::Split *used = nullptr);

}  // namespace tw
}  // namespace mb
