// Tensor-core (tcgen05) GEMM for the batched paths: prefill of a long prompt and
// decode of many sequences at once.
//
//   D[n][m] = sum_k W[m][k] * X[n][k]      W: grouped-Q8 weights, X: fp32 activations
//
// Both operands are carried as bf16 pairs: w = q*s = w_hi + w_lo and x = x_hi + x_lo
// with hi = bf16(v) and lo = bf16(v - hi), each pair holding about 17 significant
// bits.  The product is accumulated in fp32 TMEM from three bf16 MMAs per K slice:
// w_hi*x_hi + w_hi*x_lo + w_lo*x_hi (the dropped lo*lo term is below 2^-16 of the
// product).  The weight pairs are made once at load time (k_split_weights).
//
// Tiles: 128 weight rows (UMMA M) x BN activation rows (UMMA N) x 64 K per stage, fed
// by TMA with 128-byte swizzle through a STAGES-deep ring; one thread issues the MMAs
// into a TMEM accumulator of BN fp32 columns; four epilogue warps drain TMEM to global.
// The K range may be split over gridDim.z: split z writes its own partial tile to
// d + z*split_stride, and the consumer kernels sum the partials in a fixed order.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {
namespace tc {

struct GemmParams {
    CUtensorMap a_hi, a_lo;  // weights [M][K] bf16, box {64, 128}
    CUtensorMap b_hi, b_lo;  // activations [N][K] bf16, box {64, BN}
    float *d;                // partials [splits][N][ldd] fp32
    long long ldd;           // row stride of d in floats (>= M)
    long long split_stride;  // floats between split partials
    int M, N, K;             // M % 128 == 0, K % 64 == 0
    int ksteps;              // 64-wide K steps per split
    int *err;                // device error word: 0 ok, else the first failure code
};

// One GEMM call site: tensor maps for a fixed weight and a fixed activation buffer.
// The K split is chosen per launch from the row count; split s of a launch with n
// rows writes d + s * n * ldd.
struct Gemm {
    GemmParams p;
    int bn = 0;
    int fixed_splits = 0;  // > 0: always this many splits
    size_t smem = 0;
};

struct Split {
    int splits;              // partial tiles to sum, in order
    long long split_stride;  // floats between them (n * ldd)
};

// Split count and stride a launch with n rows uses.
Split gemm_split(const Gemm &g, int n);

// Largest splits * n * ldd over n in [1, n_max]: the partial-buffer size in floats.
size_t gemm_partial_floats(const Gemm &g);

// Builds a call site: weights `w_hi/w_lo` [M][K], activations `x_hi/x_lo` [n_max][K]
// (rows beyond the `n` given at launch are never read into results), output `d`.
// `splits` = 0 picks, per launch, a split count that fills the GPU.  Returns 0 on
// success.
int gemm_plan(Gemm *g, const __nv_bfloat16 *w_hi, const __nv_bfloat16 *w_lo, int M, int K,
              const __nv_bfloat16 *x_hi, const __nv_bfloat16 *x_lo, int n_max, float *d, long long ldd, int splits,
              int *err);

// Launches for the first `n` activation rows (n <= n_max).  `n` changes only the
// grid, never the tensor maps, so a plan can be reused inside a CUDA graph capture
// for a fixed n.
int gemm_launch(const Gemm &g, int n, cudaStream_t s, Split *used = nullptr);

// Tensor map of a row-major bf16 [rows][inner] array with boxes of {64, box_rows} and
// 128-byte swizzle (inner % 64 == 0).  Returns 0 on success.
int make_map_bf16(CUtensorMap *map, const void *base, long long rows, long long inner, int box_rows);

// Weights: bf16 pair of q*s for a grouped-Q8 matrix (int8 [M][K], fp32 scale per 64).
int split_weights(const int8_t *q, const float *scales, size_t count, __nv_bfloat16 *hi, __nv_bfloat16 *lo,
                  cudaStream_t s);

// Activations: bf16 pair of fp32 rows.
__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16 &hi, __nv_bfloat16 &lo)
{
    hi = __float2bfloat16_rn(v);
    lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}

}  // namespace tc
}  // namespace mb
