// tcgen05 int8 GEMM for grouped-Q8 weights against int8-limb activations.
//
//   D[n][m] = sum_g s_w[m][g] * s_x[n][g] * sum_{k in g} q[m][k] * x'[n][k]
//
// Weights are the reference's int8 matrices with one fp32 scale per 64 inputs, read as
// stored.  Each activation row x[n] is split per 64-group into a scale
// s_x = max|x|/127 and three int8 limbs, x = s_x * (a0 + a1/254 + a2/254^2) to within
// s_x * 0.5/254^2; the limbs are rows 3n, 3n+1, 3n+2 of the B operand.  For every
// group, two `tcgen05.mma.kind::i8` (K = 32) produce exact int32 sums
// D_limb[m][n] = sum_k q[m][k] * a_limb[n][k] in a fresh TMEM buffer; epilogue warps
// promote them, sum_limb D_limb * 254^-limb * s_w * s_x, into fp32 registers while the
// MMA thread fills the other TMEM buffer with the next group.
//
// Tiles: 128 weight rows x 64 activation rows (192 limb rows) x 128 K per stage (two
// groups), TMA with 128-byte swizzle, 4-stage ring; persistent CTAs walk
// (m tile, n tile, K split); split s writes d + s * n * ldd.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tc_gemm.cuh"  // Split

namespace mb {
namespace tq {

constexpr int kTokens = 64;  // activation rows per tile

struct Params {
    CUtensorMap a;        // int8 weights [M][K], box {128, 128}
    CUtensorMap b;        // int8 limbs [3 * n_max][K], box {128, 192}
    const float *sw;      // weight scales [M][K / 64]
    const float *sx;      // activation group scales [n_max][K / 64]
    float *d;             // partials [splits][n][ldd]
    long long ldd, split_stride;
    int M, N, K;          // M % 128 == 0, K % 128 == 0
    int kstages;          // 128-wide K stages per split
    int *err;
    // SwiGLU mode (hq set): the weight rows are gate and up interleaved in blocks of 64
    // (tile m holds gate rows 64m..64m+63, then up rows 64m..64m+63), K is not split,
    // and the epilogue writes h = silu(gate) * up of features 64m..64m+63 as the limbs
    // hq [3n][hk] and scales hs [n][hk / 64] of the next GEMM's input instead of d.
    int8_t *hq = nullptr;
    float *hs = nullptr;
    int hk = 0;
};

struct Gemm {
    Params p;
    int n_max = 0;
    int fixed_splits = 0;
};

// weights q [M][K] (int8, device), scales sw [M][K/64]; limbs [3*n_max][K] with scales
// sx [n_max][K/64]; output d with row stride ldd.  splits = 0: chosen per launch.
int plan(Gemm *g, const int8_t *q, const float *sw, int M, int K, const int8_t *limbs, const float *sx, int n_max,
         float *d, long long ldd, int splits, int *err);
// Switches a planned gate|up GEMM (M = 2 * hk rows, interleaved as in Params) to the
// SwiGLU epilogue writing limbs hq / scales hs.
int set_swiglu(Gemm *g, int8_t *hq, float *hs, int hk);
tc::Split split_for(const Gemm &g, int n);
size_t partial_floats(const Gemm &g);
int launch(const Gemm &g, int n, cudaStream_t s, tc::Split *used = nullptr);

// Limbs of one activation group held E values per thread by L consecutive lanes
// (L a power of two, lanes aligned to L): writes E bytes of each limb at
// limb0 + k, limb0 + K + k, limb0 + 2K + k and (lane 0 of the group) the scale.
template <int E, int L>
__device__ __forceinline__ void store_limbs(const float (&v)[E], int8_t *limb0, int K, int k, float *scale,
                                            int lane_in_group)
{
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < E; e++) m = fmaxf(m, fabsf(v[e]));
#pragma unroll
    for (int o = L / 2; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.f ? 127.f / m : 0.f;
    int8_t a[3][E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        const float q = v[e] * inv;
        const float a0 = fminf(fmaxf(rintf(q), -127.f), 127.f);
        const float r1 = (q - a0) * 254.f;
        const float a1 = fminf(fmaxf(rintf(r1), -127.f), 127.f);
        const float a2 = fminf(fmaxf(rintf((r1 - a1) * 254.f), -127.f), 127.f);
        a[0][e] = (int8_t)a0;
        a[1][e] = (int8_t)a1;
        a[2][e] = (int8_t)a2;
    }
#pragma unroll
    for (int l = 0; l < 3; l++) {
        int8_t *dst = limb0 + (size_t)l * K + k;
        if constexpr (E == 4) {
            *reinterpret_cast<char4 *>(dst) = make_char4(a[l][0], a[l][1], a[l][2], a[l][3]);
        } else if constexpr (E == 2) {
            *reinterpret_cast<char2 *>(dst) = make_char2(a[l][0], a[l][1]);
        } else if constexpr (E % 16 == 0) {  // dst 16-byte aligned
#pragma unroll
            for (int c = 0; c < E / 16; c++) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; i++)
                    w[i] = (uint32_t)(uint8_t)a[l][16 * c + 4 * i] | ((uint32_t)(uint8_t)a[l][16 * c + 4 * i + 1] << 8) |
                           ((uint32_t)(uint8_t)a[l][16 * c + 4 * i + 2] << 16) |
                           ((uint32_t)(uint8_t)a[l][16 * c + 4 * i + 3] << 24);
                *reinterpret_cast<uint4 *>(dst + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
#pragma unroll
            for (int e = 0; e < E; e++) dst[e] = a[l][e];
        }
    }
    if (lane_in_group == 0) *scale = m / 127.f;
}

}  // namespace tq
}  // namespace mb
