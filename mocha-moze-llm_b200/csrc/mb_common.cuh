// Shared device helpers for the B200 (sm_100a) kernels of libmocha_b200.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#define MB_DEV __device__ __forceinline__

#define MB_CHECK(call)                                                                      \
    do {                                                                                    \
        cudaError_t mb_err_ = (call);                                                       \
        if (mb_err_ != cudaSuccess) {                                                       \
            fprintf(stderr, "CUDA %s: %d %s\n", #call, (int)mb_err_, cudaGetErrorString(mb_err_)); \
            return 1;                                                                       \
        }                                                                                   \
    } while (0)

namespace mb {

constexpr int kSMs = 148;  // B200: 2 dies x 74 SMs

MB_DEV float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Maximum over the warp in one instruction (sm_100a's floating-point redux): the
// result is one of the inputs, as a tree of fmaxf would give, but without five
// dependent shuffles.  NaN inputs are skipped, as fmaxf skips them.
MB_DEV float warp_max(float v)
{
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// Weights are read once per token: bypass L1 and give the L2 lines an evict-first
// policy so the stream does not push the KV cache and activations out of L2.
MB_DEV uint64_t evict_first_policy()
{
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

MB_DEV int4 ld_stream16(const void *ptr)
{
    int4 r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(ptr), "l"(evict_first_policy()));
    return r;
}

MB_DEV uint4 ld_stream16u(const void *ptr)
{
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(ptr), "l"(evict_first_policy()));
    return r;
}

MB_DEV uint2 ld_stream8(const void *ptr)
{
    uint2 r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
        : "=r"(r.x), "=r"(r.y)
        : "l"(ptr), "l"(evict_first_policy()));
    return r;
}

MB_DEV uint32_t ld_stream4(const void *ptr)
{
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(r) : "l"(ptr), "l"(evict_first_policy()));
    return r;
}

MB_DEV float ld_stream_f32(const float *ptr)
{
    float r;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(r) : "l"(ptr), "l"(evict_first_policy()));
    return r;
}

// Activations written by another CTA earlier in the same kernel sequence: read at L2.
MB_DEV float ld_cg(const float *p) { return __ldcg(p); }
MB_DEV float4 ld_cg4(const float4 *p) { return __ldcg(p); }

// Exact int8 -> fp32 for the four bytes of a word.  Each byte is biased to
// u = s + 128 (xor 0x80), placed in the low mantissa byte of 2^23 with one byte
// permute, and the bias removed with one exact float subtraction: the result is the
// integer s with no int->float conversion instruction.
MB_DEV float s8_lane(uint32_t biased, uint32_t selector)
{
    return __uint_as_float(__byte_perm(biased, 0x4B000000u, selector)) - 8388736.0f;
}

// sum_{k<16} w[k] * x[k] for 16 int8 weights packed in an int4 and 16 fp32 inputs.
MB_DEV float dot16_s8_f32(int4 w, const float *x)
{
    const uint32_t u[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u,
                           (uint32_t)w.z ^ 0x80808080u, (uint32_t)w.w ^ 0x80808080u};
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float4 xv = x4[i];
        acc = fmaf(s8_lane(u[i], 0x7540), xv.x, acc);
        acc = fmaf(s8_lane(u[i], 0x7541), xv.y, acc);
        acc = fmaf(s8_lane(u[i], 0x7542), xv.z, acc);
        acc = fmaf(s8_lane(u[i], 0x7543), xv.w, acc);
    }
    return acc;
}

// Deterministic block-wide sum; every CTA running the same code gets the same bits.
template <int THREADS>
MB_DEV float block_sum(float v, float *scratch /* >= THREADS/32 floats */)
{
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.f;
    if (warp == 0) {
        t = lane < THREADS / 32 ? scratch[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) scratch[0] = t;
    }
    __syncthreads();
    t = scratch[0];
    __syncthreads();
    return t;
}

// Orderable 64-bit key: larger value first, ties to the lower id.
MB_DEV unsigned long long rank_key(float v, int id)
{
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (uint32_t)(0x7fffffff - id);
}
MB_DEV float key_value(unsigned long long k)
{
    uint32_t b = (uint32_t)(k >> 32);
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    return __uint_as_float(b);
}
MB_DEV int key_id(unsigned long long k) { return 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu); }

}  // namespace mb
