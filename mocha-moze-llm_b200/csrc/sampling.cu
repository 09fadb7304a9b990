// Candidate selection and sampling on the device.
//
// Semantics follow the reference: the repetition penalty divides positive and
// multiplies negative logits of each distinct id among the last 64 history tokens
// once (src/minimind.cu:142, src/minimind.cpp:160-164); ids >= 151643 except EOS are
// masked to -1e30 (src/minimind.cu:144); candidates are ordered by value with ties
// to the lower id (src/minimind.cu:154-156); the draw is the reference host's
// top-k / temperature / top-p / xorshift32 sampler (src/minimind.cpp:171-179).
//
// Unlike the reference's 64 interleaved partitions with k candidates each, the two
// stages here return the exact global top k; the union the reference returns always
// contains that set, so the host sampler sees the same candidates.
#include <float.h>
#include <math.h>
#include <string.h>

#include "mb_common.cuh"
#include "sampling.cuh"
#include "sampling_dev.cuh"

namespace sampling {
namespace {

constexpr int kSlice = 2048;  // ids per stage-1 CTA after padding (rows <= 148*2048)
constexpr int kThreads = 1024;

MB_DEV void bitonic_desc(unsigned long long *keys, int n /* power of two */)
{
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
                const int i = 2 * t - (t & (stride - 1));
                const int j = i + stride;
                const unsigned long long a = keys[i], b = keys[j];
                const bool desc = (i & size) == 0;
                if (desc ? (a < b) : (a > b)) {
                    keys[i] = b;
                    keys[j] = a;
                }
            }
            __syncthreads();
        }
    }
}

MB_DEV unsigned long long block_max_key(unsigned long long v, unsigned long long *red)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0ull;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
            v = w > v ? w : v;
        }
    }
    return v;  // valid in thread 0
}

__global__ void __launch_bounds__(kThreads)
    k_topk_stage1(const float *__restrict__ logits, int rows, const int *__restrict__ hist,
                  const int *__restrict__ count_ptr, const Params *__restrict__ prm,
                  unsigned long long *__restrict__ out)
{
    const float penalty = prm->penalty;
    const int k = min(max(prm->top_k, 1), kMaxK), eos = prm->eos, control_first = prm->control_first;
    __shared__ float vals[kSlice];
    __shared__ unsigned long long keys[kSlice];
    __shared__ unsigned long long red[32];
    const int slice = (rows + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * slice;
    const int n = max(0, min(rows, lo + slice) - lo);
    const int count = min(max(*count_ptr, 0), kHistory);
    for (int i = threadIdx.x; i < kSlice; i += blockDim.x) vals[i] = i < n ? logits[lo + i] : 0.f;
    __syncthreads();
    if (threadIdx.x < 32) {
        for (int j = threadIdx.x; j < count; j += 32) {
            const int id = hist[j];
            if (id < lo || id >= lo + n) continue;  // not in this slice: no duplicate scan
            bool dup = false;
            for (int t = 0; t < j; t++) dup |= hist[t] == id;
            if (!dup) {
                const float v = vals[id - lo];
                vals[id - lo] = v < 0 ? v * penalty : v / penalty;
            }
        }
    }
    __syncthreads();
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < kSlice; i += blockDim.x) {
        unsigned long long key = 0ull;
        if (i < n) {
            const int id = lo + i;
            float v = vals[i];
            if (id >= control_first && id != eos) v = -1e30f;
            key = mb::rank_key(v, id);
        }
        keys[i] = key;
        best = key > best ? key : best;
    }
    if (k == 1) {
        best = block_max_key(best, red);
        if (threadIdx.x == 0) out[blockIdx.x] = best;
        return;
    }
    __syncthreads();
    bitonic_desc(keys, kSlice);
    for (int r = threadIdx.x; r < k; r += blockDim.x) out[blockIdx.x * k + r] = keys[r];
}

__global__ void __launch_bounds__(kThreads)
    k_topk_stage2(const unsigned long long *__restrict__ in, const Params *__restrict__ prm,
                  unsigned long long *__restrict__ out)
{
    const int k = min(max(prm->top_k, 1), kMaxK), nin = kStage1Blocks * k;
    extern __shared__ unsigned long long skeys[];
    __shared__ unsigned long long red[32];
    if (k == 1) {
        unsigned long long best = 0ull;
        for (int i = threadIdx.x; i < nin; i += blockDim.x) best = in[i] > best ? in[i] : best;
        best = block_max_key(best, red);
        if (threadIdx.x == 0) out[0] = best;
        return;
    }
    int n = 1;
    while (n < nin) n <<= 1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) skeys[i] = i < nin ? in[i] : 0ull;
    __syncthreads();
    bitonic_desc(skeys, n);
    for (int r = threadIdx.x; r < k; r += blockDim.x) out[r] = skeys[r];
}

__global__ void k_sample(const unsigned long long *__restrict__ keys, const Params *__restrict__ prm, SeqState *st,
                         int *token_out, int *pos_inout, int *out_ring, int *out_count)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const Params p = *prm;
    uint32_t seed = st->seed;
    int token = draw_token(keys, p, seed);
    st->seed = seed;
    if (token < 0 || token >= p.vocab) token = p.eos >= 0 ? p.eos : 0;  // never index past the embedding
    record_token(token, p, st, out_ring, out_count);
    *token_out = token;
    if (pos_inout) (*pos_inout)++;
}

}  // namespace

constexpr int kMergeSmem = 16384 * (int)sizeof(unsigned long long);  // next power of two >= 148*64 keys

int init_device()
{
    const cudaError_t e =
        cudaFuncSetAttribute(k_topk_stage2, cudaFuncAttributeMaxDynamicSharedMemorySize, kMergeSmem);
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA top-k init: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

int enqueue_topk(const float *logits, int rows, const int *history, const int *count, const Params *p,
                 unsigned long long *scratch, unsigned long long *keys_out, cudaStream_t s)
{
    if (rows < 1 || rows > kStage1Blocks * kSlice) return 1;
    k_topk_stage1<<<kStage1Blocks, kThreads, 0, s>>>(logits, rows, history, count, p, scratch);
    k_topk_stage2<<<1, kThreads, kMergeSmem, s>>>(scratch, p, keys_out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA top-k launch: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

int enqueue_sample(const unsigned long long *keys, const Params *p, SeqState *st, int *token_out, int *pos_inout,
                   int *out_ring, int *out_count, cudaStream_t s)
{
    k_sample<<<1, 32, 0, s>>>(keys, p, st, token_out, pos_inout, out_ring, out_count);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA sample launch: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

float key_value_host(unsigned long long k)
{
    uint32_t b = (uint32_t)(k >> 32);
    b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

int key_id_host(unsigned long long k) { return 0x7fffffff - (int)(uint32_t)(k & 0xffffffffu); }

}  // namespace sampling
