// tcgen05 GEMM of grouped-Q8 weights converted on chip (see tc_w8gemm.cuh).
#include <stdio.h>

#include "mb_async.cuh"
#include "tc_w8gemm.cuh"

namespace mb {
namespace tw {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;                  // one weight group per stage
constexpr uint32_t kA8Bytes = kBM * kBK; // int8 weight tile
constexpr uint32_t kAHBytes = kBM * kBK * 2;
constexpr int kThreads = 320;            // producer, MMA, 4 converter warps, 4 epilogue warps

template <int BN>
struct Cfg {
    static constexpr int stages = BN >= 256 ? 2 : (BN >= 128 ? 3 : 4);
    static constexpr uint32_t b_bytes = BN * kBK * 2;
    static constexpr uint32_t stage_bytes = kA8Bytes + 2 * kAHBytes + 2 * b_bytes;
    static constexpr uint32_t tx_bytes = kA8Bytes + 2 * b_bytes;
    static constexpr uint32_t tmem_cols = 2 * BN;  // two accumulator buffers
    static constexpr size_t smem = 1024 + (size_t)stages * stage_bytes + 256;
};

MB_DEV void fail(int *err, volatile int *abort, int code)
{
    *abort = 1;
    atomicCAS(err, 0, code);
}

// byte offset of element (r, c) of a [rows][64] bf16 tile in the SW128 K-major layout
MB_DEV uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2); }

// exact float of each signed byte of a word, via the biased-byte trick
MB_DEV float s8f(uint32_t biased, uint32_t sel)
{
    return __uint_as_float(__byte_perm(biased, 0x4B000000u, sel)) - 8388736.0f;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_w8(const __grid_constant__ Params p, int m_tiles, int n_tiles,
                                                         int tiles)
{
    using Cf = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + Cf::stages * Cf::stage_bytes);
    uint64_t *conv = full + Cf::stages;
    uint64_t *empty = conv + Cf::stages;
    uint64_t *acc_full = empty + Cf::stages;  // [2]
    uint64_t *acc_empty = acc_full + 2;       // [2]
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = (uint32_t *)(drain + 1);
    volatile int *abort = (volatile int *)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kst_total = p.K / kBK, G = p.K / 64;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < Cf::stages; s++) {
            as::mbar_init(&full[s], 1);
            as::mbar_init(&conv[s], 4);
            as::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            as::mbar_init(&acc_full[b], 1);
            as::mbar_init(&acc_empty[b], 4);
        }
        as::mbar_init(drain, 1);
        *abort = 0;
        as::fence_barrier_init();
        // weights do not depend on the kernel ahead: start pulling the first tile into L2
        if ((int)blockIdx.x < tiles) {
            const int mt = blockIdx.x % m_tiles, z = blockIdx.x / (m_tiles * n_tiles);
            const int s0 = z * p.kstages, ns = min(p.kstages, kst_total - s0);
            for (int k = 0; k < ns && k < 16; k++) as::tma_prefetch_2d(&p.a, (s0 + k) * kBK, mt * kBM);
        }
    }
    if (warp == 1) as::tmem_alloc(tmem_slot, Cf::tmem_cols);
    as::tc_fence_before();
    __syncthreads();
    as::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    as::griddep_wait();  // activations and the partial buffer belong to earlier kernels

    if (warp == 0 && lane == 0) {
        // TMA producer
        as::prefetch_map(&p.a);
        as::prefetch_map(&p.b_hi);
        as::prefetch_map(&p.b_lo);
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int mt = tile % m_tiles, nt = (tile / m_tiles) % n_tiles, z = tile / (m_tiles * n_tiles);
            const int s0 = z * p.kstages, ns = min(p.kstages, kst_total - s0);
            for (int k = 0; k < ns; k++, it++) {
                const int s = it % Cf::stages;
                if (it >= Cf::stages && !as::mbar_wait(&empty[s], ((it / Cf::stages) & 1) ^ 1, abort)) {
                    fail(p.err, abort, 41);
                    break;
                }
                uint8_t *st = smem + s * Cf::stage_bytes;
                as::mbar_expect_tx(&full[s], Cf::tx_bytes);
                const int kc = (s0 + k) * kBK;
                as::tma_load_2d(st, &p.a, kc, mt * kBM, &full[s]);
                as::tma_load_2d(st + kA8Bytes + 2 * kAHBytes, &p.b_hi, kc, nt * BN, &full[s]);
                as::tma_load_2d(st + kA8Bytes + 2 * kAHBytes + Cf::b_bytes, &p.b_lo, kc, nt * BN, &full[s]);
            }
        }
        if (*abort) {
            const int first = it > Cf::stages ? it - Cf::stages : 0;
            for (int k = first; k < it; k++) {
                const volatile int never = 0;
                as::mbar_wait(&full[k % Cf::stages], (k / Cf::stages) & 1, &never);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: three bf16 products per 16-wide K slice, one accumulator per tile
        constexpr uint32_t idesc = as::idesc_bf16_f32(kBM, BN);
        int it = 0, local = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x, local++) {
            const int z = tile / (m_tiles * n_tiles);
            const int ns = min(p.kstages, kst_total - z * p.kstages);
            const int buf = local & 1;
            if (local >= 2 && !as::mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1, abort)) {
                fail(p.err, abort, 44);
                break;
            }
            const uint32_t acc = tmem + (uint32_t)(buf * BN);
            for (int k = 0; k < ns; k++, it++) {
                const int s = it % Cf::stages;
                if (!as::mbar_wait(&full[s], (it / Cf::stages) & 1, abort) ||
                    !as::mbar_wait(&conv[s], (it / Cf::stages) & 1, abort)) {
                    fail(p.err, abort, 42);
                    break;
                }
                as::tc_fence_after();
                const uint32_t base = as::smem_u32(smem + s * Cf::stage_bytes);
                const uint32_t a_hi = base + kA8Bytes, a_lo = a_hi + kAHBytes;
                const uint32_t b_hi = a_lo + kAHBytes, b_lo = b_hi + Cf::b_bytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; kk++) {
                    const uint32_t off = kk * 32;
                    as::mma_bf16(acc, as::sw128_desc(a_hi + off), as::sw128_desc(b_hi + off), idesc, k > 0 || kk > 0);
                    as::mma_bf16(acc, as::sw128_desc(a_hi + off), as::sw128_desc(b_lo + off), idesc, true);
                    as::mma_bf16(acc, as::sw128_desc(a_lo + off), as::sw128_desc(b_hi + off), idesc, true);
                }
                as::mma_commit(&empty[s]);
            }
            as::mma_commit(&acc_full[buf]);
        }
        if (*abort) {
            as::mma_commit(drain);
            const volatile int never = 0;
            as::mbar_wait(drain, 0, &never);
        }
    } else if (warp >= 2 && warp < 6) {
        // converters: thread r owns weight row r of the tile
        const int r = threadIdx.x - 64;
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int mt = tile % m_tiles, z = tile / (m_tiles * n_tiles);
            const int s0 = z * p.kstages, ns = min(p.kstages, kst_total - s0);
            const float *swr = p.sw + (size_t)(mt * kBM + r) * G + s0;
            float sc_next = __ldg(swr);
            for (int k = 0; k < ns; k++, it++) {
                const int s = it % Cf::stages;
                const float sc = sc_next;
                if (k + 1 < ns) sc_next = __ldg(swr + k + 1);
                const bool ok = as::mbar_wait(&full[s], (it / Cf::stages) & 1, abort);
                if (!__all_sync(0xffffffffu, ok)) {
                    if (!ok) fail(p.err, abort, 43);
                    break;
                }
                uint8_t *st = smem + s * Cf::stage_bytes;
                const int4 *row = reinterpret_cast<const int4 *>(st + r * kBK);
                uint8_t *ah = st + kA8Bytes, *al = ah + kAHBytes;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int cc = (c + r) & 3;  // rotate the 16-byte reads across rows
                    const int4 v = row[cc];
                    const uint32_t w4[4] = {(uint32_t)v.x ^ 0x80808080u, (uint32_t)v.y ^ 0x80808080u,
                                            (uint32_t)v.z ^ 0x80808080u, (uint32_t)v.w ^ 0x80808080u};
#pragma unroll
                    for (int h = 0; h < 2; h++) {  // 8 weights -> one 16-byte chunk of hi and of lo
                        __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            const int j = h * 8 + e;
                            const float w = s8f(w4[j >> 2], 0x7540u + (uint32_t)(j & 3)) * sc;
                            hi[e] = __float2bfloat16_rn(w);
                            lo[e] = __float2bfloat16_rn(w - __bfloat162float(hi[e]));
                        }
                        const uint32_t off = sw128_off(r, cc * 16 + h * 8);
                        *reinterpret_cast<uint4 *>(ah + off) = *reinterpret_cast<const uint4 *>(hi);
                        *reinterpret_cast<uint4 *>(al + off) = *reinterpret_cast<const uint4 *>(lo);
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) as::mbar_arrive(&conv[s]);
            }
        }
    } else if (warp >= 6) {
        // epilogue: TMEM lanes (warp % 4) * 32 .. +31 are weight rows of this warp
        const int q = warp & 3;
        int local = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, local++) {
            const int mt = tile % m_tiles, nt = (tile / m_tiles) % n_tiles, z = tile / (m_tiles * n_tiles);
            const int buf = local & 1;
            const bool waited = as::mbar_wait(&acc_full[buf], (local >> 1) & 1, abort);
            as::tc_fence_after();
            const bool ok = __all_sync(0xffffffffu, waited && !*abort);
            if (!ok) {
                if (!waited) fail(p.err, abort, 45);
                break;
            }
            const int n0 = nt * BN;
            const int m = mt * kBM + q * 32 + lane;
            float *d = p.d + (long long)z * p.split_stride + m;
            const int n_end = min(BN, p.N - n0);
            const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                if (c >= n_end) break;
                uint32_t rr[16];
                as::tmem_ld16(acc + (uint32_t)c, rr);
                as::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (c + j < n_end) d[(long long)(n0 + c + j) * p.ldd] = __uint_as_float(rr[j]);
            }
            as::tc_fence_before();
            __syncwarp();
            if (lane == 0) as::mbar_arrive(&acc_empty[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        as::tc_fence_after();
        as::tmem_free(tmem, Cf::tmem_cols);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// int8 [rows][K] with a box of {64, 128} and no swizzle (rows of 64 bytes)
int make_map_s8(CUtensorMap *map, const void *base, long long rows, long long K)
{
    static EncodeTiledFn enc = nullptr;
    if (!enc) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            enc = (EncodeTiledFn)ptr;
    }
    if (!enc || ((uintptr_t)base & 15) || K % kBK) {
        fprintf(stderr, "mocha: int8 weight tensor map unavailable or misaligned\n");
        return 1;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "mocha: cuTensorMapEncodeTiled (int8 weights) failed (%d)\n", (int)r);
        return 1;
    }
    return 0;
}

template <int BN>
int set_attr()
{
    static bool done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 1;
    if (!done[dev]) {
        MB_CHECK(cudaFuncSetAttribute(k_gemm_w8<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<BN>::smem));
        done[dev] = true;
    }
    return 0;
}

}  // namespace

int plan(Gemm *g, const int8_t *q, const float *sw, int M, int K, const __nv_bfloat16 *x_hi,
         const __nv_bfloat16 *x_lo, int n_max, float *d, long long ldd, int splits, int *err)
{
    if (M <= 0 || M % kBM || K <= 0 || K % kBK || n_max <= 0 || ldd < M) {
        fprintf(stderr, "mocha: converted-weight gemm plan: unsupported shape M=%d K=%d n=%d\n", M, K, n_max);
        return 1;
    }
    g->bn = n_max <= 64 ? 64 : (n_max <= 128 ? 128 : 256);
    if (make_map_s8(&g->p.a, q, M, K) || tc::make_map_bf16(&g->p.b_hi, x_hi, n_max, K, g->bn) ||
        tc::make_map_bf16(&g->p.b_lo, x_lo, n_max, K, g->bn))
        return 1;
    g->p.sw = sw;
    g->p.d = d;
    g->p.ldd = ldd;
    g->p.split_stride = (long long)n_max * ldd;
    g->p.M = M;
    g->p.N = n_max;
    g->p.K = K;
    g->p.kstages = K / kBK;
    g->p.err = err;
    g->n_max = n_max;
    g->fixed_splits = splits > 0 ? splits : 0;
    g->smem = g->bn == 64 ? Cfg<64>::smem : (g->bn == 128 ? Cfg<128>::smem : Cfg<256>::smem);
    return g->bn == 64 ? set_attr<64>() : (g->bn == 128 ? set_attr<128>() : set_attr<256>());
}

tc::Split split_for(const Gemm &g, int n)
{
    const int stages = g.p.K / kBK;
    const int tiles = (g.p.M / kBM) * ((n + g.bn - 1) / g.bn);
    int splits = g.fixed_splits > 0 ? g.fixed_splits : (kSMs + tiles - 1) / tiles;
    splits = splits < 1 ? 1 : (splits > stages ? stages : splits);
    const int per = (stages + splits - 1) / splits;
    return tc::Split{(stages + per - 1) / per, (long long)n * g.p.ldd};
}

size_t partial_floats(const Gemm &g)
{
    size_t m = 0;
    for (int n = 1; n <= g.n_max; n++) {
        const tc::Split s = split_for(g, n);
        const size_t f = (size_t)s.splits * (size_t)s.split_stride;
        m = f > m ? f : m;
    }
    return m;
}

int launch(const Gemm &g, int n, cudaStream_t s, tc::Split *used)
{
    if (n <= 0 || n > g.n_max) {
        fprintf(stderr, "mocha: converted-weight gemm launch: n=%d outside 1..%d\n", n, g.n_max);
        return 1;
    }
    const tc::Split sp = split_for(g, n);
    const int stages = g.p.K / kBK;
    Params p = g.p;
    p.N = n;
    p.kstages = (stages + sp.splits - 1) / sp.splits;
    p.split_stride = sp.split_stride;
    if (used) *used = sp;
    const int m_tiles = p.M / kBM, n_tiles = (n + g.bn - 1) / g.bn;
    const int tiles = m_tiles * n_tiles * sp.splits;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles < kSMs ? tiles : kSMs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (g.bn == 64)
        e = cudaLaunchKernelEx(&cfg, k_gemm_w8<64>, p, m_tiles, n_tiles, tiles);
    else if (g.bn == 128)
        e = cudaLaunchKernelEx(&cfg, k_gemm_w8<128>, p, m_tiles, n_tiles, tiles);
    else
        e = cudaLaunchKernelEx(&cfg, k_gemm_w8<256>, p, m_tiles, n_tiles, tiles);
    MB_CHECK(e);
    return 0;
}

}  // namespace tw
}  // namespace mb
