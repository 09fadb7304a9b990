// tcgen05 GEMM with TMA-fed shared-memory ring and TMEM accumulator (see tc_gemm.cuh).
#include <stdio.h>

#include "mb_async.cuh"
#include "tc_gemm.cuh"

namespace mb {
namespace tc {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // bf16 elements per 128-byte swizzle row
constexpr int kThreads = 192;
constexpr uint32_t kABytes = kBM * kBK * 2;

template <int BN>
struct Cfg {
    static constexpr int stages = BN <= 64 ? 4 : (BN <= 128 ? 3 : 2);
    static constexpr uint32_t b_bytes = BN * kBK * 2;
    static constexpr uint32_t stage_bytes = 2 * kABytes + 2 * b_bytes;
    static constexpr uint32_t tmem_cols = BN < 32 ? 32 : BN;  // per accumulator buffer
    static constexpr size_t smem = 1024 + (size_t)stages * stage_bytes + 256;
};

MB_DEV void gemm_fail(int *err, volatile int *abort, int code)
{
    *abort = 1;
    atomicCAS(err, 0, code);
}

// Persistent form: gridDim.x CTAs walk the tiles (m fastest, then n, then split) in
// a static stride.  The TMA ring runs continuously across tiles; the accumulator is
// double-buffered in TMEM so the epilogue of one tile overlaps the MMAs of the next.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_bf16x3(const __grid_constant__ GemmParams p, int m_tiles,
                                                             int n_tiles, int tiles)
{
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + C::stages * C::stage_bytes);
    uint64_t *empty = full + C::stages;
    uint64_t *acc_full = empty + C::stages;  // [2]
    uint64_t *acc_empty = acc_full + 2;      // [2]
    uint64_t *drain = acc_empty + 2;         // MMA completion on the abort path
    uint32_t *tmem_slot = (uint32_t *)(drain + 1);
    volatile int *abort = (volatile int *)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ksteps_total = p.K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::stages; s++) {
            as::mbar_init(&full[s], 1);
            as::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            as::mbar_init(&acc_full[b], 1);
            as::mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
        }
        as::mbar_init(drain, 1);
        *abort = 0;
        as::fence_barrier_init();
    }
    if (warp == 1) as::tmem_alloc(tmem_slot, 2 * C::tmem_cols);
    as::tc_fence_before();
    __syncthreads();
    as::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // TMA producer: every k step of every tile of this CTA through the ring
        as::prefetch_map(&p.a_hi);
        as::prefetch_map(&p.a_lo);
        as::prefetch_map(&p.b_hi);
        as::prefetch_map(&p.b_lo);
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int mt = tile % m_tiles, nt = (tile / m_tiles) % n_tiles, z = tile / (m_tiles * n_tiles);
            const int ks0 = z * p.ksteps, nk = min(p.ksteps, ksteps_total - ks0);
            for (int k = 0; k < nk; k++, it++) {
                const int s = it % C::stages;
                if (it >= C::stages && !as::mbar_wait(&empty[s], ((it / C::stages) & 1) ^ 1, abort)) {
                    gemm_fail(p.err, abort, 11);
                    break;
                }
                uint8_t *st = smem + s * C::stage_bytes;
                as::mbar_expect_tx(&full[s], C::stage_bytes);
                const int kc = (ks0 + k) * kBK;
                as::tma_load_2d(st, &p.a_hi, kc, mt * kBM, &full[s]);
                as::tma_load_2d(st + kABytes, &p.a_lo, kc, mt * kBM, &full[s]);
                as::tma_load_2d(st + 2 * kABytes, &p.b_hi, kc, nt * BN, &full[s]);
                as::tma_load_2d(st + 2 * kABytes + C::b_bytes, &p.b_lo, kc, nt * BN, &full[s]);
            }
        }
        if (*abort) {
            // let the copies already in flight land before the CTA can exit
            const int first = it > C::stages ? it - C::stages : 0;
            for (int k = first; k < it; k++) {
                const volatile int never = 0;
                as::mbar_wait(&full[k % C::stages], (k / C::stages) & 1, &never);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        constexpr uint32_t idesc = as::idesc_bf16_f32(kBM, BN);
        int it = 0, local = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x, local++) {
            const int z = tile / (m_tiles * n_tiles);
            const int nk = min(p.ksteps, ksteps_total - z * p.ksteps);
            const int buf = local & 1;
            if (local >= 2 && !as::mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1, abort)) {
                gemm_fail(p.err, abort, 14);
                break;
            }
            as::tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(buf * C::tmem_cols);
            for (int k = 0; k < nk; k++, it++) {
                const int s = it % C::stages;
                if (!as::mbar_wait(&full[s], (it / C::stages) & 1, abort)) {
                    gemm_fail(p.err, abort, 12);
                    break;
                }
                as::tc_fence_after();
                const uint32_t a_hi = as::smem_u32(smem + s * C::stage_bytes);
                const uint32_t a_lo = a_hi + kABytes, b_hi = a_hi + 2 * kABytes, b_lo = b_hi + C::b_bytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; kk++) {
                    const uint32_t off = kk * 32;  // 16 bf16 along K inside the swizzled row
                    as::mma_bf16(acc, as::sw128_desc(a_hi + off), as::sw128_desc(b_hi + off), idesc, k > 0 || kk > 0);
                    as::mma_bf16(acc, as::sw128_desc(a_hi + off), as::sw128_desc(b_lo + off), idesc, true);
                    as::mma_bf16(acc, as::sw128_desc(a_lo + off), as::sw128_desc(b_hi + off), idesc, true);
                }
                as::mma_commit(&empty[s]);
            }
            as::mma_commit(&acc_full[buf]);
        }
        if (*abort) {
            // every issued MMA has finished with shared memory and TMEM
            as::mma_commit(drain);
            const volatile int never = 0;
            as::mbar_wait(drain, 0, &never);
        }
    } else if (warp >= 2) {
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
                if (!waited) gemm_fail(p.err, abort, 13);
                break;
            }
            const int n0 = nt * BN;
            const int m = mt * kBM + q * 32 + lane;
            float *d = p.d + (long long)z * p.split_stride + m;
            const int n_end = min(BN, p.N - n0);
            const uint32_t acc = tmem + (uint32_t)(buf * C::tmem_cols) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                if (c >= n_end) break;
                uint32_t r[16];
                as::tmem_ld16(acc + (uint32_t)c, r);
                as::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (c + j < n_end) d[(long long)(n0 + c + j) * p.ldd] = __uint_as_float(r[j]);
            }
            as::tc_fence_before();
            __syncwarp();
            if (lane == 0) as::mbar_arrive(&acc_empty[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        as::tc_fence_after();
        as::tmem_free(tmem, 2 * C::tmem_cols);
    }
}

__global__ void k_split_weights(const int8_t *__restrict__ q, const float *__restrict__ scales, size_t count,
                                __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        const float w = (float)q[i] * scales[i >> 6];
        split_bf16(w, hi[i], lo[i]);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)ptr;
    }
    return fn;
}

// Row-major bf16 [rows][K] with a box of {64, box_rows} and 128-byte swizzle.
int make_map(CUtensorMap *map, const void *base, long long rows, long long K, int box_rows)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        fprintf(stderr, "mocha: cuTensorMapEncodeTiled unavailable\n");
        return 1;
    }
    if (((uintptr_t)base & 15) || (K * 2) % 16 || K % kBK || box_rows < 1 || box_rows > 256) {
        fprintf(stderr, "mocha: bad tensor map geometry\n");
        return 1;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "mocha: cuTensorMapEncodeTiled failed (%d)\n", (int)r);
        return 1;
    }
    return 0;
}

template <int BN>
int setup_attr()
{
    static bool done = false;
    if (!done) {
        MB_CHECK(cudaFuncSetAttribute(k_gemm_bf16x3<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)Cfg<BN>::smem));
        done = true;
    }
    return 0;
}

}  // namespace

int make_map_bf16(CUtensorMap *map, const void *base, long long rows, long long inner, int box_rows)
{
    return make_map(map, base, rows, inner, box_rows);
}

int gemm_plan(Gemm *g, const __nv_bfloat16 *w_hi, const __nv_bfloat16 *w_lo, int M, int K,
              const __nv_bfloat16 *x_hi, const __nv_bfloat16 *x_lo, int n_max, float *d, long long ldd, int splits,
              int *err)
{
    if (M <= 0 || M % kBM || K <= 0 || K % kBK || n_max <= 0 || ldd < M) {
        fprintf(stderr, "mocha: gemm_plan: unsupported shape M=%d K=%d n=%d\n", M, K, n_max);
        return 1;
    }
    g->bn = n_max <= 64 ? 64 : 128;
    if (make_map(&g->p.a_hi, w_hi, M, K, kBM) || make_map(&g->p.a_lo, w_lo, M, K, kBM) ||
        make_map(&g->p.b_hi, x_hi, n_max, K, g->bn) || make_map(&g->p.b_lo, x_lo, n_max, K, g->bn))
        return 1;
    g->fixed_splits = splits > 0 ? splits : 0;
    g->p.d = d;
    g->p.ldd = ldd;
    g->p.split_stride = (long long)n_max * ldd;
    g->p.ksteps = K / kBK;
    g->p.M = M;
    g->p.N = n_max;
    g->p.K = K;
    g->p.err = err;
    g->smem = g->bn == 64 ? Cfg<64>::smem : Cfg<128>::smem;
    return g->bn == 64 ? setup_attr<64>() : setup_attr<128>();
}

Split gemm_split(const Gemm &g, int n)
{
    const int ksteps = g.p.K / kBK;
    const int tiles = (g.p.M / kBM) * ((n + g.bn - 1) / g.bn);
    // persistent CTAs: one wave of tiles is enough, more splits only add partial traffic
    int splits = g.fixed_splits > 0 ? g.fixed_splits : (kSMs + tiles - 1) / tiles;
    splits = splits < 1 ? 1 : (splits > ksteps ? ksteps : splits);
    const int per = (ksteps + splits - 1) / splits;
    return Split{(ksteps + per - 1) / per, (long long)n * g.p.ldd};
}

size_t gemm_partial_floats(const Gemm &g)
{
    size_t m = 0;
    for (int n = 1; n <= g.p.N; n++) {
        const Split s = gemm_split(g, n);
        const size_t f = (size_t)s.splits * (size_t)s.split_stride;
        m = f > m ? f : m;
    }
    return m;
}

int gemm_launch(const Gemm &g, int n, cudaStream_t s, Split *used)
{
    if (n <= 0 || n > g.p.N) {
        fprintf(stderr, "mocha: gemm_launch: n=%d outside 1..%d\n", n, g.p.N);
        return 1;
    }
    const Split sp = gemm_split(g, n);
    const int ksteps = g.p.K / kBK;
    GemmParams p = g.p;
    p.N = n;
    p.ksteps = (ksteps + sp.splits - 1) / sp.splits;
    p.split_stride = sp.split_stride;
    if (used) *used = sp;
    const int m_tiles = p.M / kBM, n_tiles = (n + g.bn - 1) / g.bn;
    const int tiles = m_tiles * n_tiles * sp.splits;
    const int grid = tiles < kSMs ? tiles : kSMs;
    if (g.bn == 64)
        k_gemm_bf16x3<64><<<grid, kThreads, g.smem, s>>>(p, m_tiles, n_tiles, tiles);
    else
        k_gemm_bf16x3<128><<<grid, kThreads, g.smem, s>>>(p, m_tiles, n_tiles, tiles);
    MB_CHECK(cudaGetLastError());
    return 0;
}

int split_weights(const int8_t *q, const float *scales, size_t count, __nv_bfloat16 *hi, __nv_bfloat16 *lo,
                  cudaStream_t s)
{
    k_split_weights<<<kSMs * 8, 256, 0, s>>>(q, scales, count, hi, lo);
    MB_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace tc
}  // namespace mb
