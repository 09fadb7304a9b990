// tcgen05 int8 GEMM: grouped-Q8 weights x int8 activation limbs (see tc_q8gemm.cuh).
#include <stdio.h>

#include "mb_async.cuh"
#include "tc_q8gemm.cuh"

namespace mb {
namespace tq {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;                        // int8 K per stage (two groups of 64)
constexpr int kLimbRows = 3 * kTokens;          // 192 B rows
constexpr int kStages = 4;
constexpr uint32_t kABytes = kBM * kBK;         // 16 KiB
constexpr uint32_t kBBytes = kLimbRows * kBK;   // 24 KiB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kEpiWarps = 16;                   // four per TMEM lane quarter
constexpr int kEpiTokens = kTokens / (kEpiWarps / 4);  // tokens per epilogue warp
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kAccCols = kLimbRows;        // one group's int32 sums
constexpr uint32_t kTmemCols = 512;             // two accumulator buffers (384 used)
constexpr int kMaxGroups = 76;                  // groups of one split kept in shared memory (K <= 4864)
constexpr size_t kSxBytes = (size_t)kMaxGroups * kTokens * 4;
constexpr int kShLd = kTokens + 1;              // SwiGLU exchange tile [128 rows][64 tokens], padded
constexpr size_t kShBytes = (size_t)kBM * kShLd * 4;
constexpr size_t kSmemBase = 1024 + (size_t)kStages * kStageBytes + 256;
constexpr size_t kSmem = kSmemBase + kSxBytes + kShBytes;  // the largest launch

// Dynamic shared memory of one launch: the ring, the activation scales of one split's
// groups and, in SwiGLU mode, the exchange tile.  Sized per launch so that small
// launches leave room for the CTAs of the neighbouring kernels (programmatic dependent
// launch starts them on the same SMs).
size_t smem_bytes(const Params &p) { return kSmemBase + (size_t)2 * p.kstages * kTokens * 4 + (p.hq ? kShBytes : 0); }

// Two IEEE fp32 operations in one instruction (sm_100 paired FP32 lanes):
// (d0, d1) = (a0 * b0 + c0, a1 * b1 + c1), each rounded to nearest.
MB_DEV void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0, float c1)
{
    asm("{\n\t.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// (d0, d1) = (a0 * b0, a1 * b1), each rounded to nearest.
MB_DEV void mul2(float &d0, float &d1, float a0, float a1, float b0, float b1)
{
    asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

MB_DEV void fail(int *err, volatile int *abort, int code)
{
    *abort = 1;
    atomicCAS(err, 0, code);
}

__global__ void __launch_bounds__(kThreads, 1) k_gemm_q8(const __grid_constant__ Params p, int m_tiles, int n_tiles,
                                                          int tiles)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + kStages * kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *acc_full = empty + kStages;  // [2]
    uint64_t *acc_empty = acc_full + 2;    // [2]
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = (uint32_t *)(drain + 1);
    volatile int *abort = (volatile int *)(tmem_slot + 1);
    // activation scales of the current tile, [group of the split][token] / 254
    float *sxs = (float *)(smem + kStages * kStageBytes + 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stages_total = p.K / kBK, G = p.K / 64;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            as::mbar_init(&full[s], 1);
            as::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            as::mbar_init(&acc_full[b], 1);
            as::mbar_init(&acc_empty[b], kEpiWarps);
        }
        as::mbar_init(drain, 1);
        *abort = 0;
        as::fence_barrier_init();
    }
    as::griddep_launch();
    if (threadIdx.x == 32) {
        // weights do not depend on the kernel ahead: start pulling this CTA's first tile
        // into L2 while that kernel finishes
        const int tile = blockIdx.x;
        if (tile < tiles) {
            const int mt = tile % m_tiles, z = tile / (m_tiles * n_tiles);
            const int s0 = z * p.kstages, ns = min(p.kstages, stages_total - s0);
            for (int k = 0; k < ns && k < 8; k++) as::tma_prefetch_2d(&p.a, (s0 + k) * kBK, mt * kBM);
        }
    }
    if (warp == 1) as::tmem_alloc(tmem_slot, kTmemCols);
    as::tc_fence_before();
    __syncthreads();
    as::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    as::griddep_wait();  // activations, scales and the partial buffer belong to earlier kernels

    if (warp == 0 && lane == 0) {
        // TMA producer: every stage of every tile of this CTA through the ring
        as::prefetch_map(&p.a);
        as::prefetch_map(&p.b);
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int mt = tile % m_tiles, nt = (tile / m_tiles) % n_tiles, z = tile / (m_tiles * n_tiles);
            const int s0 = z * p.kstages, ns = min(p.kstages, stages_total - s0);
            for (int k = 0; k < ns; k++, it++) {
                const int s = it % kStages;
                if (it >= kStages && !as::mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, abort)) {
                    fail(p.err, abort, 21);
                    break;
                }
                uint8_t *st = smem + s * kStageBytes;
                as::mbar_expect_tx(&full[s], kStageBytes);
                const int kc = (s0 + k) * kBK;
                as::tma_load_2d(st, &p.a, kc, mt * kBM, &full[s]);
                as::tma_load_2d(st + kABytes, &p.b, kc, nt * kLimbRows, &full[s]);
            }
        }
        if (*abort) {
            const int first = it > kStages ? it - kStages : 0;
            for (int k = first; k < it; k++) {
                const volatile int never = 0;
                as::mbar_wait(&full[k % kStages], (k / kStages) & 1, &never);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: per group, two K = 32 MMAs into a fresh TMEM buffer
        constexpr uint32_t idesc = as::idesc_s8_s32(kBM, kLimbRows);
        int it = 0, grp = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const int z = tile / (m_tiles * n_tiles);
            const int ns = min(p.kstages, stages_total - z * p.kstages);
            for (int k = 0; k < ns && !*abort; k++, it++) {
                const int s = it % kStages;
                if (!as::mbar_wait(&full[s], (it / kStages) & 1, abort)) {
                    fail(p.err, abort, 22);
                    break;
                }
                const uint32_t a = as::smem_u32(smem + s * kStageBytes), b = a + kABytes;
                for (int gg = 0; gg < 2; gg++, grp++) {
                    const int buf = grp & 1;
                    if (grp >= 2 && !as::mbar_wait(&acc_empty[buf], ((grp >> 1) & 1) ^ 1, abort)) {
                        fail(p.err, abort, 24);
                        break;
                    }
                    as::tc_fence_after();
                    const uint32_t acc = tmem + (uint32_t)buf * kAccCols;
#pragma unroll
                    for (int kk = 0; kk < 2; kk++) {
                        const uint32_t off = gg * 64 + kk * 32;  // 32 int8 of K inside the swizzled row
                        as::mma_s8(acc, as::sw128_desc(a + off), as::sw128_desc(b + off), idesc, kk > 0);
                    }
                    as::mma_commit(&acc_full[buf]);
                }
                as::mma_commit(&empty[s]);
            }
        }
        if (*abort) {
            as::mma_commit(drain);
            const volatile int never = 0;
            as::mbar_wait(drain, 0, &never);
        }
    } else if (warp >= 2) {
        // epilogue: lane quarter warp % 4, tokens [kEpiTokens * part, +kEpiTokens) of the tile
        const int q = warp & 3, part = (warp - 2) >> 2, et = threadIdx.x - 64;
        // every epilogue warp walks all tiles and meets both named barriers of each, also
        // after an abort (waits then return at once), so no warp is left at a barrier
        int grp = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int mt = tile % m_tiles, nt = (tile / m_tiles) % n_tiles, z = tile / (m_tiles * n_tiles);
            const int s0 = z * p.kstages, ns = min(p.kstages, stages_total - s0), ng = 2 * ns;
            const int m = mt * kBM + q * 32 + lane;
            const int t0 = nt * kTokens + part * kEpiTokens;
            // stage this tile's activation scales (0 for rows past N), pre-divided by 254
            asm volatile("bar.sync 2, %0;" ::"n"(32 * kEpiWarps) : "memory");
            for (int i = et; i < ng * kTokens; i += 32 * kEpiWarps) {
                const int gi = i / kTokens, tok = nt * kTokens + i % kTokens;
                sxs[i] = tok < p.N ? __ldg(p.sx + (size_t)tok * G + 2 * s0 + gi) * (1.f / 254.f) : 0.f;
            }
            asm volatile("bar.sync 2, %0;" ::"n"(32 * kEpiWarps) : "memory");
            const float *swr = p.sw + (size_t)m * G + 2 * s0;
            float acc[kEpiTokens];
#pragma unroll
            for (int t = 0; t < kEpiTokens; t++) acc[t] = 0.f;
            for (int gi = 0; gi < ng; gi++, grp++) {
                const int buf = grp & 1;
                if (!ok) continue;
                const float sw = __ldg(swr + gi);
                const bool waited = as::mbar_wait(&acc_full[buf], (grp >> 1) & 1, abort);
                as::tc_fence_after();
                ok = __all_sync(0xffffffffu, waited && !*abort);
                if (!ok) {
                    if (!waited) fail(p.err, abort, 23);
                    continue;
                }
                uint32_t r[3 * kEpiTokens];
                const uint32_t base =
                    tmem + (uint32_t)buf * kAccCols + ((uint32_t)(q * 32) << 16) + part * 3 * kEpiTokens;
#pragma unroll
                for (int c = 0; c < 3 * kEpiTokens / 16; c++)
                    as::tmem_ld16(base + c * 16, *reinterpret_cast<uint32_t(*)[16]>(&r[c * 16]));
                as::tmem_wait_ld();
                as::tc_fence_before();
                __syncwarp();
                if (lane == 0) as::mbar_arrive(&acc_empty[buf]);
                const float4 *sx4 = reinterpret_cast<const float4 *>(sxs + gi * kTokens + part * kEpiTokens);
#pragma unroll
                for (int t4 = 0; t4 < kEpiTokens / 4; t4++) {
                    const float4 f = sx4[t4];
                    const float fs[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                    for (int e = 0; e < 4; e += 2) {
                        const int t = 4 * t4 + e;
                        // 254 * (D0 + D1/254 + D2/254^2) for tokens t, t + 1, the float work
                        // on paired FP32 lanes; D0*254 + D1 is exact in int32
                        float v0, v1, w0, w1;
                        const int da = (int)r[3 * t] * 254 + (int)r[3 * t + 1];
                        const int db = (int)r[3 * t + 3] * 254 + (int)r[3 * t + 4];
                        fma2(v0, v1, (float)(int)r[3 * t + 2], (float)(int)r[3 * t + 5], 1.f / 254.f, 1.f / 254.f,
                             (float)da, (float)db);
                        mul2(w0, w1, sw, sw, fs[e], fs[e + 1]);
                        fma2(acc[t], acc[t + 1], v0, v1, w0, w1, acc[t], acc[t + 1]);
                    }
                }
            }
            if (p.hq) {
                // SwiGLU: gate rows are tile rows 0..63, up rows 64..127; the 16 warps
                // exchange the tile through shared memory (every warp meets the barrier,
                // also after an abort), then warp e takes tokens 4e..4e+3 with lane l on
                // features 2l, 2l + 1 (one 64-group of the next GEMM per token)
                float *sh = sxs + 2 * p.kstages * kTokens;
                if (ok) {
#pragma unroll
                    for (int t = 0; t < kEpiTokens; t++) sh[(q * 32 + lane) * kShLd + part * kEpiTokens + t] = acc[t];
                }
                asm volatile("bar.sync 2, %0;" ::"n"(32 * kEpiWarps) : "memory");
                if (*abort) continue;
                const int ew = warp - 2;
#pragma unroll
                for (int i = 0; i < kTokens / kEpiWarps; i++) {
                    const int tl = (kTokens / kEpiWarps) * ew + i, tok = nt * kTokens + tl;
                    if (tok >= p.N) break;
                    const float g0 = sh[(2 * lane) * kShLd + tl], g1 = sh[(2 * lane + 1) * kShLd + tl];
                    const float u0 = sh[(64 + 2 * lane) * kShLd + tl], u1 = sh[(65 + 2 * lane) * kShLd + tl];
                    const float hv[2] = {(g0 / (1.f + expf(-g0))) * u0, (g1 / (1.f + expf(-g1))) * u1};
                    store_limbs<2, 32>(hv, p.hq + (size_t)tok * 3 * p.hk, p.hk, mt * 64 + 2 * lane,
                                       p.hs + (size_t)tok * (p.hk / 64) + mt, lane);
                }
                continue;
            }
            if (!ok) continue;
            float *d = p.d + (long long)z * p.split_stride + m;
#pragma unroll
            for (int t = 0; t < kEpiTokens; t++)
                if (t0 + t < p.N) d[(long long)(t0 + t) * p.ldd] = acc[t];
        }
    }
    __syncthreads();
    if (warp == 1) {
        as::tc_fence_after();
        as::tmem_free(tmem, kTmemCols);
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
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)ptr;
    }
    return fn;
}

// Row-major int8 [rows][K] with a box of {128, box_rows} and 128-byte swizzle.
int make_map(CUtensorMap *map, const void *base, long long rows, long long K, int box_rows)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        fprintf(stderr, "mocha: cuTensorMapEncodeTiled unavailable\n");
        return 1;
    }
    if (((uintptr_t)base & 15) || K % kBK || box_rows < 1 || box_rows > 256 || rows < 1) {
        fprintf(stderr, "mocha: bad int8 tensor map geometry\n");
        return 1;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "mocha: cuTensorMapEncodeTiled (int8) failed (%d)\n", (int)r);
        return 1;
    }
    return 0;
}

}  // namespace

int plan(Gemm *g, const int8_t *q, const float *sw, int M, int K, const int8_t *limbs, const float *sx, int n_max,
         float *d, long long ldd, int splits, int *err)
{
    if (M <= 0 || M % kBM || K <= 0 || K % kBK || K / 64 > kMaxGroups || n_max <= 0 || ldd < M) {
        fprintf(stderr, "mocha: int8 gemm plan: unsupported shape M=%d K=%d n=%d\n", M, K, n_max);
        return 1;
    }
    if (make_map(&g->p.a, q, M, K, kBM) || make_map(&g->p.b, limbs, 3LL * n_max, K, kLimbRows)) return 1;
    static bool attr = false;
    if (!attr) {
        MB_CHECK(cudaFuncSetAttribute(k_gemm_q8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
        attr = true;
    }
    g->p.sw = sw;
    g->p.sx = sx;
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
    return 0;
}

int set_swiglu(Gemm *g, int8_t *hq, float *hs, int hk)
{
    if (!hq || !hs || hk <= 0 || hk % 64 || g->p.M != 2 * hk) {
        fprintf(stderr, "mocha: int8 gemm swiglu: bad geometry (M=%d hk=%d)\n", g->p.M, hk);
        return 1;
    }
    g->p.hq = hq;
    g->p.hs = hs;
    g->p.hk = hk;
    g->fixed_splits = 1;
    return 0;
}

tc::Split split_for(const Gemm &g, int n)
{
    const int stages = g.p.K / kBK;
    const int tiles = (g.p.M / kBM) * ((n + kTokens - 1) / kTokens);
    // as many K splits as keep the tiles within one wave: a second partial wave would
    // add a tile's fixed costs (scale staging, output stores, a partial to reduce)
    // without shortening the longest CTA's K walk
    int splits = g.fixed_splits > 0 ? g.fixed_splits : kSMs / tiles;
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
        fprintf(stderr, "mocha: int8 gemm launch: n=%d outside 1..%d\n", n, g.n_max);
        return 1;
    }
    const tc::Split sp = split_for(g, n);
    const int stages = g.p.K / kBK;
    Params p = g.p;
    p.N = n;
    p.kstages = (stages + sp.splits - 1) / sp.splits;
    p.split_stride = sp.split_stride;
    if (used) *used = sp;
    const int m_tiles = p.M / kBM, n_tiles = (n + kTokens - 1) / kTokens;
    const int tiles = m_tiles * n_tiles * sp.splits;
    const int grid = tiles < kSMs ? tiles : kSMs;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes(p);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MB_CHECK(cudaLaunchKernelEx(&cfg, k_gemm_q8, p, m_tiles, n_tiles, tiles));
    return 0;
}

}  // namespace tq
}  // namespace mb
