// GGUF Q4_K / Q6_K / Q8_0 matrix-vector products on the int8 tensor cores
// (mma.sync m16n8k32 / m16n8k16) for the GGUF engine.
//
// Layout.  At load time every matrix is repacked into 16-row tiles whose quant bytes
// are already in the A-fragment order of the MMA, with exactly the file's bytes per
// weight; the block scales stay in their GGUF encoding beside them:
//   Q4_K, per (tile, 256-column block), 2,304 B: the 16 rows' 16-byte block headers
//     (d, dmin, 12 packed 6-bit scale/min bytes), then for each of the 8 sub-blocks of
//     32 columns and each lane l = 4g + t an 8-byte record: byte i (i < 4) holds the
//     nibbles of row g, columns 4t + i (low) and 16 + 4t + i (high); byte 4 + i the
//     same for row g + 8.  Unpacking is two masks and one shift per register.
//   Q6_K, per (tile, block), 3,360 B: for each pair of 16-column scale groups (32
//     columns) and lane, 8 bytes of low nibbles arranged as for Q4_K (2,048 B), then
//     4 bytes of the top two bits -- byte i: row g's bits at 4-5 (column 4t + i) and
//     6-7 (column 16 + 4t + i), row g + 8's at 0-1 and 2-3 (1,024 B); then the 16 rows'
//     16 int8 scales (256 B) and fp16 d (32 B).  Values are unsigned 0..63; the -32 of
//     the format is applied through the activation sums.
//   Q8_0, per tile: for each 32-column block and lane, the 16 int8 A-fragment bytes
//     (rows g, g + 8; columns 4t + i and 16 + 4t + i), then the 16 rows' fp16 d per block.
//
// Arithmetic.  The input vector (optionally RMS-normalised first, as in the reference's
// llama.cpp path) is split per 32 columns into a scale s = max|x|/127 and three int8
// limbs, x = s (a0 + a1/254 + a2/254^2) to within s/(2*254^2), which are the B
// fragment's columns 0..2.  The int32 products of one 32-column step (Q6_K: of each
// 16-column group) are exact; they are combined as (254 D0 + D1 + D2/254) * s/254 and
// the block's scales applied in fp32: Q4_K d*sc*(...) - dmin*m*sum(x) over the 32
// columns, Q6_K d*scale*(... - 32*sum of the limbs), Q8_0 d*(...).  Rows are tiles
// of 16; a CTA takes a contiguous range of tiles and its 16 warps split the CTA's
// (tile, 4-step batch) work evenly; per-warp row sums are added in warp order.
//
// Weight staging.  When a CTA's whole range fits in shared memory next to the input
// fragments (every per-layer GEMV of the two GGUF models: at most ~130 KB per CTA), its
// first thread copies the range into shared memory with bulk asynchronous copies
// (cp.async.bulk, completing on an mbarrier) before it waits for the kernel ahead --
// weights do not depend on it -- so the HBM stream of every CTA starts at once and runs
// while the input is being quantized; the warps then read their batches from shared
// memory.  Otherwise (the vocabulary head) each warp loads its batches from global
// memory into registers, keeping the next batch's loads in flight.
#include <algorithm>

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

#include "gguf_kernels.cuh"
#include "mb_common.cuh"

namespace gguf {
namespace {

constexpr int kThreads = 512, kWarps = kThreads / 32;
constexpr int kGrid = mb::kSMs;  // one CTA per SM (512 threads x ~100 registers)
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: v + kMagic rounds v to an integer (|v| < 2^22)
constexpr size_t kPrefetchBytes = 160 * 1024;  // per CTA: 148 CTAs x 160 KB = 24 MB of the 126 MB L2
constexpr size_t kSmemLimit = 220 * 1024;      // dynamic shared memory per CTA
constexpr int kMaxUnits = 3;                   // input units per thread: K <= 3 * 512 * 8 = 12,288

// fp16 bits -> fp32 (exact for every fp16 value)
MB_DEV float half_to_float(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu))); }

// Repacked Q4_K record of one (16-row tile, 256-column block), kQ4Rec bytes:
//   [0, 64)      per row r: d | dmin << 16 (the file's fp16 pair)
//   [64, 320)    per row r: the 8 sub-block scales, then the 8 sub-block mins, one byte
//                each, unpacked from the file's 6-bit fields (ggml's get_scale_min_k4)
//   [320, 2368)  per 32-column step: per lane 8 bytes of nibbles in mma fragment order
constexpr int kQ4Hdr = 64, kQ4Scales = 320, kQ4Rec = 2368;

// byte j & 3 of w as an integer (the upper bytes of the selector pick the zero word)
MB_DEV uint32_t byte_of(uint32_t w, int j) { return __byte_perm(w, 0u, 0x4440u | (uint32_t)(j & 3)); }

MB_DEV void mma_u8s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

MB_DEV void mma_s8s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint2 b)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b.x), "r"(b.y));
}

MB_DEV void mma_u8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b));
}

// limb combination (254 D0 + D1 + D2/254) of rows g (v0) and g + 8 (v1), valid in
// lanes with t == 0 (limb 2 comes from lane + 1)
MB_DEV void combine(const int (&d)[4], float &v0, float &v1)
{
    const int e0 = __shfl_down_sync(0xffffffffu, d[0], 1), e2 = __shfl_down_sync(0xffffffffu, d[2], 1);
    v0 = fmaf((float)e0, 1.f / 254.f, (float)(d[0] * 254 + d[1]));
    v1 = fmaf((float)e2, 1.f / 254.f, (float)(d[2] * 254 + d[3]));
}

// ---- repack ------------------------------------------------------------------------------

// Q4_K: one thread per (tile, block)
__global__ void k_repack_q4k_mma(const uint8_t *__restrict__ raw, int tiles, int nb, uint8_t *__restrict__ dst)
{
    const size_t n = (size_t)tiles * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / nb), b = (int)(i % nb);
        uint8_t *o = dst + i * kQ4Rec;
        const uint8_t *blk[16];
        for (int j = 0; j < 16; j++) blk[j] = raw + ((size_t)(16 * t + j) * nb + b) * 144;
        for (int j = 0; j < 16; j++) {
            for (int k = 0; k < 4; k++) o[4 * j + k] = blk[j][k];
            // 6-bit scale / min of sub-block u from the 12 scale bytes q = header bytes 4..15
            const uint8_t *q = blk[j] + 4;
            for (int u = 0; u < 8; u++) {
                uint8_t sc, mn;
                if (u < 4) {
                    sc = q[u] & 63;
                    mn = q[u + 4] & 63;
                } else {
                    sc = (uint8_t)((q[u + 4] & 15) | ((q[u - 4] >> 6) << 4));
                    mn = (uint8_t)((q[u + 4] >> 4) | ((q[u] >> 6) << 4));
                }
                o[kQ4Hdr + 16 * j + u] = sc;
                o[kQ4Hdr + 16 * j + 8 + u] = mn;
            }
        }
        // nibble q of column c (0..255) of a block: qs[32 (c / 64) + c % 32] >> 4 ((c / 32) & 1)
        auto q = [&](int j, int c) -> uint32_t {
            return (blk[j][16 + 32 * (c >> 6) + (c & 31)] >> (4 * ((c >> 5) & 1))) & 15u;
        };
        for (int s = 0; s < 8; s++)
            for (int l = 0; l < 32; l++) {
                const int g = l >> 2, tg = l & 3;
                uint8_t *r = o + kQ4Scales + s * 256 + l * 8;
                for (int ii = 0; ii < 4; ii++) {
                    const int c0 = 32 * s + 4 * tg + ii, c1 = c0 + 16;
                    r[ii] = (uint8_t)(q(g, c0) | (q(g, c1) << 4));
                    r[4 + ii] = (uint8_t)(q(g + 8, c0) | (q(g + 8, c1) << 4));
                }
            }
    }
}

// Q6_K: one thread per (tile, block); file blocks are 210 B (ql 128, qh 64, scales 16, d)
__global__ void k_repack_q6k_mma(const uint8_t *__restrict__ raw, int tiles, int nb, uint8_t *__restrict__ dst)
{
    const size_t n = (size_t)tiles * nb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / nb), b = (int)(i % nb);
        uint8_t *o = dst + i * 3360;
        const uint8_t *blk[16];
        for (int j = 0; j < 16; j++) blk[j] = raw + ((size_t)(16 * t + j) * nb + b) * 210;
        // 6-bit value (0..63) of column c of a block (src/gguf-cuda.cu dequantisation order)
        auto q = [&](int j, int c) -> uint32_t {
            const uint8_t *ql = blk[j], *qh = blk[j] + 128;
            const int nh = c >> 7, r = c & 127, quarter = r >> 5, l = r & 31;
            const uint32_t lo = quarter & 1 ? ql[64 * nh + l + 32] : ql[64 * nh + l];
            const uint32_t lo4 = quarter < 2 ? lo & 15u : lo >> 4;
            return lo4 | (((qh[32 * nh + l] >> (2 * quarter)) & 3u) << 4);
        };
        for (int p = 0; p < 8; p++)
            for (int l = 0; l < 32; l++) {
                const int g = l >> 2, tg = l & 3;
                uint8_t *lo = o + p * 256 + l * 8;
                uint8_t *hi = o + 2048 + p * 128 + l * 4;
                for (int ii = 0; ii < 4; ii++) {
                    const int c0 = 32 * p + 4 * tg + ii, c1 = c0 + 16;
                    const uint32_t a0 = q(g, c0), a2 = q(g, c1), a1 = q(g + 8, c0), a3 = q(g + 8, c1);
                    lo[ii] = (uint8_t)((a0 & 15u) | ((a2 & 15u) << 4));
                    lo[4 + ii] = (uint8_t)((a1 & 15u) | ((a3 & 15u) << 4));
                    hi[ii] = (uint8_t)(((a0 >> 4) << 4) | ((a2 >> 4) << 6) | (a1 >> 4) | ((a3 >> 4) << 2));
                }
            }
        for (int j = 0; j < 16; j++)
            for (int k = 0; k < 16; k++) o[3072 + 16 * j + k] = blk[j][192 + k];
        for (int j = 0; j < 16; j++) {
            o[3328 + 2 * j] = blk[j][208];
            o[3328 + 2 * j + 1] = blk[j][209];
        }
    }
}

// Q8_0: one thread per (tile, 32-column block); file blocks are 34 B (d, 32 int8)
__global__ void k_repack_q80_mma(const uint8_t *__restrict__ raw, int tiles, int ks, uint8_t *__restrict__ dst)
{
    const size_t n = (size_t)tiles * ks;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / ks), s = (int)(i % ks);
        uint8_t *tile = dst + (size_t)t * ks * 544;
        uint8_t *f = tile + (size_t)s * 512;
        uint8_t *dd = tile + (size_t)ks * 512 + s * 32;
        const uint8_t *blk[16];
        for (int j = 0; j < 16; j++) blk[j] = raw + ((size_t)(16 * t + j) * ks + s) * 34;
        for (int l = 0; l < 32; l++) {
            const int g = l >> 2, tg = l & 3;
            for (int ii = 0; ii < 4; ii++) {
                f[16 * l + ii] = blk[g][2 + 4 * tg + ii];
                f[16 * l + 4 + ii] = blk[g + 8][2 + 4 * tg + ii];
                f[16 * l + 8 + ii] = blk[g][2 + 16 + 4 * tg + ii];
                f[16 * l + 12 + ii] = blk[g + 8][2 + 16 + 4 * tg + ii];
            }
        }
        for (int j = 0; j < 16; j++) {
            dd[2 * j] = blk[j][0];
            dd[2 * j + 1] = blk[j][1];
        }
    }
}

// ---- the GEMV ----------------------------------------------------------------------------

// Shared memory of one CTA (cols = K): B fragments bf[K/32][32],
// per 32-column step the scale / 254 (sx) and the sum of x (x32), per 16-column group
// the limb sums (sa), and the per-warp row sums gp.
struct Lay {
    int cols, steps;
    size_t bf, sx, x32, sa, gp, bytes;
};

__host__ __device__ inline Lay layout(int cols, int max_tiles)
{
    Lay L;
    L.cols = cols;
    L.steps = cols / 32;
    L.bf = 0;
    L.sx = L.bf + (size_t)L.steps * 32 * 8;
    L.x32 = L.sx + (size_t)L.steps * 4;
    L.sa = L.x32 + (size_t)L.steps * 4;
    L.gp = L.sa + (size_t)(cols / 16) * 16;
    L.bytes = L.gp + (size_t)max_tiles * 16 * (kWarps + 1) * 4;
    return L;
}

// batches of 4 consecutive 32-column steps of one tile
constexpr int kBatch = 4;

struct Job {
    const uint8_t *body;
    int type;
    int tile;       // tile within its matrix
    int steps;      // 32-column steps per row
};

// Loads of one batch (all lanes), kept in registers until the batch is computed.
struct Batch {
    uint4 w[kBatch];     // Q4_K: nibble records (x, y); Q6_K: lo (x, y) + hi (z); Q8_0: fragments
    uint4 h0, h1;        // Q4_K sub-block scale / min bytes of rows g, g + 8; Q6_K scales of rows g, g + 8
    uint32_t dd[kBatch]; // Q4_K: d | dmin of rows g, g + 8; Q6_K: d of rows g (low 16) and g + 8
                         // (high 16); Q8_0: per step likewise
};

// plain loads from the staged shared-memory copy, or read-only / streaming global loads
template <bool S, typename T>
MB_DEV T ld_w(const void *p)
{
    return *reinterpret_cast<const T *>(p);
}
template <>
MB_DEV uint32_t ld_w<false, uint32_t>(const void *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
template <>
MB_DEV uint4 ld_w<false, uint4>(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
template <>
MB_DEV uint16_t ld_w<false, uint16_t>(const void *p) { return __ldg(reinterpret_cast<const uint16_t *>(p)); }
template <bool S>
MB_DEV uint2 ld_s8(const void *p)
{
    if constexpr (S) return *reinterpret_cast<const uint2 *>(p);
    else return mb::ld_stream8(p);
}
template <bool S>
MB_DEV uint32_t ld_s4(const void *p)
{
    if constexpr (S) return *reinterpret_cast<const uint32_t *>(p);
    else return mb::ld_stream4(p);
}
template <bool S>
MB_DEV uint4 ld_s16(const void *p)
{
    if constexpr (S) return *reinterpret_cast<const uint4 *>(p);
    else return mb::ld_stream16u(p);
}

template <bool S>
MB_DEV void load_batch(const Job &jb, int s0, int lane, Batch &B)
{
    const int g = lane >> 2;
    if (jb.type == Q4_K) {
        const int blk = s0 >> 3, nb = jb.steps >> 3;
        const uint8_t *rec = jb.body + ((size_t)jb.tile * nb + blk) * kQ4Rec;
        B.dd[0] = ld_w<S, uint32_t>(rec + 4 * g);
        B.dd[1] = ld_w<S, uint32_t>(rec + 4 * (g + 8));
        B.h0 = ld_w<S, uint4>(rec + kQ4Hdr + 16 * g);
        B.h1 = ld_w<S, uint4>(rec + kQ4Hdr + 16 * (g + 8));
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const uint2 v = ld_s8<S>(rec + kQ4Scales + ((s0 & 7) + k) * 256 + lane * 8);
            B.w[k] = make_uint4(v.x, v.y, 0u, 0u);
        }
    } else if (jb.type == Q6_K) {
        const int blk = s0 >> 3, nb = jb.steps >> 3;
        const uint8_t *rec = jb.body + ((size_t)jb.tile * nb + blk) * 3360;
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int p = (s0 & 7) + k;
            const uint2 v = ld_s8<S>(rec + p * 256 + lane * 8);
            const uint32_t hw = ld_s4<S>(rec + 2048 + p * 128 + lane * 4);
            B.w[k] = make_uint4(v.x, v.y, hw, 0u);
        }
        B.h0 = ld_w<S, uint4>(rec + 3072 + 16 * g);
        B.h1 = ld_w<S, uint4>(rec + 3072 + 16 * (g + 8));
        const uint8_t *dp = rec + 3328;
        B.dd[0] = (uint32_t)ld_w<S, uint16_t>(dp + 2 * g) | ((uint32_t)ld_w<S, uint16_t>(dp + 2 * (g + 8)) << 16);
    } else {
        const uint8_t *tile = jb.body + (size_t)jb.tile * jb.steps * 544;
        const uint8_t *dp = tile + (size_t)jb.steps * 512;
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            B.w[k] = ld_s16<S>(tile + (size_t)(s0 + k) * 512 + lane * 16);
            B.dd[k] = (uint32_t)ld_w<S, uint16_t>(dp + 2 * ((s0 + k) * 16 + g)) |
                      ((uint32_t)ld_w<S, uint16_t>(dp + 2 * ((s0 + k) * 16 + g + 8)) << 16);
        }
    }
}

MB_DEV uint32_t byte_u4(const uint4 &v, int n)
{
    const uint32_t w = n < 4 ? v.x : n < 8 ? v.y : n < 12 ? v.z : v.w;
    return (w >> (8 * (n & 3))) & 0xffu;
}

// The batch's MMAs, then its scale epilogue spread over the quad: lane t of each quad
// (rows g, g + 8) takes step s0 + t.  acc0 / acc1 gain that step's contribution to
// rows g / g + 8 (summed over the quad when the tile is done).
MB_DEV void run_batch(const Job &jb, int s0, int lane, const Batch &B, const uint2 *bf, const float *sx,
                      const float *x32, const int *sa, float &acc0, float &acc1)
{
    const int tg = lane & 3, src = lane & ~3;
    if (jb.type == Q6_K) {
        // two 16-column groups per step: values p[hh] of rows g / g + 8 for this lane's step
        float p0[2] = {0.f, 0.f}, p1[2] = {0.f, 0.f};
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int s = s0 + k;
            const uint2 b = bf[s * 32 + lane];
            const uint32_t w0 = B.w[k].x, w1 = B.w[k].y, h = B.w[k].z;
            const uint32_t a0 = (w0 & 0x0F0F0F0Fu) | (h & 0x30303030u);
            const uint32_t a2 = ((w0 >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
            const uint32_t a1 = (w1 & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
            const uint32_t a3 = ((w1 >> 4) & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                int e[4] = {0, 0, 0, 0};
                mma_u8s8_k16(e, hh ? a2 : a0, hh ? a3 : a1, hh ? b.y : b.x);
                // -32 per value: 32 * (sum of this lane's limb column over the group)
                const int grp = 2 * s + hh, c0 = 2 * tg, c1 = 2 * tg + 1;
                const int l0 = c0 < 3 ? sa[4 * grp + c0] : 0, l1 = c1 < 3 ? sa[4 * grp + c1] : 0;
                e[0] -= 32 * l0;
                e[1] -= 32 * l1;
                e[2] -= 32 * l0;
                e[3] -= 32 * l1;
                float v0, v1;
                combine(e, v0, v1);
                v0 = __shfl_sync(0xffffffffu, v0, src);
                v1 = __shfl_sync(0xffffffffu, v1, src);
                if (tg == k) {
                    p0[hh] = v0;
                    p1[hh] = v1;
                }
            }
        }
        const int s = s0 + tg, gi = 2 * (s & 7);
        const float dv0 = half_to_float(B.dd[0]), dv1 = half_to_float(B.dd[0] >> 16);
        const float f = sx[s];
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            acc0 += (dv0 * (float)(int8_t)byte_u4(B.h0, gi + hh)) * (p0[hh] * f);
            acc1 += (dv1 * (float)(int8_t)byte_u4(B.h1, gi + hh)) * (p1[hh] * f);
        }
        return;
    }
    if (jb.type == Q4_K) {
        // the 4 steps are 4 sub-blocks of one 256-column block, whose activation limbs
        // share one scale: the sub-block scales fold into int32 sums (|sum| <= 4 x 63 x
        // 32 x 15 x 127 < 2^31), the limbs are combined once per batch, and the mins take
        // sum_j m_j x32_j.  Lanes t = 0 hold limbs 0 and 1, lanes t = 1 limb 2; lane t = 0
        // of each quad accumulates rows g / g + 8.
        int T[4] = {0, 0, 0, 0};
        float mn0 = 0.f, mn1 = 0.f;
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int s = s0 + k, j = s & 7;
            const uint2 b = bf[s * 32 + lane];
            int d[4] = {0, 0, 0, 0};
            const uint32_t w0 = B.w[k].x, w1 = B.w[k].y;
            mma_u8s8_k32(d, w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu, (w1 >> 4) & 0x0F0F0F0Fu, b);
            const bool lo = j < 4;
            const int sc0 = (int)byte_of(lo ? B.h0.x : B.h0.y, j), sc1 = (int)byte_of(lo ? B.h1.x : B.h1.y, j);
            T[0] += sc0 * d[0];
            T[1] += sc0 * d[1];
            T[2] += sc1 * d[2];
            T[3] += sc1 * d[3];
            const float xs = x32[s];
            mn0 = fmaf((float)byte_of(lo ? B.h0.z : B.h0.w, j), xs, mn0);
            mn1 = fmaf((float)byte_of(lo ? B.h1.z : B.h1.w, j), xs, mn1);
        }
        // 254 T0 + T1 + T2 / 254 per row (T2 from lane t + 1)
        const int e0 = __shfl_down_sync(0xffffffffu, T[0], 1), e2 = __shfl_down_sync(0xffffffffu, T[2], 1);
        const float v0 = fmaf((float)e0, 1.f / 254.f, fmaf((float)T[0], 254.f, (float)T[1]));
        const float v1 = fmaf((float)e2, 1.f / 254.f, fmaf((float)T[2], 254.f, (float)T[3]));
        if (tg == 0) {
            const float f = sx[s0];
            const float d0 = half_to_float(B.dd[0]), dm0 = half_to_float(B.dd[0] >> 16);
            const float d1 = half_to_float(B.dd[1]), dm1 = half_to_float(B.dd[1] >> 16);
            acc0 += d0 * (v0 * f) - dm0 * mn0;
            acc1 += d1 * (v1 * f) - dm1 * mn1;
        }
        return;
    }
    float q0 = 0.f, q1 = 0.f;  // this lane's step: limb values of rows g / g + 8
#pragma unroll
    for (int k = 0; k < kBatch; k++) {
        const int s = s0 + k;
        const uint2 b = bf[s * 32 + lane];
        int d[4] = {0, 0, 0, 0};
        mma_s8s8_k32(d, B.w[k].x, B.w[k].y, B.w[k].z, B.w[k].w, b);
        float v0, v1;
        combine(d, v0, v1);
        v0 = __shfl_sync(0xffffffffu, v0, src);
        v1 = __shfl_sync(0xffffffffu, v1, src);
        if (tg == k) {
            q0 = v0;
            q1 = v1;
        }
    }
    const int s = s0 + tg;
    const float f = sx[s];
    {
        const uint32_t dd = tg == 0 ? B.dd[0] : tg == 1 ? B.dd[1] : tg == 2 ? B.dd[2] : B.dd[3];
        acc0 += half_to_float(dd) * (q0 * f);
        acc1 += half_to_float(dd >> 16) * (q1 * f);
    }
}

struct Gemv {
    MmaMat m[3];
    float *y[3];
    int tile_end[3];  // tiles of matrices 0..i together
    int n, cols, accumulate;
    const float *x, *gain, *up;  // up: the input is silu(x) * up (the SwiGLU of the FFN)
    float eps;
    int max_tiles;    // tiles per CTA at most (shared-memory row sums)
    size_t ring;      // staged: offset of the weight copy in dynamic shared memory
};

// Set when a staged GEMV's copy did not complete within its bound (read by the engine).
__device__ unsigned g_gemv_timeout;
constexpr long long kStageTimeoutCycles = 4000000000LL;

MB_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

template <bool Staged>
__global__ void __launch_bounds__(kThreads) k_gemv_mma(const Gemv g)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) unsigned long long stage_bar;
    const int total = g.tile_end[g.n - 1];
    const int t_begin = (int)((long long)total * blockIdx.x / gridDim.x);
    const int t_end = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
    const int steps = g.cols / 32;
    // this CTA's tiles of each matrix, [ra[i], rb[i]) in matrix i's own numbering, and
    // where their copy starts in the staged range
    int ra[3], rb[3];
    size_t roff[3];
    {
        size_t off = 0;
#pragma unroll
        for (int i = 0; i < 3; i++) {
            const int start = i ? g.tile_end[i - 1] : 0, end = i < g.n ? g.tile_end[i] : start;
            ra[i] = max(t_begin, start) - start;
            rb[i] = max(min(t_end, end) - start, ra[i]);
            roff[i] = off;
            if (i < g.n) off += (size_t)(rb[i] - ra[i]) * mma_tile_bytes(g.m[i].type, g.cols);
        }
    }
    if (Staged) {
        // the whole range into shared memory: bulk copies of at most 32 KB, all completing
        // on one mbarrier, started before the wait (nothing here depends on the kernel ahead)
        if (threadIdx.x == 0) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&stage_bar)) : "memory");
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            size_t bytes = 0;
#pragma unroll
            for (int i = 0; i < 3; i++)
                if (i < g.n) bytes += (size_t)(rb[i] - ra[i]) * mma_tile_bytes(g.m[i].type, g.cols);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&stage_bar)),
                         "r"((uint32_t)bytes)
                         : "memory");
            const uint64_t policy = mb::evict_first_policy();
#pragma unroll
            for (int i = 0; i < 3; i++) {
                if (i >= g.n) break;
                const size_t tb = mma_tile_bytes(g.m[i].type, g.cols);
                const uint8_t *src = g.m[i].body + (size_t)ra[i] * tb;
                uint8_t *dst = smem + g.ring + roff[i];
                for (size_t left = (size_t)(rb[i] - ra[i]) * tb; left > 0;) {
                    const uint32_t n = (uint32_t)(left < 32768 ? left : 32768);
                    asm volatile(
                        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
                        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
                        "l"(src), "r"(n), "r"(smem_u32(&stage_bar)), "l"(policy)
                        : "memory");
                    src += n;
                    dst += n;
                    left -= n;
                }
            }
        }
    } else if (threadIdx.x < g.n) {
        // this CTA's weight bytes into L2 while the kernel ahead finishes
        const int i = threadIdx.x, start = i ? g.tile_end[i - 1] : 0;
        const int a = max(t_begin, start), b = min(t_end, g.tile_end[i]);
        if (a < b) {
            const size_t tb = mma_tile_bytes(g.m[i].type, g.cols);
            const uint8_t *p0 = g.m[i].body + (size_t)(a - start) * tb;
            // at most kPrefetchBytes per CTA: a head larger than L2 would evict its own lines
            size_t left = (size_t)(b - a) * tb;
            left = left < kPrefetchBytes ? left : kPrefetchBytes;
            for (const uint8_t *q = p0; left > 0;) {
                const unsigned n = (unsigned)(left < 32768 ? left : 32768);
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(n) : "memory");
                q += n;
                left -= n;
            }
        }
    }
    // the warp's first batch of weights, loaded before the wait: weights do not depend on
    // the kernel ahead, so their latency overlaps the input staging below
    const int nt = t_end - t_begin, bpt = steps / kBatch, nbatch = nt * bpt;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = nbatch * warp / kWarps, b1 = nbatch * (warp + 1) / kWarps;
    auto job = [&](int tile_local) {
        const int tt = t_begin + tile_local;
        const int mi = tt < g.tile_end[0] ? 0 : (tt < g.tile_end[1] ? 1 : 2);
        Job j;
        j.type = g.m[mi].type;
        j.tile = tt - (mi ? g.tile_end[mi - 1] : 0);
        j.steps = steps;
        if (Staged) {  // the staged copy of matrix mi's range starts at its tile ra[mi]
            j.body = smem + g.ring + (mi == 0 ? roff[0] : mi == 1 ? roff[1] : roff[2]);
            j.tile -= mi == 0 ? ra[0] : mi == 1 ? ra[1] : ra[2];
        } else {
            j.body = g.m[mi].body;
        }
        return j;
    };
    int tl = b0 / bpt, s0 = (b0 - tl * bpt) * kBatch;
    Job jb = job(tl);
    Batch buf[2];
    if (!Staged && b0 < b1) load_batch<false>(jb, s0, lane, buf[0]);
    // the RMSNorm gain of this thread's columns does not depend on the kernel ahead
    // either (a normed input has at most 512 units: its K is the model width)
    float4 gv[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    if (g.gain && (int)threadIdx.x < steps * 4) {
        const int th = threadIdx.x;
        gv[0] = __ldg(reinterpret_cast<const float4 *>(g.gain + 32 * (th >> 2) + 4 * (th & 3)));
        gv[1] = __ldg(reinterpret_cast<const float4 *>(g.gain + 32 * (th >> 2) + 16 + 4 * (th & 3)));
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const Lay L = layout(g.cols, g.max_tiles);
    uint2 *bf = reinterpret_cast<uint2 *>(smem + L.bf);
    float *sx = reinterpret_cast<float *>(smem + L.sx);
    float *x32 = reinterpret_cast<float *>(smem + L.x32);
    int *sa = reinterpret_cast<int *>(smem + L.sa);
    float(*gp)[kWarps + 1] = reinterpret_cast<float(*)[kWarps + 1]>(smem + L.gp);
    __shared__ float red[kWarps];

    // input limbs: thread th = (s, t) owns columns 32 s + 16 h + 4 t + {0..3} for h = 0, 1,
    // B-fragment registers h of lanes 4 n + t (limb n); a warp covers one 256-column block
    // (8 steps), whose scale max|x| / 127 all its limbs share (one activation scale per
    // 256 columns, like the weights' super-blocks).  The values come straight from global
    // memory: silu(x) * up for the FFN down GEMV, x * (1/sqrt(sum x^2 / cols + eps)) * gain
    // for a normed input (the sum of squares by a block reduction first), else x.
    auto col_of = [&](int th, int h) { return 32 * (th >> 2) + 16 * h + 4 * (th & 3); };
    // every input value this thread quantizes (units th = tid + 512 e, e < kMaxUnits),
    // loaded with all requests in flight at once; the gain was loaded before the wait
    float4 xv[kMaxUnits][2], uv[kMaxUnits][2];
    const int units = steps * 4;
#pragma unroll
    for (int e = 0; e < kMaxUnits; e++) {
        const int th = threadIdx.x + e * kThreads;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            xv[e][h] = uv[e][h] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (th < units) {
                xv[e][h] = *reinterpret_cast<const float4 *>(g.x + col_of(th, h));
                if (g.up) uv[e][h] = *reinterpret_cast<const float4 *>(g.up + col_of(th, h));
            }
        }
    }
    float sc = 1.f;
    if (g.gain) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < kMaxUnits; e++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float4 v = xv[e][h];
                ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
            }
        ss = mb::warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) tot += red[w];
        sc = rsqrtf(tot / g.cols + g.eps);
    }
#pragma unroll
    for (int e = 0; e < kMaxUnits; e++) {
        const int th = threadIdx.x + e * kThreads;
        if (e * kThreads + (threadIdx.x & ~31) >= units) break;  // whole warps: units % 32 == 0
        const int s = th >> 2, tq = th & 3;
        float v[2][4];
        float m = 0.f, sum = 0.f;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float4 x = xv[e][h];
            if (g.up) {  // h = silu(gate) * up, as the reference's FFN
                const float4 u = uv[e][h];
                x = make_float4(__fdividef(x.x, 1.0f + expf(-x.x)) * u.x, __fdividef(x.y, 1.0f + expf(-x.y)) * u.y,
                                __fdividef(x.z, 1.0f + expf(-x.z)) * u.z, __fdividef(x.w, 1.0f + expf(-x.w)) * u.w);
            }
            if (g.gain) {
                const float4 gn = gv[h];
                x = make_float4(x.x * sc * gn.x, x.y * sc * gn.y, x.z * sc * gn.z, x.w * sc * gn.w);
            }
            v[h][0] = x.x;
            v[h][1] = x.y;
            v[h][2] = x.z;
            v[h][3] = x.w;
            m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            sum += (x.x + x.y) + (x.z + x.w);
        }
        // block max over the warp; step sum over its 4 threads
        m = mb::warp_max(m);
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float inv = m > 0.f ? __fdividef(127.f, m) : 0.f;
        uint32_t *bw = reinterpret_cast<uint32_t *>(&bf[s * 32]);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t b[3][4];
            int ls[3] = {0, 0, 0};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float q = v[h][j] * inv;
                const float t0 = __fadd_rn(q, kMagic), a0 = __fsub_rn(t0, kMagic);
                const float r1 = __fmul_rn(__fsub_rn(q, a0), 254.f);
                const float t1 = __fadd_rn(r1, kMagic), a1 = __fsub_rn(t1, kMagic);
                const float r2 = __fmul_rn(__fsub_rn(r1, a1), 254.f);
                const float t2 = __fadd_rn(r2, kMagic), a2 = __fsub_rn(t2, kMagic);
                b[0][j] = __float_as_uint(t0);
                b[1][j] = __float_as_uint(t1);
                b[2][j] = __float_as_uint(t2);
                ls[0] += (int)a0;
                ls[1] += (int)a1;
                ls[2] += (int)a2;
            }
            // limb sums of the 16-column group (s, h): the step's 4 threads
#pragma unroll
            for (int n = 0; n < 3; n++) {
                ls[n] += __shfl_xor_sync(0xffffffffu, ls[n], 1);
                ls[n] += __shfl_xor_sync(0xffffffffu, ls[n], 2);
            }
#pragma unroll
            for (int n = 0; n < 3; n++)
                bw[2 * (4 * n + tq) + h] =
                    __byte_perm(__byte_perm(b[n][0], b[n][1], 0x0040), __byte_perm(b[n][2], b[n][3], 0x0040), 0x5410);
            if (tq == 0) {
                const int grp = 2 * s + h;
                sa[4 * grp + 0] = ls[0];
                sa[4 * grp + 1] = ls[1];
                sa[4 * grp + 2] = ls[2];
                sa[4 * grp + 3] = 0;
            }
        }
        if (tq == 0) {
            sx[s] = m * (1.0f / (127.f * 254.f));
            x32[s] = sum;
        }
    }
    // B-fragment columns 3..7 (lanes 12..31) are zero
    for (int i = threadIdx.x; i < steps * 20; i += kThreads) bf[(i / 20) * 32 + 12 + i % 20] = make_uint2(0u, 0u);
    __syncthreads();
    if (Staged) {  // the weights have landed (bounded wait; the phase flips once)
        uint32_t done = 0;
        const long long t0 = clock64();
        while (!done) {
            asm volatile(
                "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(done)
                : "r"(smem_u32(&stage_bar))
                : "memory");
            if (!done && clock64() - t0 > kStageTimeoutCycles) break;
        }
        if (__syncthreads_or(!done)) {
            if (threadIdx.x == 0) atomicOr(&g_gemv_timeout, 1u);
            return;
        }
        if (b0 < b1) load_batch<true>(jb, s0, lane, buf[0]);
    }

    // batches (tile, 4 steps) of this CTA, split evenly over the warps; a warp walks its
    // range tile by tile, loading the next batch before computing the current one
    const int g8 = lane >> 2, tg = lane & 3;
    if (b0 < b1) {
        float acc0 = 0.f, acc1 = 0.f;
        // step: compute batch bi from buf[cur] after starting batch bi + 1 into buf[cur ^ 1]
        auto step = [&](int bi, Batch &cur, Batch &nxt) {
            int tln = tl, s0n = s0 + kBatch;
            if (s0n == steps) {
                tln = tl + 1;
                s0n = 0;
            }
            Job jn = jb;
            if (bi + 1 < b1) {
                if (tln != tl) jn = job(tln);
                load_batch<Staged>(jn, s0n, lane, nxt);
            }
            run_batch(jb, s0, lane, cur, bf, sx, x32, sa, acc0, acc1);
            if (bi + 1 == b1 || tln != tl) {
                // the quad's steps -> row sums in lane t == 0
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
                if (tg == 0) {
                    gp[16 * tl + g8][warp] = acc0;
                    gp[16 * tl + g8 + 8][warp] = acc1;
                }
                acc0 = acc1 = 0.f;
            }
            tl = tln;
            s0 = s0n;
            jb = jn;
        };
        for (int bi = b0; bi < b1; bi += 2) {
            step(bi, buf[0], buf[1]);
            if (bi + 1 < b1) step(bi + 1, buf[1], buf[0]);
        }
    }
    __syncthreads();
    // row sums: the warps whose batch ranges cover the row's tile, in warp order
    for (int r = threadIdx.x; r < nt * 16; r += kThreads) {
        const int tl = r >> 4;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
            const int wb0 = nbatch * w / kWarps, wb1 = nbatch * (w + 1) / kWarps;
            if (wb0 < wb1 && wb0 < (tl + 1) * bpt && wb1 > tl * bpt) sum += gp[r][w];
        }
        const int tt = t_begin + tl;
        const int mi = tt < g.tile_end[0] ? 0 : (tt < g.tile_end[1] ? 1 : 2);
        const int row = 16 * (tt - (mi ? g.tile_end[mi - 1] : 0)) + (r & 15);
        float *out = g.y[mi] + row;
        *out = g.accumulate ? *out + sum : sum;
    }
}

}  // namespace

int enqueue_repack_mma(int type, const uint8_t *raw, int rows, int cols, uint8_t *dst, cudaStream_t s)
{
    if (rows % 16 || !mma_tile_bytes(type, cols)) return 1;
    const int tiles = rows / 16;
    if (type == Q4_K)
        k_repack_q4k_mma<<<mb::kSMs * 4, 128, 0, s>>>(raw, tiles, cols / 256, dst);
    else if (type == Q6_K)
        k_repack_q6k_mma<<<mb::kSMs * 4, 128, 0, s>>>(raw, tiles, cols / 256, dst);
    else
        k_repack_q80_mma<<<mb::kSMs * 4, 128, 0, s>>>(raw, tiles, cols / 32, dst);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA gguf mma repack: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

int enqueue_gemv_mma(const MultiGemvMma &in, cudaStream_t s)
{
    Gemv g{};
    int tiles = 0;
    for (int i = 0; i < in.n; i++) {
        if (in.m[i].rows % 16 || in.m[i].cols != in.cols || !mma_tile_bytes(in.m[i].type, in.cols)) return 1;
        g.m[i] = in.m[i];
        g.y[i] = in.y[i];
        tiles += in.m[i].rows / 16;
        g.tile_end[i] = tiles;
    }
    // input units of 8 columns: at most kMaxUnits per thread, one when normed (the gain
    // of one unit is loaded before the wait)
    if (in.cols > kMaxUnits * kThreads * 8 || (in.gain && in.cols > kThreads * 8)) {
        fprintf(stderr, "gguf mma gemv: %d input columns exceed the kernel's staging\n", in.cols);
        return 1;
    }
    g.n = in.n;
    g.cols = in.cols;
    g.accumulate = in.accumulate;
    g.x = in.x;
    g.gain = in.gain;
    g.up = in.up;
    g.eps = in.eps;
    const int grid = tiles < kGrid ? tiles : kGrid;
    g.max_tiles = (tiles + grid - 1) / grid;
    const Lay L = layout(in.cols, g.max_tiles);
    if (L.bytes > kSmemLimit) return 1;
    // the largest CTA range (each CTA takes tiles [total c / grid, total (c+1) / grid))
    size_t range = 0;
    for (int c = 0; c < grid; c++) {
        const int tb = (int)((long long)tiles * c / grid), te = (int)((long long)tiles * (c + 1) / grid);
        size_t bytes = 0;
        for (int i = 0; i < in.n; i++) {
            const int start = i ? g.tile_end[i - 1] : 0;
            const int a = std::max(tb, start), b = std::min(te, g.tile_end[i]);
            if (a < b) bytes += (size_t)(b - a) * mma_tile_bytes(in.m[i].type, in.cols);
        }
        range = std::max(range, bytes);
    }
    g.ring = (L.bytes + 127) & ~(size_t)127;
    const bool staged = g.ring + range <= kSmemLimit;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(k_gemv_mma<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) !=
                cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_mma<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit) !=
                cudaSuccess)
            return 1;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = staged ? g.ring + range : L.bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e =
        staged ? cudaLaunchKernelEx(&cfg, k_gemv_mma<true>, g) : cudaLaunchKernelEx(&cfg, k_gemv_mma<false>, g);
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA gguf mma gemv: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

int gemv_take_timeout()
{
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_timeout, sizeof v) != cudaSuccess) return 1;
    if (!v) return 0;
    fprintf(stderr, "MOCHA_B200: a staged GGUF GEMV's weight copy did not complete (bounded wait expired)\n");
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_gemv_timeout, &zero, sizeof zero);
    return 1;
}

}  // namespace gguf
