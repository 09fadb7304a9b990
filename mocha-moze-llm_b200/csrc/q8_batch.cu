// Batched grouped-Q8 engine: prompt prefill and multi-sequence decode on tcgen05
// GEMMs (tc_gemm.cuh), with attention, norms, RoPE, KV cache and sampling on the
// device.
//
// Every step processes a set of activation rows; row t carries (token, position,
// KV slot), so one pipeline serves a 1024-token prompt (one slot, positions
// 0..1023), the prompts of many sequences at once (rows of several slots), and one
// decode step of a batch (one row per slot).  Per layer:
//
//   norm+split -> QKV GEMM (q|k|v rows fused, 1152 x 896) -> bias + RoPE + KV write
//   -> attention (prompt blocks: key spans + span combine; decode rows: one kernel)
//   + split -> O GEMM -> residual + norm + split
//   -> gate|up GEMM (9728 x 896, rows interleaved per 64) with SwiGLU + split in its
//   epilogue (prompt passes) or in its own kernel (decode steps) -> down GEMM -> residual + norm (next layer, or the final norm of
//   projected rows)
//
// then the tied-embedding head GEMM for the projected rows and, in the token loop,
// the reference sampler for each projected row (penalty over the last 64 tokens,
// control mask, top-k / temperature / top-p / xorshift32; src/minimind.cpp:160-179).
// The math follows the reference CPU forward (src/minimind.cpp:51-82): RMSNorm
// y = x * (1/sqrt(sum x^2/896 + 1e-6)) * g, bias after the projection, split-half RoPE
// with the CPU's own powf/cosf/sinf tables, scores * 0.125 (applied to q, exact),
// softmax over positions 0..pos, SwiGLU g/(1+exp(-g))*u, residual adds.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "mb_common.cuh"
#include "mocha_b200.h"
#include "q8_decode.cuh"
#include "q8_layout.h"
#include "sampling.cuh"
#include "sampling_dev.cuh"
#include "tc_gemm.cuh"
#include "mb_async.cuh"
#include "tc_q8gemm.cuh"

namespace qb {

using namespace q8;
using bf16 = __nv_bfloat16;
using mb::tq::Gemm;

constexpr int QKV_ROWS = DIM + 2 * KV;  // q | k | v output rows of the fused projection
constexpr int GU_ROWS = 2 * HIDDEN;     // gate | up
constexpr int CHUNK = 64;               // keys per chunk of the block attention kernel
constexpr int NCHUNK = CONTEXT / CHUNK;
constexpr int PART = 2 + HEAD_DIM;      // chunk max, chunk sum, 64 weighted-V sums
constexpr int NT = DIM / 4;             // row kernels: 4 features per thread
constexpr int QKV_THREADS = (DIM + 2 * KV) / 2;  // one thread per RoPE pair / V pair
constexpr int SLICE = 8192;             // sampler stage 1: ids per CTA (keys in dynamic shared memory)
constexpr int NSLICE = (VOCAB + SLICE - 1) / SLICE;
constexpr int SAMPLE_THREADS = 1024;

// Every kernel of the batched pipeline is launched with programmatic stream
// serialisation: it lets the next kernel launch at once and waits for the previous
// one before it touches any activation.
MB_DEV void pdl_enter()
{
    mb::as::griddep_launch();
    mb::as::griddep_wait();
}

// KV cache: [slot][layer][kv head][position][64] fp32.
__host__ __device__ __forceinline__ size_t kv_off(int slot, int layer, int kvh, int pos)
{
    return ((((size_t)slot * LAYERS + layer) * KV_HEADS + kvh) * CONTEXT + pos) * HEAD_DIM;
}

struct Rows {
    const int *tok, *pos, *slot;
};

// bf16 pairs of the KV cache for the tensor-core prompt attention: K as
// [slot][layer][kv head][pos][64] (the fp32 cache's indexing) and V transposed as
// [slot][layer][kv head][64][pos].
struct KvShadow {
    bf16 *k_hi, *k_lo, *vt_hi, *vt_lo;
};

__host__ __device__ __forceinline__ size_t vt_off(int slot, int layer, int kvh, int d, int pos)
{
    return ((((size_t)slot * LAYERS + layer) * KV_HEADS + kvh) * HEAD_DIM + d) * CONTEXT + pos;
}

// ---- row kernels ----------------------------------------------------------------------

// Sum over K splits of a GEMM's partials, p[0] + p[stride] + p[2 stride] + ... in split
// order; the loads are issued several splits at a time so their latencies overlap.
MB_DEV float4 f4add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }

template <int B>
MB_DEV float4 sum_splits4(const float *p, int splits, long long stride)
{
    float4 acc = *reinterpret_cast<const float4 *>(p);
    for (int s = 1; s < splits; s += B) {
        float4 v[B];
#pragma unroll
        for (int j = 0; j < B; j++)
            if (s + j < splits) v[j] = *reinterpret_cast<const float4 *>(p + (s + j) * stride);
#pragma unroll
        for (int j = 0; j < B; j++)
            if (s + j < splits) acc = f4add(acc, v[j]);
    }
    return acc;
}

MB_DEV float sum_splits1(const float *p, int splits, long long stride)
{
    float acc = *p;
    for (int s = 1; s < splits; s += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (s + j < splits) v[j] = p[(s + j) * stride];
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (s + j < splits) acc += v[j];
    }
    return acc;
}

// Limbs of a DIM-wide GEMM input: int8 [rows * 3][DIM] and group scales [rows][DIM/64].
struct Limbs {
    int8_t *q;
    float *s;
};

// y = x * (1/sqrt(sum x^2 / DIM + eps)) * gain, stored as int8 limbs of row `dst`
// (16 lanes hold one 64-group).
MB_DEV void norm_store(const float (&v)[4], float *red, const float *__restrict__ gain, Limbs out, int dst)
{
    const float ss = mb::block_sum<NT>(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3], red);
    if (dst < 0) return;
    const float s = 1.f / sqrtf(ss / DIM + RMS_EPS);
    const int i0 = threadIdx.x * 4;
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; j++) y[j] = v[j] * s * __ldg(gain + i0 + j);
    mb::tq::store_limbs<4, 16>(y, out.q + (size_t)dst * 3 * DIM, DIM, i0, out.s + (size_t)dst * (DIM / GROUP) + i0 / GROUP,
                               threadIdx.x & 15);
}

// x[t] = dequant(embed[tok[t]]); xn[t] = split(rms(x[t]) * gain)
__global__ void __launch_bounds__(NT) k_embed_norm(Mat embed, Rows rows, const float *__restrict__ gain, float *x,
                                                   Limbs out)
{
    pdl_enter();
    __shared__ float red[32];
    const int t = blockIdx.x, i0 = threadIdx.x * 4;
    const int token = rows.tok[t];
    const char4 c = *reinterpret_cast<const char4 *>(embed.w + (size_t)token * DIM + i0);
    const float sc = embed.s[((size_t)token * DIM + i0) / GROUP];
    const float v[4] = {c.x * sc, c.y * sc, c.z * sc, c.w * sc};
    *reinterpret_cast<float4 *>(x + (size_t)t * DIM + i0) = make_float4(v[0], v[1], v[2], v[3]);
    norm_store(v, red, gain, out, t);
}

// x[t] += sum_s part[s][t]; then the norm of the new x into row dst_row[t] (or t).
// B: partial loads in flight per thread (20 for the many-split decode GEMMs: every
// partial of the down projection's 19 in one round of loads; 1 keeps the register
// count, and the occupancy of the prompt passes' thousands of rows, low).
template <int B>
__global__ void __launch_bounds__(NT) k_residual_norm(float *x, const float *__restrict__ part, int splits,
                                                      long long sstride, const float *__restrict__ gain, Limbs out,
                                                      const int *__restrict__ dst_row)
{
    pdl_enter();
    __shared__ float red[32];
    const int t = blockIdx.x, i0 = threadIdx.x * 4;
    const float4 acc = sum_splits4<B>(part + (size_t)t * DIM + i0, splits, sstride);
    float4 *xp = reinterpret_cast<float4 *>(x + (size_t)t * DIM + i0);
    const float4 xv = *xp;
    const float v[4] = {xv.x + acc.x, xv.y + acc.y, xv.z + acc.z, xv.w + acc.w};
    *xp = make_float4(v[0], v[1], v[2], v[3]);
    norm_store(v, red, gain, out, dst_row ? dst_row[t] : t);
}

// q/k/v = sum of partials + bias; split-half RoPE on q and k; q (times 0.125) to the
// query buffer, k and v to the KV cache at (slot, layer, pos).
__global__ void __launch_bounds__(QKV_THREADS) k_qkv_post(const float *__restrict__ part, int splits, long long sstride,
                                                          const float *__restrict__ bias, Rows rows,
                                                          const float *__restrict__ rope_cos,
                                                          const float *__restrict__ rope_sin, float *q, float *kc,
                                                          float *vc, int layer, KvShadow sh)
{
    pdl_enter();
    const int t = blockIdx.x, j = threadIdx.x;
    const int pos = rows.pos[t], slot = rows.slot[t];
    int kind, head, i;
    if (j < DIM / 2) {
        kind = 0;
        head = j / 32;
        i = j % 32;
    } else if (j < DIM / 2 + KV / 2) {
        kind = 1;
        head = (j - DIM / 2) / 32;
        i = (j - DIM / 2) % 32;
    } else {
        kind = 2;
        head = (j - DIM / 2 - KV / 2) / 32;
        i = (j - DIM / 2 - KV / 2) % 32;
    }
    const int r0 = (kind == 0 ? 0 : kind == 1 ? DIM : DIM + KV) + head * HEAD_DIM + i;
    const float *p = part + (size_t)t * QKV_ROWS;
    float d0 = p[r0], d1 = p[r0 + 32];
    for (int s = 1; s < splits; s++) {
        d0 += p[s * sstride + r0];
        d1 += p[s * sstride + r0 + 32];
    }
    d0 += __ldg(bias + r0);
    d1 += __ldg(bias + r0 + 32);
    if (kind == 2) {
        float *v = vc + kv_off(slot, layer, head, pos);
        v[i] = d0;
        v[i + 32] = d1;
        mb::tc::split_bf16(d0, sh.vt_hi[vt_off(slot, layer, head, i, pos)], sh.vt_lo[vt_off(slot, layer, head, i, pos)]);
        mb::tc::split_bf16(d1, sh.vt_hi[vt_off(slot, layer, head, i + 32, pos)],
                           sh.vt_lo[vt_off(slot, layer, head, i + 32, pos)]);
        return;
    }
    const float cs = __ldg(rope_cos + pos * 32 + i), sn = __ldg(rope_sin + pos * 32 + i);
    const float a = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
    const float b = __fadd_rn(__fmul_rn(d1, cs), __fmul_rn(d0, sn));
    if (kind == 0) {
        q[(size_t)t * DIM + head * HEAD_DIM + i] = a * 0.125f;
        q[(size_t)t * DIM + head * HEAD_DIM + i + 32] = b * 0.125f;
    } else {
        const size_t o = kv_off(slot, layer, head, pos);
        kc[o + i] = a;
        kc[o + i + 32] = b;
        mb::tc::split_bf16(a, sh.k_hi[o + i], sh.k_lo[o + i]);
        mb::tc::split_bf16(b, sh.k_hi[o + i + 32], sh.k_lo[o + i + 32]);
    }
}

// Combine the key spans of (row, head) pairs into the attention output, as limbs for
// the O GEMM: one warp per pair, two dims per lane (the head is one 64-group), kCombWarps
// pairs per CTA (one-warp CTAs left the SMs at half their warps: an SM holds at most 32
// CTAs), the spans' partials loaded before the first use (at most kCombSpans of `per`
// keys each).
constexpr int kCombWarps = 8;
template <int kCombSpans>
__global__ void __launch_bounds__(32 * kCombWarps) k_attn_combine(const float *__restrict__ part, Rows rows, Limbs out,
                                                                   int per, int n)
{
    pdl_enter();
    const int pair = blockIdx.x * kCombWarps + (int)(threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (pair >= n * HEADS) return;  // whole warps
    const int t = pair / HEADS, h = pair % HEADS, d = 2 * lane;
    if (rows.pos[t] < per) return;  // one span: k_attn_tc wrote the row's limbs
    const int nc = min(rows.pos[t] / per + 1, kCombSpans);  // partials of `per` keys each
    const float *p = part + ((size_t)t * HEADS + h) * NCHUNK * PART;
    float pm[kCombSpans], pl[kCombSpans], pa[kCombSpans], pb[kCombSpans];
#pragma unroll
    for (int c = 0; c < kCombSpans; c++) {
        const bool in = c < nc;
        pm[c] = in ? p[c * PART] : -INFINITY;
        pl[c] = in ? p[c * PART + 1] : 0.f;
        pa[c] = in ? p[c * PART + 2 + d] : 0.f;
        pb[c] = in ? p[c * PART + 3 + d] : 0.f;
    }
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < kCombSpans; c++)
        if (c < nc) m = fmaxf(m, pm[c]);
    float l = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int c = 0; c < kCombSpans; c++)
        if (c < nc) {
            const float w = expf(pm[c] - m);
            l += pl[c] * w;
            a0 += pa[c] * w;
            a1 += pb[c] * w;
        }
    const float v[2] = {a0 / l, a1 / l};
    mb::tq::store_limbs<2, 32>(v, out.q + (size_t)t * 3 * DIM, DIM, h * HEAD_DIM + d,
                               out.s + (size_t)t * (DIM / GROUP) + h, lane);
}

// Rows of any shape: the attention of one row (one query position) for one KV head
// and the GQA query heads that share it, over keys 0..pos, written as limbs for the O
// GEMM.  One CTA of 256 threads per (KV head, row):
//   post    (kPost, rows of distinct slots such as decode steps) the head's q (7 x 64),
//           k and v from the QKV GEMM partials exactly as k_qkv_post computes them
//           (split sum, bias, split-half RoPE, q * 0.125); k and v go to the cache and
//           its bf16 shadow, q and the new k / v stay in shared memory.  Without kPost
//           k_qkv_post has run and q comes from the query buffer;
//   scores  one key per thread: its 64-float key row against the 7 queries, s[h][k]
//           in shared memory;
//   softmax warp h takes head h: max, exp(s - max) in place, sum;
//   P V     warp w takes keys w, w + 8, ...; lane l accumulates dims 2l, 2l + 1 of all
//           7 heads (coalesced 256-byte V rows), the 8 warp partials are added in
//           warp order;
//   output  warp h divides by the sum and stores head h (one 64-group) as limbs.
// The cache rows of earlier positions are read through the read-only path; with kPost
// the row written by this CTA (k == pos) is taken from shared memory.
constexpr int ATTN_ROWS_POST = 3;  // attention kind: rows of distinct slots, QKV post fused
constexpr int AR_THREADS = 256;
constexpr int AR_WARPS = AR_THREADS / 32;
static_assert(GQA * 32 + 32 == AR_THREADS, "one thread per q RoPE pair plus one warp of k pairs");

struct QkvPost {
    const float *part;  // QKV GEMM partials [splits][rows][QKV_ROWS]
    int splits;
    long long sstride;
    const float *bias, *rope_cos, *rope_sin;
    KvShadow sh;
};

template <bool kPost>
__global__ void __launch_bounds__(AR_THREADS) k_attn_row(const QkvPost pp, const float *__restrict__ q, Rows rows,
                                                         float *__restrict__ kc, float *__restrict__ vc, int layer,
                                                         Limbs out)
{
    pdl_enter();
    const int g = blockIdx.x, t = blockIdx.y;
    const int pos = rows.pos[t], slot = rows.slot[t];
    const int nk = min(pos, CONTEXT - 1) + 1;
    __shared__ __align__(16) float sq[GQA][HEAD_DIM];
    __shared__ __align__(16) float snk[HEAD_DIM];
    __shared__ float snv[HEAD_DIM];
    __shared__ float ss[GQA][CONTEXT];
    __shared__ __align__(16) float sred[AR_WARPS][GQA * HEAD_DIM];
    __shared__ float sl[GQA];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (!kPost) {
        for (int i = tid; i < GQA * HEAD_DIM; i += AR_THREADS)
            sq[i / HEAD_DIM][i % HEAD_DIM] = q[(size_t)t * DIM + g * GQA * HEAD_DIM + i];
    } else {
        const float *p = pp.part + (size_t)t * QKV_ROWS;
        auto sum2 = [&](int r0, float &d0, float &d1) {
            d0 = sum_splits1(p + r0, pp.splits, pp.sstride) + __ldg(pp.bias + r0);
            d1 = sum_splits1(p + r0 + 32, pp.splits, pp.sstride) + __ldg(pp.bias + r0 + 32);
        };
        float d0, d1;
        const int i = lane;
        const int r0 = warp < GQA ? (g * GQA + warp) * HEAD_DIM + i : DIM + g * HEAD_DIM + i;
        sum2(r0, d0, d1);
        const float cs = __ldg(pp.rope_cos + pos * 32 + i), sn = __ldg(pp.rope_sin + pos * 32 + i);
        const float a = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
        const float b = __fadd_rn(__fmul_rn(d1, cs), __fmul_rn(d0, sn));
        if (warp < GQA) {
            sq[warp][i] = a * 0.125f;
            sq[warp][i + 32] = b * 0.125f;
        } else {
            const size_t o = kv_off(slot, layer, g, pos);
            kc[o + i] = a;
            kc[o + i + 32] = b;
            mb::tc::split_bf16(a, pp.sh.k_hi[o + i], pp.sh.k_lo[o + i]);
            mb::tc::split_bf16(b, pp.sh.k_hi[o + i + 32], pp.sh.k_lo[o + i + 32]);
            snk[i] = a;
            snk[i + 32] = b;
        }
        if (warp == 0) {
            sum2(DIM + KV + g * HEAD_DIM + i, d0, d1);
            float *v = vc + kv_off(slot, layer, g, pos);
            v[i] = d0;
            v[i + 32] = d1;
            mb::tc::split_bf16(d0, pp.sh.vt_hi[vt_off(slot, layer, g, i, pos)], pp.sh.vt_lo[vt_off(slot, layer, g, i, pos)]);
            mb::tc::split_bf16(d1, pp.sh.vt_hi[vt_off(slot, layer, g, i + 32, pos)],
                               pp.sh.vt_lo[vt_off(slot, layer, g, i + 32, pos)]);
            snv[i] = d0;
            snv[i + 32] = d1;
        }
    }
    __syncthreads();
    const float *kb = kc + kv_off(slot, layer, g, 0);
    const float *vb = vc + kv_off(slot, layer, g, 0);
    for (int k = tid; k < nk; k += AR_THREADS) {
        const bool own = kPost && k == pos;
        const float4 *kr = own ? reinterpret_cast<const float4 *>(snk)
                               : reinterpret_cast<const float4 *>(kb + (size_t)k * HEAD_DIM);
        float z[GQA];
#pragma unroll
        for (int h = 0; h < GQA; h++) z[h] = 0.f;
#pragma unroll
        for (int j = 0; j < HEAD_DIM / 4; j++) {
            const float4 kv = own ? kr[j] : __ldg(kr + j);
#pragma unroll
            for (int h = 0; h < GQA; h++) {
                const float4 qv = *reinterpret_cast<const float4 *>(&sq[h][4 * j]);
                z[h] = fmaf(qv.x, kv.x, z[h]);
                z[h] = fmaf(qv.y, kv.y, z[h]);
                z[h] = fmaf(qv.z, kv.z, z[h]);
                z[h] = fmaf(qv.w, kv.w, z[h]);
            }
        }
#pragma unroll
        for (int h = 0; h < GQA; h++) ss[h][k] = z[h];
    }
    __syncthreads();
    if (warp < GQA) {
        float m = -INFINITY;
        for (int k = lane; k < nk; k += 32) m = fmaxf(m, ss[warp][k]);
        m = mb::warp_max(m);
        float l = 0.f;
        for (int k = lane; k < nk; k += 32) {
            const float e = expf(ss[warp][k] - m);
            ss[warp][k] = e;
            l += e;
        }
        l = mb::warp_sum(l);
        if (lane == 0) sl[warp] = l;
    }
    __syncthreads();
    float a[GQA][2];
#pragma unroll
    for (int h = 0; h < GQA; h++) a[h][0] = a[h][1] = 0.f;
    // cache rows first (16 iterations unrolled: their loads are in flight together), then
    // with kPost the row of `pos` (the last key, so the order per warp is unchanged) from
    // shared memory
    const int nglob = kPost ? nk - 1 : nk;
#pragma unroll 16
    for (int k = warp; k < nglob; k += AR_WARPS) {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(vb + (size_t)k * HEAD_DIM) + lane);
#pragma unroll
        for (int h = 0; h < GQA; h++) {
            const float p = ss[h][k];
            a[h][0] = fmaf(p, v.x, a[h][0]);
            a[h][1] = fmaf(p, v.y, a[h][1]);
        }
    }
    if (kPost && warp == (nk - 1) % AR_WARPS) {
        const float2 v = make_float2(snv[2 * lane], snv[2 * lane + 1]);
#pragma unroll
        for (int h = 0; h < GQA; h++) {
            const float p = ss[h][nk - 1];
            a[h][0] = fmaf(p, v.x, a[h][0]);
            a[h][1] = fmaf(p, v.y, a[h][1]);
        }
    }
#pragma unroll
    for (int h = 0; h < GQA; h++)
        *reinterpret_cast<float2 *>(&sred[warp][h * HEAD_DIM + 2 * lane]) = make_float2(a[h][0], a[h][1]);
    __syncthreads();
    if (warp < GQA) {
        float sx = 0.f, sy = 0.f;
#pragma unroll
        for (int w = 0; w < AR_WARPS; w++) {
            const float2 p = *reinterpret_cast<const float2 *>(&sred[w][warp * HEAD_DIM + 2 * lane]);
            sx += p.x;
            sy += p.y;
        }
        const float l = sl[warp];
        const float v[2] = {sx / l, sy / l};
        const int head = g * GQA + warp;
        mb::tq::store_limbs<2, 32>(v, out.q + (size_t)t * 3 * DIM, DIM, head * HEAD_DIM + 2 * lane,
                                   out.s + (size_t)t * (DIM / GROUP) + head, lane);
    }
}

// h = silu(gate) * up from the gate|up partials (rows interleaved per 64: gate feature
// f at row 128 (f / 64) + f % 64, up feature f 64 rows further), as limbs for the down
// GEMM; two features per thread.  grid (ceil(HIDDEN / 512), rows).  Decode steps use
// it: their gate|up GEMM covers only half the SMs, so the SwiGLU runs better as its own
// launch over all of them than as a tail of that GEMM.
__global__ void __launch_bounds__(256) k_swiglu(const float *__restrict__ part, int splits, long long sstride,
                                                int8_t *hq, float *hs)
{
    pdl_enter();
    const int t = blockIdx.y, i = (blockIdx.x * 256 + threadIdx.x) * 2;
    if (i >= HIDDEN) return;
    const float *p = part + (size_t)t * GU_ROWS + (i / 64) * 128 + i % 64;
    float2 g = *reinterpret_cast<const float2 *>(p), u = *reinterpret_cast<const float2 *>(p + 64);
    for (int s = 1; s < splits; s++) {
        const float2 gs = *reinterpret_cast<const float2 *>(p + s * sstride);
        const float2 us = *reinterpret_cast<const float2 *>(p + s * sstride + 64);
        g.x += gs.x;
        g.y += gs.y;
        u.x += us.x;
        u.y += us.y;
    }
    const float hv[2] = {(g.x / (1.f + expf(-g.x))) * u.x, (g.y / (1.f + expf(-g.y))) * u.y};
    // a warp holds 64 consecutive features: one group of the down projection's input
    mb::tq::store_limbs<2, 32>(hv, hq + (size_t)t * 3 * HIDDEN, HIDDEN, i,
                               hs + (size_t)t * (HIDDEN / GROUP) + i / GROUP, threadIdx.x & 31);
}

// ---- prompt attention on the tensor cores ---------------------------------------------
//
// One CTA per (block of 128 consecutive rows of one slot at positions p0..p0+127, p0 a
// multiple of 128; query head h; span z of up to 256 keys).  Keys come as bf16 pairs
// from the cache shadow (written by k_qkv_post) through TMA into a two-stage ring; for
// each chunk of 64 keys, S = Q K^T (q carries the 0.125) is three tcgen05 MMAs
// (hi*hi + hi*lo + lo*hi) into TMEM; each of the 128 threads owns one query row: causal
// mask and online softmax over its 64 scores, P written as a bf16 pair in the
// 128-byte-swizzled layout; O_c = P V is three more MMAs; the thread folds O_c into its
// fp32 row.  The span's (max, sum, 64 weighted sums) go to the partial buffer and
// k_attn_combine merges the spans.
constexpr int TQ = 128;           // queries per CTA
constexpr int TK = 64;            // keys per chunk
constexpr int TSPAN = 256;        // keys per CTA
constexpr int TSPLIT = CONTEXT / TSPAN;
constexpr uint32_t kTileQ = TQ * HEAD_DIM * 2;   // 16 KiB: one bf16 [128][64] tile
constexpr uint32_t kTileK = TK * HEAD_DIM * 2;   // 8 KiB: one bf16 [64][64] tile
constexpr uint32_t kStageKV = 4 * kTileK;        // K hi, K lo, Vt hi, Vt lo
constexpr int kAttnStages = 1;                   // key chunks in flight per CTA
constexpr size_t TC_SMEM = 1024 + 2 * kTileQ /*Q*/ + kAttnStages * kStageKV + 2 * kTileQ /*P*/ + 128;

struct AttnMaps {
    CUtensorMap k_hi, k_lo;    // [slot*LAYERS*KV_HEADS*CONTEXT][64], box {64, 64}
    CUtensorMap vt_hi, vt_lo;  // [slot*LAYERS*KV_HEADS*64][CONTEXT], box {64, 64}
};

// byte offset of element (r, c) of a [rows][64] bf16 tile in the SW128 K-major layout
MB_DEV uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2); }

MB_DEV void put8(uint8_t *tile, int r, int c0, const float (&v)[8], uint8_t *tile_lo)
{
    __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
    for (int i = 0; i < 8; i++) mb::tc::split_bf16(v[i], hi[i], lo[i]);
    const uint32_t off = sw128_off(r, c0);
    *reinterpret_cast<uint4 *>(tile + off) = *reinterpret_cast<const uint4 *>(hi);
    *reinterpret_cast<uint4 *>(tile_lo + off) = *reinterpret_cast<const uint4 *>(lo);
}

__global__ void __launch_bounds__(TQ, 1) k_attn_tc(const float *__restrict__ q, Rows rows,
                                                  const __grid_constant__ AttnMaps maps, int layer,
                                                  float *__restrict__ part, Limbs out, int *err)
{
    pdl_enter();
    const int h = blockIdx.y, g = h / GQA, t0 = blockIdx.x * TQ, z = blockIdx.z;
    const int slot = rows.slot[t0], p0 = rows.pos[t0];
    const int key_begin = z * TSPAN, key_end = min(key_begin + TSPAN, p0 + TQ);
    if (key_begin >= key_end) return;  // this span lies after the block's last query
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *q_hi = sm, *q_lo = q_hi + kTileQ, *kv = q_lo + kTileQ;
    uint8_t *p_hi = kv + kAttnStages * kStageKV, *p_lo = p_hi + kTileQ;
    uint64_t *bar = reinterpret_cast<uint64_t *>(p_lo + kTileQ);  // [0, stages) stage full, [2] S, [3] O, [4] drain
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 5);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int nch = (key_end - key_begin + TK - 1) / TK;
    const int krow0 = (((slot * LAYERS + layer) * KV_HEADS + g) * CONTEXT);  // K map row of key 0
    const int vrow0 = (((slot * LAYERS + layer) * KV_HEADS + g) * HEAD_DIM);  // Vt map row of dim 0
    int issued = 0, landed_n = 0;  // thread 0: chunks whose copies were issued / have landed
    auto issue = [&](int c) {  // TMA of chunk c into stage c % kAttnStages (thread 0)
        issued = c + 1;
        const int st = c % kAttnStages, k0 = key_begin + c * TK;
        uint8_t *b = kv + st * kStageKV;
        mb::as::mbar_expect_tx(&bar[st], kStageKV);
        mb::as::tma_load_2d(b, &maps.k_hi, 0, krow0 + k0, &bar[st]);
        mb::as::tma_load_2d(b + kTileK, &maps.k_lo, 0, krow0 + k0, &bar[st]);
        mb::as::tma_load_2d(b + 2 * kTileK, &maps.vt_hi, k0, vrow0, &bar[st]);
        mb::as::tma_load_2d(b + 3 * kTileK, &maps.vt_lo, k0, vrow0, &bar[st]);
    };
    if (tid == 0) {
        for (int i = 0; i < 5; i++) mb::as::mbar_init(&bar[i], 1);
        *abort = 0;
        mb::as::fence_barrier_init();
        for (int c = 0; c < kAttnStages && c < nch; c++) issue(c);
    }
    if (warp == 0) mb::as::tmem_alloc(tmem_slot, 128);
    for (int ci = tid; ci < TQ * 8; ci += TQ) {
        const int r = ci >> 3, c0 = (ci & 7) * 8;
        const float4 *src = reinterpret_cast<const float4 *>(q + (size_t)(t0 + r) * DIM + h * HEAD_DIM + c0);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        put8(q_hi, r, c0, v, q_lo);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mb::as::tc_fence_before();
    __syncthreads();
    mb::as::tc_fence_after();
    const uint32_t tmem = *tmem_slot, tm_s = tmem, tm_o = tmem + 64;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    constexpr uint32_t idesc = mb::as::idesc_bf16_f32(TQ, TK);
    const int row = tid, qpos = p0 + row;
    float o[HEAD_DIM];
#pragma unroll
    for (int d = 0; d < HEAD_DIM; d++) o[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int c = 0; c < nch; c++) {
        const int st = c % kAttnStages, k0 = key_begin + c * TK;
        uint8_t *kvs = kv + st * kStageKV;
        if (tid == 0) {
            const bool landed = mb::as::mbar_wait(&bar[st], (c / kAttnStages) & 1, abort);
            if (landed) {
                landed_n = c + 1;
                mb::as::tc_fence_after();
                const uint32_t qa = mb::as::smem_u32(q_hi), qb = mb::as::smem_u32(q_lo);
                const uint32_t ka = mb::as::smem_u32(kvs), kb = ka + kTileK;
#pragma unroll
                for (int kk = 0; kk < HEAD_DIM / 16; kk++) {
                    const uint32_t off = kk * 32;
                    mb::as::mma_bf16(tm_s, mb::as::sw128_desc(qa + off), mb::as::sw128_desc(ka + off), idesc, kk > 0);
                    mb::as::mma_bf16(tm_s, mb::as::sw128_desc(qa + off), mb::as::sw128_desc(kb + off), idesc, true);
                    mb::as::mma_bf16(tm_s, mb::as::sw128_desc(qb + off), mb::as::sw128_desc(ka + off), idesc, true);
                }
                mb::as::mma_commit(&bar[2]);
            } else {
                *abort = 1;
            }
        }
        ok = mb::as::mbar_wait(&bar[2], c & 1, abort);
        mb::as::tc_fence_after();
        if (__syncthreads_or(!ok)) {  // block-uniform: every thread leaves together
            if (tid == 0) atomicCAS(err, 0, 31);
            ok = false;
            break;
        }
        // pass 1: row max of the masked scores; pass 2: exponentials, P row, sum
        float mx = m;
#pragma unroll
        for (int j = 0; j < TK / 16; j++) {
            uint32_t r16[16];
            mb::as::tmem_ld16(tm_s + lane_base + j * 16, r16);
            mb::as::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (k0 + j * 16 + i <= qpos) mx = fmaxf(mx, __uint_as_float(r16[i]));
        }
        const float scale = __expf(m - mx);
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < TK / 16; j++) {
            uint32_t r16[16];
            mb::as::tmem_ld16(tm_s + lane_base + j * 16, r16);
            mb::as::tmem_wait_ld();
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                float pv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int key = k0 + j * 16 + hh * 8 + i;
                    pv[i] = key <= qpos ? __expf(__uint_as_float(r16[hh * 8 + i]) - mx) : 0.f;
                    sum += pv[i];
                }
                put8(p_hi, row, j * 16 + hh * 8, pv, p_lo);
            }
        }
        l = l * scale + sum;
        m = mx;
#pragma unroll
        for (int d = 0; d < HEAD_DIM; d++) o[d] *= scale;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mb::as::tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            mb::as::tc_fence_after();
            const uint32_t pa = mb::as::smem_u32(p_hi), pb = mb::as::smem_u32(p_lo);
            const uint32_t va = mb::as::smem_u32(kvs + 2 * kTileK), vb = va + kTileK;
#pragma unroll
            for (int kk = 0; kk < TK / 16; kk++) {
                const uint32_t off = kk * 32;
                mb::as::mma_bf16(tm_o, mb::as::sw128_desc(pa + off), mb::as::sw128_desc(va + off), idesc, kk > 0);
                mb::as::mma_bf16(tm_o, mb::as::sw128_desc(pa + off), mb::as::sw128_desc(vb + off), idesc, true);
                mb::as::mma_bf16(tm_o, mb::as::sw128_desc(pb + off), mb::as::sw128_desc(va + off), idesc, true);
            }
            mb::as::mma_commit(&bar[3]);
        }
        ok = mb::as::mbar_wait(&bar[3], c & 1, abort);
        mb::as::tc_fence_after();
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicCAS(err, 0, 32);
            ok = false;
            break;
        }
#pragma unroll
        for (int j = 0; j < HEAD_DIM / 16; j++) {
            uint32_t r16[16];
            mb::as::tmem_ld16(tm_o + lane_base + j * 16, r16);
            mb::as::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; i++) o[j * 16 + i] += __uint_as_float(r16[i]);
        }
        mb::as::tc_fence_before();
        __syncthreads();  // stage st, S and P are free again
        if (tid == 0 && c + kAttnStages < nch) issue(c + kAttnStages);
    }
    if (!ok && tid == 0) {
        // every MMA issued so far has finished, and the copies in flight have landed,
        // before TMEM and shared memory go away
        mb::as::mma_commit(&bar[4]);
        const volatile int never = 0;
        mb::as::mbar_wait(&bar[4], 0, &never);
        for (int k = landed_n; k < issued; k++) mb::as::mbar_wait(&bar[k % kAttnStages], (k / kAttnStages) & 1, &never);
    }
    if (ok && p0 + TQ <= TSPAN) {
        // the block's keys lie in this one span: the row is finished here, as the span
        // combine would finish it from one partial (weight exp(0) = 1), and written as
        // limbs of the O GEMM (this thread holds the head's whole 64-group)
#pragma unroll
        for (int d = 0; d < HEAD_DIM; d++) o[d] = o[d] / l;
        mb::tq::store_limbs<HEAD_DIM, 1>(o, out.q + (size_t)(t0 + row) * 3 * DIM, DIM, h * HEAD_DIM,
                                         out.s + (size_t)(t0 + row) * (DIM / GROUP) + h, 0);
    } else if (ok) {
        float *pt = part + (((size_t)(t0 + row) * HEADS + h) * NCHUNK + z) * PART;
        // a partial is PART = 66 floats: its payload is 8-byte aligned, so float2 stores
        pt[0] = m;
        pt[1] = l;
#pragma unroll
        for (int d = 0; d < HEAD_DIM; d += 2) *reinterpret_cast<float2 *>(pt + 2 + d) = make_float2(o[d], o[d + 1]);
    }
    mb::as::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        mb::as::tc_fence_after();
        mb::as::tmem_free(tmem, 128);
    }
}

// Prompt attention for a block of 64 consecutive rows of one slot (positions
// p0..p0+63, p0 a multiple of 64) and one query head: key chunks of 64 staged in
// shared memory, online softmax, fp32 throughout.  Thread (ty, tx) owns query rows
// ty + 16i and, for scores, keys tx + 16j (strided so the float4 reads of K rows hit
// distinct banks); for the output, dims 4tx..4tx+3.
constexpr int QB = 64;
constexpr int QB_LD = HEAD_DIM + 4;  // padded row (floats) of the Q, K and P tiles
constexpr size_t QB_SMEM = sizeof(float) * (3 * QB * QB_LD + CHUNK * HEAD_DIM);

__global__ void __launch_bounds__(256) k_attn_block(const float *__restrict__ q, Rows rows,
                                                    const float *__restrict__ kc, const float *__restrict__ vc,
                                                    int layer, Limbs out)
{
    pdl_enter();
    extern __shared__ float4 smem4[];
    float *sQ = reinterpret_cast<float *>(smem4);
    float *sK = sQ + QB * QB_LD;
    float *sP = sK + CHUNK * QB_LD;
    float *sV = sP + QB * QB_LD;
    const int h = blockIdx.y, g = h / GQA, t0 = blockIdx.x * QB;
    const int slot = rows.slot[t0], p0 = rows.pos[t0];
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    for (int idx = tid; idx < QB * HEAD_DIM / 4; idx += 256) {
        const int r = idx / (HEAD_DIM / 4), c4 = idx % (HEAD_DIM / 4);
        reinterpret_cast<float4 *>(sQ + r * QB_LD)[c4] =
            *reinterpret_cast<const float4 *>(q + (size_t)(t0 + r) * DIM + h * HEAD_DIM + c4 * 4);
    }
    float m[4], l[4], acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
    }
    const int nchunks = p0 / CHUNK + 1;
    for (int c = 0; c < nchunks; c++) {
        const size_t base = kv_off(slot, layer, g, c * CHUNK);
        __syncthreads();  // previous chunk's K, V and P are no longer read
        for (int idx = tid; idx < CHUNK * HEAD_DIM / 4; idx += 256) {
            const int r = idx / (HEAD_DIM / 4), c4 = idx % (HEAD_DIM / 4);
            reinterpret_cast<float4 *>(sK + r * QB_LD)[c4] = *reinterpret_cast<const float4 *>(kc + base + idx * 4);
            reinterpret_cast<float4 *>(sV)[idx] = *reinterpret_cast<const float4 *>(vc + base + idx * 4);
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll 4
        for (int d4 = 0; d4 < HEAD_DIM / 4; d4++) {
            float4 qa[4], kb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qa[i] = reinterpret_cast<const float4 *>(sQ + (ty + 16 * i) * QB_LD)[d4];
#pragma unroll
            for (int j = 0; j < 4; j++) kb[j] = reinterpret_cast<const float4 *>(sK + (tx + 16 * j) * QB_LD)[d4];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    sc[i][j] = fmaf(qa[i].x, kb[j].x, sc[i][j]);
                    sc[i][j] = fmaf(qa[i].y, kb[j].y, sc[i][j]);
                    sc[i][j] = fmaf(qa[i].z, kb[j].z, sc[i][j]);
                    sc[i][j] = fmaf(qa[i].w, kb[j].w, sc[i][j]);
                }
        }
        const bool diagonal = c == nchunks - 1;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qpos = ty + 16 * i;  // relative to p0; the diagonal chunk starts at p0
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (diagonal && tx + 16 * j > qpos) sc[i][j] = -INFINITY;
                mx = fmaxf(mx, sc[i][j]);
            }
#pragma unroll
            for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mnew = fmaxf(m[i], mx);
            const float scale = expf(m[i] - mnew);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float e = expf(sc[i][j] - mnew);
                sP[(ty + 16 * i) * QB_LD + tx + 16 * j] = e;
                sum += e;
            }
#pragma unroll
            for (int o = 8; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            l[i] = l[i] * scale + sum;
            m[i] = mnew;
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] *= scale;
        }
        __syncthreads();
#pragma unroll 2
        for (int k4 = 0; k4 < CHUNK / 4; k4++) {
            float4 pa[4], vb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pa[i] = reinterpret_cast<const float4 *>(sP + (ty + 16 * i) * QB_LD)[k4];
#pragma unroll
            for (int kk = 0; kk < 4; kk++) vb[kk] = reinterpret_cast<const float4 *>(sV + (k4 * 4 + kk) * HEAD_DIM)[tx];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float pv[4] = {pa[i].x, pa[i].y, pa[i].z, pa[i].w};
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    acc[i][0] = fmaf(pv[kk], vb[kk].x, acc[i][0]);
                    acc[i][1] = fmaf(pv[kk], vb[kk].y, acc[i][1]);
                    acc[i][2] = fmaf(pv[kk], vb[kk].z, acc[i][2]);
                    acc[i][3] = fmaf(pv[kk], vb[kk].w, acc[i][3]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = t0 + ty + 16 * i;
        const float inv = 1.f / l[i];
        const float v[4] = {acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv};
        // the 16 lanes of one ty hold the head's 64 dims: one group
        mb::tq::store_limbs<4, 16>(v, out.q + (size_t)row * 3 * DIM, DIM, h * HEAD_DIM + tx * 4,
                                   out.s + (size_t)row * (DIM / GROUP) + h, tx);
    }
}

// ---- batched sampler -----------------------------------------------------------------

MB_DEV void bitonic_desc(unsigned long long *keys, int n)
{
    for (int size = 2; size <= n; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
                const int i = 2 * t - (t & (stride - 1)), j = i + stride;
                const unsigned long long a = keys[i], b = keys[j];
                if (((i & size) == 0) ? (a < b) : (a > b)) {
                    keys[i] = b;
                    keys[j] = a;
                }
            }
            __syncthreads();
        }
}

// Exact top k (k <= 64) of n unique 64-bit keys in shared memory, best first, into
// out[0..k): radix select of the k-th largest key over 8-bit digits from the top
// (passes stop once the boundary digit holds exactly the keys still needed), then
// compaction of the keys >= that threshold and a one-warp bitonic sort of the k
// survivors.  All threads of the block call it.
struct TopkScratch {
    unsigned hist[256];
    unsigned long long prefix, mask;
    int need, count;
};

MB_DEV void block_topk(const unsigned long long *keys, int n, int k, unsigned long long *out, TopkScratch &sc)
{
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) {
        sc.prefix = 0ull;
        sc.mask = 0ull;
        sc.need = k;
        sc.count = 0;
    }
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += nt) sc.hist[b] = 0u;
        __syncthreads();
        const unsigned long long prefix = sc.prefix, mask = sc.mask;
        for (int i = tid; i < n; i += nt)
            if ((keys[i] & mask) == prefix) atomicAdd(&sc.hist[(unsigned)(keys[i] >> shift) & 255u], 1u);
        __syncthreads();
        if (tid < 32) {
            // digit d where the keys above d number < need <= keys at or above d
            const int lane = tid;
            unsigned above = 0u;  // keys in digits greater than this lane's 8-digit group
            unsigned grp = 0u;
#pragma unroll
            for (int j = 0; j < 8; j++) grp += sc.hist[255 - (lane * 8 + j)];
            unsigned incl = grp;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            above = incl - grp;
            const unsigned need = (unsigned)sc.need;
            const bool mine = above < need && need <= incl;
            const unsigned who = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                unsigned acc = above;
                int d = 255 - lane * 8;
                for (int j = 0; j < 8; j++, d--) {
                    const unsigned c = sc.hist[d];
                    if (acc + c >= need) break;
                    acc += c;
                }
                sc.need = (int)(need - acc);
                sc.prefix = prefix | ((unsigned long long)d << shift);
                sc.mask = mask | (255ull << shift);
                sc.count = (int)sc.hist[d];
            }
            (void)who;
        }
        __syncthreads();
        if (sc.count == sc.need) break;  // every key with this prefix is in
    }
    // keys strictly above the prefix group, plus the prefix group when it is all in
    const unsigned long long prefix = sc.prefix, mask = sc.mask;
    const bool all_group = sc.count == sc.need;
    __syncthreads();
    if (tid == 0) sc.count = 0;
    __syncthreads();
    for (int i = tid; i < n; i += nt) {
        const unsigned long long key = keys[i];
        const unsigned long long kp = key & mask;
        if (kp > prefix || (kp == prefix && all_group)) {
            const int slot = atomicAdd(&sc.count, 1);
            if (slot < 64) out[slot] = key;
        }
    }
    __syncthreads();
    if (tid < 32) {
        const int m = min(sc.count, 64);
        unsigned long long a = tid < m ? out[tid] : 0ull, b = tid + 32 < m ? out[tid + 32] : 0ull;
        // bitonic sort of 64 keys held two per lane (a = element lane, b = element lane + 32), descending
        for (int size = 2; size <= 64; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                if (stride == 32) {
                    const bool desc = true;
                    if (desc ? (a < b) : (a > b)) {
                        const unsigned long long t = a;
                        a = b;
                        b = t;
                    }
                } else {
                    // elements i = lane and i = lane + 32 paired with i ^ stride (same half)
                    const unsigned long long pa = __shfl_xor_sync(0xffffffffu, a, stride);
                    const unsigned long long pb = __shfl_xor_sync(0xffffffffu, b, stride);
                    const int ia = tid, ib = tid + 32;
                    const bool da = (ia & size) == 0, db = (ib & size) == 0;
                    const bool lowa = (ia & stride) == 0, lowb = (ib & stride) == 0;
                    // low element keeps the larger value in a descending run
                    a = (lowa == da) ? (a > pa ? a : pa) : (a < pa ? a : pa);
                    b = (lowb == db) ? (b > pb ? b : pb) : (b < pb ? b : pb);
                }
            }
        }
        __syncwarp();
        if (tid < k) out[tid] = a;
        if (tid + 32 < k) out[tid + 32] = b;
    }
    __syncthreads();
}

// Stage 1: for projected row r and a slice of SLICE ids, penalty (once per distinct
// id of the slot's history), control mask, and the slice's top k keys.
__global__ void __launch_bounds__(SAMPLE_THREADS) k_bs_stage1(const float *__restrict__ logits, const int *proj_src,
                                                              Rows rows, int nslots, const sampling::SeqState *st,
                                                              const sampling::Params *prm,
                                                              unsigned long long *__restrict__ out)
{
    pdl_enter();
    extern __shared__ unsigned long long keys[];  // [SLICE]
    __shared__ int hist[sampling::kHistory];
    const int r = blockIdx.y, lo = blockIdx.x * SLICE;
    const int n = min(VOCAB - lo, SLICE);
    const sampling::Params p = *prm;
    const int k = min(max(p.top_k, 1), sampling::kMaxK);
    const int slot = rows.slot[proj_src[r]];
    if (slot < 0 || slot >= nslots) return;
    const sampling::SeqState *s = st + slot;
    const float *lg = logits + (size_t)r * VOCAB + lo;
    const int count = min(max(s->history_count, 0), sampling::kHistory);
    if (threadIdx.x < count) hist[threadIdx.x] = s->history[threadIdx.x];
    // keys of the masked logits; penalised ids are rewritten below
    for (int i = threadIdx.x; i < SLICE; i += SAMPLE_THREADS) {
        unsigned long long key = 0ull;
        if (i < n) {
            const int id = lo + i;
            key = mb::rank_key((id >= p.control_first && id != p.eos) ? -1e30f : lg[i], id);
        }
        keys[i] = key;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        for (int j = threadIdx.x; j < count; j += 32) {
            const int id = hist[j];
            // ids outside this slice (most of the window) skip the duplicate scan
            if (id < lo || id >= lo + n || (id >= p.control_first && id != p.eos)) continue;
            bool dup = false;
            for (int u = 0; u < j; u++) dup |= hist[u] == id;
            if (!dup) {
                const float v = lg[id - lo];
                keys[id - lo] = mb::rank_key(v < 0 ? v * p.penalty : v / p.penalty, id);
            }
        }
    }
    __syncthreads();
    __shared__ unsigned long long best[sampling::kMaxK];
    __shared__ TopkScratch sc;
    block_topk(keys, SLICE, k, best, sc);
    for (int j = threadIdx.x; j < k; j += SAMPLE_THREADS)
        out[((size_t)r * NSLICE + blockIdx.x) * sampling::kMaxK + j] = best[j];
}

// Stage 2: merge the slices, draw the token, record it for the slot and set up the
// slot's next decode row (next_* arrays, at next_index[r] for projected row r, or at r
// when next_index is null).
__global__ void __launch_bounds__(SAMPLE_THREADS) k_bs_stage2(const unsigned long long *__restrict__ in,
                                                              const int *proj_src, Rows rows, int nslots,
                                                              sampling::SeqState *st, const sampling::Params *prm,
                                                              int *next_tok, int *next_pos, int *next_slot,
                                                              const int *next_index, int *out_tokens,
                                                              int *out_count, int out_stride)
{
    pdl_enter();
    constexpr int kMerge = 2048;  // >= NSLICE * kMaxK = 1216
    static_assert(kMerge >= NSLICE * sampling::kMaxK && kMerge % SAMPLE_THREADS == 0, "merge buffer");
    __shared__ unsigned long long keys[kMerge];
    const int r = blockIdx.x;
    const sampling::Params p = *prm;
    const int k = min(max(p.top_k, 1), sampling::kMaxK);
    const int src = proj_src[r];
    const int slot = rows.slot[src], pos = rows.pos[src];
    if (slot < 0 || slot >= nslots) return;
    for (int i = threadIdx.x; i < kMerge; i += SAMPLE_THREADS) {
        const int sl = i / k, j = i % k;
        keys[i] = (sl < NSLICE) ? in[((size_t)r * NSLICE + sl) * sampling::kMaxK + j] : 0ull;
    }
    __syncthreads();
    __shared__ unsigned long long best[sampling::kMaxK];
    __shared__ TopkScratch sc;
    block_topk(keys, kMerge, k, best, sc);
    if (threadIdx.x == 0) {
        const unsigned long long *keys = best;
        sampling::SeqState *s = st + slot;
        uint32_t seed = s->seed;
        int token = sampling::draw_token(keys, p, seed);
        if (token < 0 || token >= VOCAB) token = p.eos;
        if (!s->finished) {
            s->seed = seed;
            const int n = s->n_out;
            if (n < out_stride) out_tokens[(size_t)slot * out_stride + n] = token;
            s->n_out = n + 1;
            out_count[slot] = n + 1;
            sampling::record_token(token, p, s, nullptr, nullptr);
        }
        const int ni = next_index ? next_index[r] : r;
        next_tok[ni] = s->finished ? p.eos : token;
        next_pos[ni] = min(pos + 1, CONTEXT - 1);
        next_slot[ni] = slot;
    }
}

// ---- engine -------------------------------------------------------------------------

// A grouped-Q8 matrix for the int8 GEMM: int8 [rows][cols] and fp32 scales [rows][cols/64].
struct Weights {
    const int8_t *q = nullptr;
    const float *s = nullptr;
    int8_t *own_q = nullptr;  // device copies owned by the handle (fused matrices)
    float *own_s = nullptr;
};

struct PlanSet {
    Gemm qkv[LAYERS], o[LAYERS], gu[LAYERS], down[LAYERS];
};

}  // namespace qb

struct mocha_q8b {
    int device = 0, max_rows = 0, slots = 0;
    cudaStream_t stream = nullptr;
    unsigned char *d_file = nullptr;
    q8::Model m{};
    qb::Weights w_qkv[q8::LAYERS], w_o[q8::LAYERS], w_gu[q8::LAYERS], w_down[q8::LAYERS], w_head;
    float *bqkv = nullptr;  // [LAYERS][1152]
    float *x = nullptr, *q = nullptr, *part = nullptr, *apart = nullptr, *logits = nullptr;
    qb::Limbs lx{}, la{}, lhead{};  // GEMM inputs: normed x, attention output, head rows
    int8_t *lhq = nullptr;          // SwiGLU output limbs [rows * 3][HIDDEN]
    float *lhs = nullptr;           // and their scales [rows][HIDDEN / 64]
    float *kc = nullptr, *vc = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    qb::KvShadow kvs{};
    qb::AttnMaps amaps{};
    int *tok = nullptr, *pos = nullptr, *slot = nullptr;            // prompt rows [max_rows]
    int *ntok = nullptr, *npos = nullptr, *nslot = nullptr;         // decode rows [slots]
    int *proj_src = nullptr, *proj_dst = nullptr, *ident = nullptr;  // [slots], [max_rows], [slots]
    int *next_index = nullptr;                                       // [slots]: decode row of a refilled slot
    int *err = nullptr;
    unsigned long long *keys = nullptr;
    sampling::SeqState *st = nullptr;
    sampling::Params *params = nullptr;
    int *out_tokens = nullptr, *out_count = nullptr;
    int out_stride = 0;
    qb::PlanSet pre, dec;
    mb::tq::Gemm head;
    cudaGraphExec_t g_step = nullptr;
    int g_step_n = 0;
    cudaEvent_t ev[4] = {};
    size_t part_floats = 0;
};

namespace qb {
namespace {

#define QB_TRY(x) MB_CHECK(x)

// Launch with programmatic stream serialisation (see pdl_enter).
template <typename... KArgs, typename... Args>
int pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QB_TRY(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
    return 0;
}

int check_err(mocha_q8b *h)
{
    int e = 0;
    QB_TRY(cudaMemcpy(&e, h->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        fprintf(stderr, "mocha_q8b: device-side wait gave up (code %d)\n", e);
        return 1;
    }
    return 0;
}

template <class T>
int dalloc(T **p, size_t count)
{
    QB_TRY(cudaMalloc((void **)p, sizeof(T) * count + 256));
    return 0;
}

// Fuse matrices along their rows into a device copy owned by `w` (int8 rows and fp32
// scales back to back, in the order given).
int fuse(mocha_q8b *h, Weights &w, std::initializer_list<std::pair<Mat, int>> parts, int cols)
{
    size_t rows = 0;
    for (auto &pr : parts) rows += (size_t)pr.second;
    if (dalloc(&w.own_q, rows * cols) || dalloc(&w.own_s, rows * (cols / GROUP))) return 1;
    size_t r0 = 0;
    for (auto &pr : parts) {
        QB_TRY(cudaMemcpyAsync(w.own_q + r0 * cols, pr.first.w, (size_t)pr.second * cols, cudaMemcpyDeviceToDevice,
                               h->stream));
        QB_TRY(cudaMemcpyAsync(w.own_s + r0 * (cols / GROUP), pr.first.s, sizeof(float) * pr.second * (cols / GROUP),
                               cudaMemcpyDeviceToDevice, h->stream));
        r0 += (size_t)pr.second;
    }
    w.q = w.own_q;
    w.s = w.own_s;
    return 0;
}

// gate|up device copy for the SwiGLU GEMM epilogue: blocks of 64 gate rows and the
// matching 64 up rows alternate (fused row 128b + j = gate row 64b + j, fused row
// 128b + 64 + j = up row 64b + j), scales likewise.
int fuse_gate_up(mocha_q8b *h, Weights &w, const Mat &gate, const Mat &up, int cols)
{
    const size_t rows = 2 * (size_t)HIDDEN, gs = cols / GROUP;
    if (dalloc(&w.own_q, rows * cols) || dalloc(&w.own_s, rows * gs)) return 1;
    const Mat *src[2] = {&gate, &up};
    for (int i = 0; i < 2; i++) {
        QB_TRY(cudaMemcpy2DAsync(w.own_q + (size_t)i * 64 * cols, 128 * (size_t)cols, src[i]->w, 64 * (size_t)cols,
                                 64 * (size_t)cols, HIDDEN / 64, cudaMemcpyDeviceToDevice, h->stream));
        QB_TRY(cudaMemcpy2DAsync(w.own_s + (size_t)i * 64 * gs, 128 * gs * sizeof(float), src[i]->s,
                                 64 * gs * sizeof(float), 64 * gs * sizeof(float), HIDDEN / 64,
                                 cudaMemcpyDeviceToDevice, h->stream));
    }
    w.q = w.own_q;
    w.s = w.own_s;
    return 0;
}

int plan_set(mocha_q8b *h, PlanSet &ps, int n_max, bool fused_swiglu)
{
    for (int l = 0; l < LAYERS; l++) {
        if (mb::tq::plan(&ps.qkv[l], h->w_qkv[l].q, h->w_qkv[l].s, QKV_ROWS, DIM, h->lx.q, h->lx.s, n_max, h->part,
                         QKV_ROWS, 0, h->err) ||
            mb::tq::plan(&ps.o[l], h->w_o[l].q, h->w_o[l].s, DIM, DIM, h->la.q, h->la.s, n_max, h->part, DIM, 0,
                         h->err) ||
            mb::tq::plan(&ps.gu[l], h->w_gu[l].q, h->w_gu[l].s, GU_ROWS, DIM, h->lx.q, h->lx.s, n_max, h->part,
                         GU_ROWS, 0, h->err) ||
            (fused_swiglu && mb::tq::set_swiglu(&ps.gu[l], h->lhq, h->lhs, HIDDEN)) ||
            mb::tq::plan(&ps.down[l], h->w_down[l].q, h->w_down[l].s, DIM, HIDDEN, h->lhq, h->lhs, n_max, h->part,
                         DIM, 0, h->err))
            return 1;
    }
    return 0;
}

size_t plan_floats(const PlanSet &ps)
{
    size_t m = 0;
    for (int l = 0; l < LAYERS; l++) {
        const Gemm *g[4] = {&ps.qkv[l], &ps.o[l], &ps.gu[l], &ps.down[l]};
        for (const Gemm *x : g) m = std::max(m, mb::tq::partial_floats(*x));
    }
    return m;
}

// Attention for rows [0, n) after k_qkv_post: block 2, the tensor-core kernel over
// 128-row blocks of one slot at consecutive positions from a multiple of 128; block 1,
// the CUDA-core kernel over such 64-row blocks; block 0, one CTA per (KV head, row).
int enqueue_attention(mocha_q8b *h, Rows rows, int n, int layer, int block, int max_pos)
{
    static bool attr_done[64] = {}, tc_done[64] = {};
    if (block == 2) {
        if (!tc_done[h->device & 63]) {
            QB_TRY(cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM));
            tc_done[h->device & 63] = true;
        }
        if (pdl(k_attn_tc, dim3(n / TQ, HEADS, TSPLIT), TQ, TC_SMEM, h->stream, h->q, rows, h->amaps, layer, h->apart,
                h->la, h->err))
            return 1;
        // rows at positions < TSPAN were finished by k_attn_tc (their block needs one span)
        if (max_pos < TSPAN) return 0;
        return pdl(k_attn_combine<TSPLIT>, dim3((HEADS * n + kCombWarps - 1) / kCombWarps), 32 * kCombWarps, 0,
                   h->stream, h->apart, rows, h->la, TSPAN, n);
    }
    if (block) {
        if (!attr_done[h->device & 63]) {
            QB_TRY(cudaFuncSetAttribute(k_attn_block, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QB_SMEM));
            attr_done[h->device & 63] = true;
        }
        if (pdl(k_attn_block, dim3(n / QB, HEADS), 256, QB_SMEM, h->stream, h->q, rows, h->kc, h->vc, layer, h->la)) return 1;
        return 0;
    }
    return pdl(k_attn_row<false>, dim3(KV_HEADS, n), AR_THREADS, 0, h->stream, QkvPost{}, h->q, rows, h->kc, h->vc,
               layer, h->la);
}

// Attention kernel for rows (host arrays): 2 when every block of 128 rows is one slot
// at consecutive positions from a multiple of 128 (tensor cores), 1 for blocks of 64
// (CUDA cores), else one CTA per (KV head, row): ATTN_ROWS_POST (QKV post-processing
// in the same kernel) when no slot has two rows, 0 otherwise.
int block_kind(int n, const int *pos, const int *slots)
{
    auto distinct = [&]() {
        std::vector<char> seen(1024, 0);
        for (int i = 0; i < n; i++) {
            if (slots[i] < 0 || slots[i] >= (int)seen.size() || seen[slots[i]]) return false;
            seen[slots[i]] = 1;
        }
        return true;
    };
    auto blocks_of = [&](int b) {
        if (n % b) return false;
        for (int r = 0; r < n; r += b) {
            if (pos[r] % b) return false;
            for (int i = 1; i < b; i++)
                if (slots[r + i] != slots[r] || pos[r + i] != pos[r] + i) return false;
        }
        return true;
    };
    return blocks_of(TQ) ? 2 : (blocks_of(QB) ? 1 : (distinct() ? ATTN_ROWS_POST : 0));
}

// The whole transformer for rows [0, n) plus the head for `np` projected rows
// (proj_dst maps row -> head row or -1; the head reads rows 0..np-1 of the head limbs).
int enqueue_forward(mocha_q8b *h, Rows rows, int n, bool decode_set, const int *proj_dst, int np,
                    int block_attention, int max_pos)
{
    const PlanSet &ps = decode_set ? h->dec : h->pre;
    cudaStream_t s = h->stream;
    if (pdl(k_embed_norm, n, NT, 0, s, h->m.embed, rows, h->m.layer[0].attn_norm, h->x, h->lx)) return 1;
    mb::tc::Split sp;
    for (int l = 0; l < LAYERS; l++) {
        const Layer &L = h->m.layer[l];
        if (mb::tq::launch(ps.qkv[l], n, s, &sp)) return 1;
        if (block_attention == ATTN_ROWS_POST) {
            // rows of distinct slots: QKV post-processing fused into the row attention
            const QkvPost pp{h->part, sp.splits, sp.split_stride, h->bqkv + (size_t)l * QKV_ROWS, h->rope_cos,
                             h->rope_sin, h->kvs};
            if (pdl(k_attn_row<true>, dim3(KV_HEADS, n), AR_THREADS, 0, s, pp, (const float *)nullptr, rows, h->kc,
                    h->vc, l, h->la))
                return 1;
        } else {
            if (pdl(k_qkv_post, n, QKV_THREADS, 0, s, h->part, sp.splits, sp.split_stride,
                    h->bqkv + (size_t)l * QKV_ROWS, rows, h->rope_cos, h->rope_sin, h->q, h->kc, h->vc, l, h->kvs))
                return 1;
            if (enqueue_attention(h, rows, n, l, block_attention, max_pos)) return 1;
        }
        if (mb::tq::launch(ps.o[l], n, s, &sp)) return 1;
        if (pdl(sp.splits > 2 ? k_residual_norm<20> : k_residual_norm<1>, n, NT, 0, s, h->x, h->part, sp.splits,
                sp.split_stride, L.ffn_norm, h->lx, nullptr))
            return 1;
        if (mb::tq::launch(ps.gu[l], n, s, &sp)) return 1;  // prompt passes: writes the SwiGLU limbs
        if (decode_set && pdl(k_swiglu, dim3((HIDDEN + 511) / 512, n), 256, 0, s, h->part, sp.splits, sp.split_stride,
                              h->lhq, h->lhs))
            return 1;
        if (mb::tq::launch(ps.down[l], n, s, &sp)) return 1;
        const bool last = l + 1 == LAYERS;
        if (pdl(sp.splits > 2 ? k_residual_norm<20> : k_residual_norm<1>, n, NT, 0, s, h->x, h->part, sp.splits,
                sp.split_stride, last ? h->m.final_norm : h->m.layer[l + 1].attn_norm, last ? h->lhead : h->lx,
                last ? proj_dst : nullptr))
            return 1;
    }
    if (np > 0 && mb::tq::launch(h->head, np, s)) return 1;
    QB_TRY(cudaGetLastError());
    return 0;
}

// Sampling for projected rows 0..np-1; proj_src[r] is the activation row of
// projected row r (the identity map in decode steps).
int enqueue_sample(mocha_q8b *h, Rows rows, int np, const int *proj_src, const int *next_index = nullptr)
{
    static bool attr_done[64] = {};
    if (!attr_done[h->device & 63]) {
        QB_TRY(cudaFuncSetAttribute(k_bs_stage1, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)(SLICE * sizeof(unsigned long long))));
        attr_done[h->device & 63] = true;
    }
    if (pdl(k_bs_stage1, dim3(NSLICE, np), SAMPLE_THREADS, SLICE * sizeof(unsigned long long), h->stream, h->logits,
            proj_src, rows, h->slots, h->st, h->params, h->keys))
        return 1;
    if (pdl(k_bs_stage2, np, SAMPLE_THREADS, 0, h->stream, h->keys, proj_src, rows, h->slots, h->st, h->params, h->ntok,
            h->npos, h->nslot, next_index, h->out_tokens, h->out_count, h->out_stride))
        return 1;
    QB_TRY(cudaGetLastError());
    return 0;
}

int upload_rows(mocha_q8b *h, int n, const int *tokens, const int *pos, const int *slots)
{
    QB_TRY(cudaMemcpyAsync(h->tok, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->pos, pos, sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->slot, slots, sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    return 0;
}

bool rows_valid(mocha_q8b *h, int n, const int *tokens, const int *pos, const int *slots)
{
    if (n <= 0 || n > h->max_rows || !tokens || !pos || !slots) return false;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= VOCAB || pos[i] < 0 || pos[i] >= CONTEXT || slots[i] < 0 ||
            slots[i] >= h->slots)
            return false;
    return true;
}

// Set the projected rows: proj_src[r] = row, proj_dst[row] = r (others -1).
int set_projection(mocha_q8b *h, int n, int np, const int *src)
{
    std::vector<int> dst(n, -1);
    for (int r = 0; r < np; r++) dst[src[r]] = r;
    QB_TRY(cudaMemcpyAsync(h->proj_src, src, sizeof(int) * np, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->proj_dst, dst.data(), sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaStreamSynchronize(h->stream));  // dst is a stack vector
    return 0;
}

int capture_step(mocha_q8b *h, int n)
{
    if (h->g_step && h->g_step_n == n) return 0;
    if (h->g_step) {
        cudaGraphExecDestroy(h->g_step);
        h->g_step = nullptr;
    }
    cudaGraph_t g;
    QB_TRY(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    const Rows r{h->ntok, h->npos, h->nslot};
    int rc = enqueue_forward(h, r, n, true, h->ident, n, ATTN_ROWS_POST, CONTEXT - 1);  // one row per slot
    if (!rc) rc = enqueue_sample(h, r, n, h->ident);
    const cudaError_t e = cudaStreamEndCapture(h->stream, &g);
    if (rc || e != cudaSuccess) {
        fprintf(stderr, "mocha_q8b: step capture failed\n");
        return 1;
    }
    QB_TRY(cudaGraphInstantiate(&h->g_step, g, 0));
    cudaGraphDestroy(g);
    h->g_step_n = n;
    return 0;
}

}  // namespace
}  // namespace qb

using namespace qb;

extern "C" int mocha_q8b_open(int device, const void *file, unsigned long long bytes, int max_rows, int slots,
                              mocha_q8b **out)
{
    if (!out || !q8::valid_file(file, (size_t)bytes, false) || max_rows < 1 || max_rows > 16384 || slots < 1 ||
        slots > 256) {
        fprintf(stderr, "mocha_q8b_open: bad arguments or not a Qwen2.5-0.5B grouped-Q8 file\n");
        return 1;
    }
    *out = nullptr;
    int ndev = 0;
    QB_TRY(cudaGetDeviceCount(&ndev));
    cudaDeviceProp prop;
    if (device < 0 || device >= ndev || cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
        fprintf(stderr, "mocha_q8b_open: device %d is not a compute capability 10.x GPU\n", device);
        return 1;
    }
    QB_TRY(cudaSetDevice(device));
    mocha_q8b *h = new mocha_q8b();
    h->device = device;
    h->max_rows = max_rows;
    h->slots = slots;
    auto fail = [&]() {
        mocha_q8b_close(h);
        return 1;
    };
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) return fail();
    if (dalloc(&h->d_file, bytes)) return fail();
    if (cudaMemcpy(h->d_file, file, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return fail();
    const q8::FileHeader *hd = (const q8::FileHeader *)file;
    auto mat = [&](const q8::FileTensor &t) {
        return q8::Mat{(const int8_t *)(h->d_file + t.data), (const float *)(h->d_file + t.scales)};
    };
    h->m.embed = mat(hd->t[0]);
    h->m.final_norm = (const float *)(h->d_file + hd->t[q8::TENSORS - 1].data);
    std::vector<float> bias((size_t)LAYERS * QKV_ROWS);
    for (int l = 0; l < LAYERS; l++) {
        const q8::FileTensor *t = hd->t + 1 + l * q8::STRIDE;
        q8::Layer &L = h->m.layer[l];
        L.attn_norm = (const float *)(h->d_file + t[q8::ATTN_NORM].data);
        L.ffn_norm = (const float *)(h->d_file + t[q8::FFN_NORM].data);
        L.q = mat(t[q8::WQ]);
        L.k = mat(t[q8::WK]);
        L.v = mat(t[q8::WV]);
        L.o = mat(t[q8::WO]);
        L.gate = mat(t[q8::WGATE]);
        L.up = mat(t[q8::WUP]);
        L.down = mat(t[q8::WDOWN]);
        const unsigned char *fb = (const unsigned char *)file;
        memcpy(&bias[(size_t)l * QKV_ROWS], fb + t[q8::BQ].data, sizeof(float) * DIM);
        memcpy(&bias[(size_t)l * QKV_ROWS + DIM], fb + t[q8::BK].data, sizeof(float) * KV);
        memcpy(&bias[(size_t)l * QKV_ROWS + DIM + KV], fb + t[q8::BV].data, sizeof(float) * KV);
    }
    if (dalloc(&h->bqkv, bias.size())) return fail();
    if (cudaMemcpy(h->bqkv, bias.data(), sizeof(float) * bias.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail();

    // int8 weights as stored; q|k|v and gate|up fused along the output rows into copies
    for (int l = 0; l < LAYERS; l++) {
        const q8::Layer &L = h->m.layer[l];
        if (fuse(h, h->w_qkv[l], {{L.q, DIM}, {L.k, KV}, {L.v, KV}}, DIM) ||
            fuse_gate_up(h, h->w_gu[l], L.gate, L.up, DIM))
            return fail();
        h->w_o[l].q = L.o.w;
        h->w_o[l].s = L.o.s;
        h->w_down[l].q = L.down.w;
        h->w_down[l].s = L.down.s;
    }
    h->w_head.q = h->m.embed.w;
    h->w_head.s = h->m.embed.s;

    // activations
    const size_t R = (size_t)max_rows;
    if (dalloc(&h->x, R * DIM) || dalloc(&h->q, R * DIM) || dalloc(&h->lx.q, 3 * R * DIM) ||
        dalloc(&h->lx.s, R * (DIM / GROUP)) || dalloc(&h->la.q, 3 * R * DIM) || dalloc(&h->la.s, R * (DIM / GROUP)) ||
        dalloc(&h->lhq, 3 * R * HIDDEN) || dalloc(&h->lhs, R * (HIDDEN / GROUP)) ||
        dalloc(&h->apart, R * HEADS * NCHUNK * PART) || dalloc(&h->lhead.q, 3 * (size_t)slots * DIM) ||
        dalloc(&h->lhead.s, (size_t)slots * (DIM / GROUP)) ||
        dalloc(&h->logits, (size_t)slots * VOCAB) || dalloc(&h->tok, R) || dalloc(&h->pos, R) ||
        dalloc(&h->slot, R) || dalloc(&h->ntok, slots) || dalloc(&h->npos, slots) || dalloc(&h->nslot, slots) ||
        dalloc(&h->proj_src, slots) || dalloc(&h->proj_dst, R) || dalloc(&h->ident, slots) || dalloc(&h->next_index, slots) || dalloc(&h->err, 1) ||
        dalloc(&h->keys, (size_t)slots * NSLICE * sampling::kMaxK) || dalloc(&h->st, slots) ||
        dalloc(&h->params, 1) || dalloc(&h->out_count, slots))
        return fail();
    const size_t kv = kv_off(slots, 0, 0, 0);
    if (dalloc(&h->kc, kv) || dalloc(&h->vc, kv) || dalloc(&h->kvs.k_hi, kv) || dalloc(&h->kvs.k_lo, kv) ||
        dalloc(&h->kvs.vt_hi, kv) || dalloc(&h->kvs.vt_lo, kv))
        return fail();
    if (mb::tc::make_map_bf16(&h->amaps.k_hi, h->kvs.k_hi, (long long)slots * LAYERS * KV_HEADS * CONTEXT, HEAD_DIM,
                              TK) ||
        mb::tc::make_map_bf16(&h->amaps.k_lo, h->kvs.k_lo, (long long)slots * LAYERS * KV_HEADS * CONTEXT, HEAD_DIM,
                              TK) ||
        mb::tc::make_map_bf16(&h->amaps.vt_hi, h->kvs.vt_hi, (long long)slots * LAYERS * KV_HEADS * HEAD_DIM, CONTEXT,
                              HEAD_DIM) ||
        mb::tc::make_map_bf16(&h->amaps.vt_lo, h->kvs.vt_lo, (long long)slots * LAYERS * KV_HEADS * HEAD_DIM, CONTEXT,
                              HEAD_DIM))
        return fail();
    if (cudaMemset(h->kc, 0, sizeof(float) * kv) || cudaMemset(h->vc, 0, sizeof(float) * kv) ||
        cudaMemset(h->err, 0, sizeof(int)) || cudaMemset(h->out_count, 0, sizeof(int) * slots) ||
        cudaMemset(h->st, 0, sizeof(sampling::SeqState) * slots))
        return fail();
    {
        std::vector<int> id(slots);
        for (int i = 0; i < slots; i++) id[i] = i;
        if (cudaMemcpy(h->ident, id.data(), sizeof(int) * slots, cudaMemcpyHostToDevice) != cudaSuccess) return fail();
    }
    std::vector<float> rc((size_t)CONTEXT * 32), rs((size_t)CONTEXT * 32);
    q8::fill_rope_tables(rc.data(), rs.data(), CONTEXT, 32, 1000000.f);
    if (dalloc(&h->rope_cos, rc.size()) || dalloc(&h->rope_sin, rs.size())) return fail();
    if (cudaMemcpy(h->rope_cos, rc.data(), sizeof(float) * rc.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(h->rope_sin, rs.data(), sizeof(float) * rs.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail();

    // GEMM call sites; the partial buffer is sized from the plans' split counts
    if (plan_set(h, h->pre, max_rows, true) || plan_set(h, h->dec, slots, false)) return fail();
    if (mb::tq::plan(&h->head, h->w_head.q, h->w_head.s, VOCAB, DIM, h->lhead.q, h->lhead.s, slots, h->logits, VOCAB,
                     1, h->err))
        return fail();
    h->part_floats = std::max(plan_floats(h->pre), plan_floats(h->dec));
    if (dalloc(&h->part, h->part_floats)) return fail();
    for (int l = 0; l < LAYERS; l++)
        for (PlanSet *ps : {&h->pre, &h->dec}) {
            ps->qkv[l].p.d = h->part;
            ps->o[l].p.d = h->part;
            ps->gu[l].p.d = h->part;
            ps->down[l].p.d = h->part;
        }
    for (int i = 0; i < 4; i++)
        if (cudaEventCreate(&h->ev[i]) != cudaSuccess) return fail();
    if (cudaStreamSynchronize(h->stream) != cudaSuccess || cudaGetLastError() != cudaSuccess) return fail();
    *out = h;
    return 0;
}

extern "C" int mocha_q8b_close(mocha_q8b *h)
{
    if (!h) return 1;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    if (h->g_step) cudaGraphExecDestroy(h->g_step);
    void *ptrs[] = {h->d_file, h->bqkv, h->x, h->q, h->part, h->apart, h->logits, h->lx.q, h->lx.s, h->la.q,
                    h->la.s, h->lhq, h->lhs, h->lhead.q, h->lhead.s, h->kc, h->vc, h->kvs.k_hi, h->kvs.k_lo,
                    h->kvs.vt_hi, h->kvs.vt_lo, h->rope_cos, h->rope_sin, h->tok,
                    h->pos, h->slot, h->ntok, h->npos, h->nslot, h->proj_src, h->proj_dst, h->ident, h->next_index,
                    h->err, h->keys, h->st, h->params, h->out_tokens, h->out_count};
    for (void *p : ptrs)
        if (p) cudaFree(p);
    for (int l = 0; l < LAYERS; l++)
        for (Weights *w : {&h->w_qkv[l], &h->w_o[l], &h->w_gu[l], &h->w_down[l]}) {
            if (w->own_q) cudaFree(w->own_q);
            if (w->own_s) cudaFree(w->own_s);
        }
    for (cudaEvent_t e : h->ev)
        if (e) cudaEventDestroy(e);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
    return 0;
}

extern "C" int mocha_q8b_forward(mocha_q8b *h, int n, const int *tokens, const int *pos, const int *slots,
                                 int n_project, const int *project_rows, float *logits)
{
    if (!h || !rows_valid(h, n, tokens, pos, slots) || n_project < 0 || n_project > h->slots ||
        (n_project && !project_rows)) {
        fprintf(stderr, "mocha_q8b_forward: bad arguments\n");
        return 1;
    }
    for (int r = 0; r < n_project; r++)
        if (project_rows[r] < 0 || project_rows[r] >= n) {
            fprintf(stderr, "mocha_q8b_forward: projected row out of range\n");
            return 1;
        }
    QB_TRY(cudaSetDevice(h->device));
    if (upload_rows(h, n, tokens, pos, slots) || set_projection(h, n, n_project, project_rows)) return 1;
    const Rows r{h->tok, h->pos, h->slot};
    int max_pos = 0;
    for (int i = 0; i < n; i++) max_pos = std::max(max_pos, pos[i]);
    if (enqueue_forward(h, r, n, n <= h->slots, h->proj_dst, n_project, block_kind(n, pos, slots), max_pos)) return 1;
    if (logits && n_project)
        QB_TRY(cudaMemcpyAsync(logits, h->logits, sizeof(float) * VOCAB * n_project, cudaMemcpyDeviceToHost,
                               h->stream));
    QB_TRY(cudaStreamSynchronize(h->stream));
    return check_err(h);
}

extern "C" int mocha_q8b_prefill(mocha_q8b *h, int slot, const int *tokens, int n, float *logits)
{
    if (!h || slot < 0 || slot >= h->slots || !tokens || n < 1 || n > CONTEXT || n > h->max_rows) {
        fprintf(stderr, "mocha_q8b_prefill: bad arguments\n");
        return 1;
    }
    std::vector<int> pos(n), sl(n, slot);
    for (int i = 0; i < n; i++) pos[i] = i;
    const int last = n - 1;
    return mocha_q8b_forward(h, n, tokens, pos.data(), sl.data(), 1, &last, logits);
}

// The reference token loop for many sequences: sequences are served `slots` at a
// time; each wave prefills its prompts in one pass (rows of all its slots), samples
// the first token from the last prompt position, then runs n_new - 1 decode steps as
// one CUDA graph per step with tokens and positions kept on the device.
namespace qb {
namespace {

// Continuous batching: the first min(slots, max_rows / prompt_len) sequences take a slot
// each and are prefilled together; every decode step then advances all of those slots
// (one row per slot, a captured graph).  The host looks at the slots between runs of
// steps -- a run lasts until the first active sequence can have reached its token
// budget, at most kCheckEvery steps, so an EOS is noticed soon -- harvests every slot
// whose sequence has finished (EOS or n_new[i] tokens) and refills it at once with the
// next waiting sequence: that sequence's prompt rows run in one prompt pass (several
// refills share it), its first token goes to the slot's decode row (next_index), and
// the next step decodes it alongside the others.  Sampler state per slot: the last 64
// prompt tokens, seed seed_base + sequence index (src/minimind.cpp:160-179).
constexpr int kCheckEvery = 32;

int generate_impl(mocha_q8b *h, int nseq, const int *prompts, int prompt_len, const int *n_new, int max_new,
                  const mocha_sampling *sp, unsigned seed_base, int *out_tokens, int *out_counts, mocha_timing *timing)
{
    QB_TRY(cudaSetDevice(h->device));
    const int wave = std::min(h->slots, std::max(1, h->max_rows / prompt_len));
    if (wave < 1) return 1;
    if (h->out_stride < max_new) {
        if (h->out_tokens) cudaFree(h->out_tokens);
        h->out_tokens = nullptr;
        if (dalloc(&h->out_tokens, (size_t)h->slots * max_new)) return 1;
        h->out_stride = max_new;
    }
    for (int i = 0; i < nseq; i++)
        for (int j = 0; j < prompt_len; j++)
            if (prompts[(size_t)i * prompt_len + j] < 0 || prompts[(size_t)i * prompt_len + j] >= VOCAB) {
                fprintf(stderr, "mocha_q8b_generate: token id out of range\n");
                return 1;
            }
    sampling::Params prm{sp->repeat_penalty, sp->temperature, sp->top_k, sp->top_p, EOS, CONTROL_FIRST, VOCAB};
    QB_TRY(cudaMemcpyAsync(h->params, &prm, sizeof(prm), cudaMemcpyHostToDevice, h->stream));
    const int b = std::min(wave, nseq);        // slots stepped together
    std::vector<int> seq_of(b, -1);             // sequence in each slot, -1 free
    std::vector<sampling::SeqState> st(b);
    std::vector<int> counts(b), row;
    int next = 0;                               // next waiting sequence
    double prefill_s = 0, decode_s = 0;
    int generated = 0;
    float ms = 0;
    // fill the free slots with waiting sequences: one prompt pass over all their rows
    auto admit = [&]() -> int {
        std::vector<int> tok, pos, sl, src, idx;
        for (int i = 0; i < b && next < nseq; i++) {
            if (seq_of[i] >= 0) continue;
            const int q = next++;
            seq_of[i] = q;
            sampling::SeqState x;
            memset(&x, 0, sizeof x);
            const int *p = prompts + (size_t)q * prompt_len;
            const int from = std::max(0, prompt_len - sampling::kHistory);
            for (int j = from; j < prompt_len; j++) x.history[x.history_count++] = p[j];
            x.history_head = x.history_count % sampling::kHistory;
            x.seed = seed_base + (unsigned)q;
            x.last_token = p[prompt_len - 1];
            QB_TRY(cudaMemcpyAsync(h->st + i, &x, sizeof x, cudaMemcpyHostToDevice, h->stream));
            QB_TRY(cudaMemsetAsync(h->out_count + i, 0, sizeof(int), h->stream));
            for (int j = 0; j < prompt_len; j++) {
                tok.push_back(p[j]);
                pos.push_back(j);
                sl.push_back(i);
            }
            src.push_back((int)tok.size() - 1);
            idx.push_back(i);
        }
        if (src.empty()) return 0;
        const int n = (int)tok.size(), np = (int)src.size();
        if (upload_rows(h, n, tok.data(), pos.data(), sl.data()) || set_projection(h, n, np, src.data())) return 1;
        QB_TRY(cudaMemcpyAsync(h->next_index, idx.data(), sizeof(int) * np, cudaMemcpyHostToDevice, h->stream));
        QB_TRY(cudaEventRecord(h->ev[0], h->stream));
        const Rows pr{h->tok, h->pos, h->slot};
        if (enqueue_forward(h, pr, n, n <= h->slots, h->proj_dst, np,
                            prompt_len % TQ == 0 ? 2 : (prompt_len % QB == 0 ? 1 : 0), prompt_len - 1) ||
            enqueue_sample(h, pr, np, h->proj_src, h->next_index))
            return 1;
        QB_TRY(cudaEventRecord(h->ev[1], h->stream));
        QB_TRY(cudaEventSynchronize(h->ev[1]));  // idx and the row vectors are host temporaries
        QB_TRY(cudaEventElapsedTime(&ms, h->ev[0], h->ev[1]));
        prefill_s += ms * 1e-3;
        return 0;
    };
    if (admit()) return 1;
    if (capture_step(h, b)) return 1;
    for (;;) {
        QB_TRY(cudaMemcpy(counts.data(), h->out_count, sizeof(int) * b, cudaMemcpyDeviceToHost));
        QB_TRY(cudaMemcpy(st.data(), h->st, sizeof(sampling::SeqState) * b, cudaMemcpyDeviceToHost));
        if (check_err(h)) return 1;
        int run = kCheckEvery, active = 0;
        for (int i = 0; i < b; i++) {
            const int q = seq_of[i];
            if (q < 0) continue;
            if (st[i].finished || counts[i] >= n_new[q]) {  // harvest: tokens before EOS, at most n_new
                const int cnt = std::min(counts[i], n_new[q]);
                row.resize((size_t)std::max(cnt, 1));
                if (cnt > 0)
                    QB_TRY(cudaMemcpy(row.data(), h->out_tokens + (size_t)i * h->out_stride, sizeof(int) * cnt,
                                      cudaMemcpyDeviceToHost));
                int kept = 0;
                while (kept < cnt && row[kept] != EOS) kept++;
                memcpy(out_tokens + (size_t)q * max_new, row.data(), sizeof(int) * kept);
                out_counts[q] = kept;
                generated += kept;
                seq_of[i] = -1;
            } else {
                active++;
                run = std::min(run, n_new[q] - counts[i]);
            }
        }
        if (next < nseq) {
            const int before = next;
            if (admit()) return 1;
            active += next - before;
            if (next > before) run = 1;  // look again once the new sequences have a token
        }
        if (!active) break;
        QB_TRY(cudaEventRecord(h->ev[2], h->stream));
        for (int k = 0; k < std::max(run, 1); k++) QB_TRY(cudaGraphLaunch(h->g_step, h->stream));
        QB_TRY(cudaEventRecord(h->ev[3], h->stream));
        QB_TRY(cudaEventSynchronize(h->ev[3]));
        QB_TRY(cudaEventElapsedTime(&ms, h->ev[2], h->ev[3]));
        decode_s += ms * 1e-3;
    }
    if (timing) {
        timing->prefill_s = prefill_s;
        timing->decode_s = decode_s;
        timing->generated = generated;
    }
    return 0;
}

bool generate_args_ok(mocha_q8b *h, int nseq, const int *prompts, int prompt_len, const mocha_sampling *sp,
                      const int *out_tokens, const int *out_counts)
{
    return h && nseq >= 1 && prompts && prompt_len >= 1 && sp && out_tokens && out_counts && sp->top_k >= 1 &&
           sp->top_k <= sampling::kMaxK && sp->top_p > 0.f && sp->top_p <= 1.f && sp->temperature >= 0.f &&
           sp->repeat_penalty >= 1.f;
}

}  // namespace
}  // namespace qb

extern "C" int mocha_q8b_generate(mocha_q8b *h, int nseq, const int *prompts, int prompt_len, int n_new,
                                  const mocha_sampling *sp, unsigned seed_base, int *out_tokens, int *out_counts,
                                  mocha_timing *timing)
{
    if (!generate_args_ok(h, nseq, prompts, prompt_len, sp, out_tokens, out_counts) || n_new < 1 ||
        prompt_len + n_new > CONTEXT) {
        fprintf(stderr, "mocha_q8b_generate: bad arguments\n");
        return 1;
    }
    std::vector<int> each((size_t)nseq, n_new);
    return generate_impl(h, nseq, prompts, prompt_len, each.data(), n_new, sp, seed_base, out_tokens, out_counts,
                         timing);
}

extern "C" int mocha_q8b_generate_each(mocha_q8b *h, int nseq, const int *prompts, int prompt_len, const int *n_new,
                                       const mocha_sampling *sp, unsigned seed_base, int *out_tokens, int out_stride,
                                       int *out_counts, mocha_timing *timing)
{
    bool ok = generate_args_ok(h, nseq, prompts, prompt_len, sp, out_tokens, out_counts) && n_new && out_stride >= 1;
    for (int i = 0; ok && i < nseq; i++) ok = n_new[i] >= 1 && n_new[i] <= out_stride && prompt_len + n_new[i] <= CONTEXT;
    if (!ok) {
        fprintf(stderr, "mocha_q8b_generate_each: bad arguments\n");
        return 1;
    }
    return generate_impl(h, nseq, prompts, prompt_len, n_new, out_stride, sp, seed_base, out_tokens, out_counts,
                         timing);
}

extern "C" int mocha_q8b_launches_per_step(mocha_q8b *h)
{
    if (!h) return -1;
    return 1 + LAYERS * 8 + 1 + 2;  // embed+norm, 8 per layer, head GEMM, two sampler kernels
}

// Sampler check: the batched sampler on caller-supplied logits (n rows of VOCAB) with
// per-row history (64 ids each, counts) and seeds; writes the drawn tokens.
extern "C" int mocha_q8b_sample_check(mocha_q8b *h, int n, const float *logits, const int *history,
                                      const int *history_counts, const mocha_sampling *sp, const unsigned *seeds,
                                      int *tokens)
{
    if (!h || n < 1 || n > h->slots || !logits || !history || !history_counts || !sp || !seeds || !tokens ||
        sp->top_k < 1 || sp->top_k > sampling::kMaxK) {
        fprintf(stderr, "mocha_q8b_sample_check: bad arguments\n");
        return 1;
    }
    QB_TRY(cudaSetDevice(h->device));
    sampling::Params prm{sp->repeat_penalty, sp->temperature, sp->top_k, sp->top_p, EOS, CONTROL_FIRST, VOCAB};
    std::vector<sampling::SeqState> st(n);
    std::vector<int> rows(n), pos(n, 0);
    for (int i = 0; i < n; i++) {
        memset(&st[i], 0, sizeof st[i]);
        const int c = std::min(std::max(history_counts[i], 0), sampling::kHistory);
        for (int j = 0; j < c; j++) st[i].history[j] = history[(size_t)i * sampling::kHistory + j];
        st[i].history_count = c;
        st[i].history_head = c % sampling::kHistory;
        st[i].seed = seeds[i];
        rows[i] = i;
    }
    if (h->out_stride < 1) {
        if (dalloc(&h->out_tokens, (size_t)h->slots)) return 1;
        h->out_stride = 1;
    }
    QB_TRY(cudaMemcpyAsync(h->params, &prm, sizeof(prm), cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->st, st.data(), sizeof(sampling::SeqState) * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->logits, logits, sizeof(float) * VOCAB * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->slot, rows.data(), sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->pos, pos.data(), sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    QB_TRY(cudaMemcpyAsync(h->proj_src, rows.data(), sizeof(int) * n, cudaMemcpyHostToDevice, h->stream));
    const Rows r{h->tok, h->pos, h->slot};
    if (enqueue_sample(h, r, n, h->proj_src)) return 1;
    QB_TRY(cudaMemcpyAsync(tokens, h->ntok, sizeof(int) * n, cudaMemcpyDeviceToHost, h->stream));
    QB_TRY(cudaStreamSynchronize(h->stream));
    return 0;
}

// Device-timed prefill: `steps` passes (after `warmup`) of an n-token prompt of
// seeded random ids in slot 0 with the head on the last position; *ms = CUDA-event
// time of the timed passes.
extern "C" int mocha_q8b_bench_prefill(mocha_q8b *h, int n, unsigned seed, int warmup, int steps, float *ms)
{
    if (!h || n < 1 || n > CONTEXT || n > h->max_rows || warmup < 0 || steps < 1 || !ms) {
        fprintf(stderr, "mocha_q8b_bench_prefill: bad arguments\n");
        return 1;
    }
    QB_TRY(cudaSetDevice(h->device));
    std::vector<int> tok(n), pos(n), sl(n, 0);
    uint32_t s = seed ? seed : 1u;
    for (int i = 0; i < n; i++) {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        tok[i] = (int)(s % (uint32_t)VOCAB);
        pos[i] = i;
    }
    const int last = n - 1;
    if (upload_rows(h, n, tok.data(), pos.data(), sl.data()) || set_projection(h, n, 1, &last)) return 1;
    const Rows r{h->tok, h->pos, h->slot};
    const int block = n % TQ == 0 ? 2 : (n % QB == 0 ? 1 : 0);
    for (int i = 0; i < warmup; i++)
        if (enqueue_forward(h, r, n, n <= h->slots, h->proj_dst, 1, block, n - 1)) return 1;
    QB_TRY(cudaEventRecord(h->ev[0], h->stream));
    for (int i = 0; i < steps; i++)
        if (enqueue_forward(h, r, n, n <= h->slots, h->proj_dst, 1, block, n - 1)) return 1;
    QB_TRY(cudaEventRecord(h->ev[1], h->stream));
    QB_TRY(cudaEventSynchronize(h->ev[1]));
    QB_TRY(cudaEventElapsedTime(ms, h->ev[0], h->ev[1]));
    return check_err(h);
}
