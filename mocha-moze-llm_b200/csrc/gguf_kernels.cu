// GGUF Q4_K / Q6_K / Q8_0 repack, exact dequantisation and dequant-GEMV on B200.
//
// Dequantisation formulas follow the reference bridge (src/gguf-cuda.cu:28-44), built
// there with --fmad=false: Q4_K (d*sc)*q - dmin*m, Q6_K (d*sc)*(q-32), Q8_0 d*q.  The
// exact kernel (enqueue_dequant) evaluates them with round-to-nearest multiplies and
// subtractions, so its output is bit-identical to the oracle and to ggml.
//
// The GEMV factors each 16-weight chunk: sum_i w_i x_i = a * sum_i q_i x_i - b * sum_i x_i
// with a = d*sc, b = dmin*m (Q4_K) or b = 32*a (Q6_K), so the int->float widening is
// one byte-permute + one exact subtraction per weight and the sums of x per 16
// inputs are computed once per CTA.  One warp per output row, one 16-byte chunk of
// quants per lane per step, streamed with evict-first loads.
#include "gguf_kernels.cuh"
#include "mb_common.cuh"

namespace gguf {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

MB_DEV float half_bits_to_float(uint32_t h)
{
    const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    if (e == 0) {
        const float f = (float)m * 5.9604644775390625e-8f;
        return sign ? -f : f;
    }
    return __uint_as_float(sign | ((e == 31 ? 255u : e + 112u) << 23) | (m << 13));
}

// exact float of each unsigned byte (value < 256) of a word
MB_DEV float u8_lane(uint32_t w, uint32_t sel) { return __uint_as_float(__byte_perm(w, 0x4B000000u, sel)) - 8388608.0f; }

// sum_{k<16} u_k * x[k] for 16 unsigned byte values packed in 4 words
MB_DEV float dot16_u8(const uint32_t u[4], const float *x)
{
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 xv = x4[i];
        acc = fmaf(u8_lane(u[i], 0x7540), xv.x, acc);
        acc = fmaf(u8_lane(u[i], 0x7541), xv.y, acc);
        acc = fmaf(u8_lane(u[i], 0x7542), xv.z, acc);
        acc = fmaf(u8_lane(u[i], 0x7543), xv.w, acc);
    }
    return acc;
}

MB_DEV uint32_t byte_of(const int4 &v, int n)
{
    const uint32_t w = n < 4 ? (uint32_t)v.x : n < 8 ? (uint32_t)v.y : n < 12 ? (uint32_t)v.z : (uint32_t)v.w;
    return (w >> (8 * (n & 3))) & 0xffu;
}

// 6-bit scale and min of Q4_K sub-block j from the 12 packed bytes at header bytes 4..15
MB_DEV void q4k_scale_min(const int4 &hdr, int j, float &sc, float &mn)
{
    uint32_t s, m;
    if (j < 4) {
        s = byte_of(hdr, 4 + j) & 63u;
        m = byte_of(hdr, 8 + j) & 63u;
    } else {
        s = (byte_of(hdr, 8 + j) & 15u) | ((byte_of(hdr, j) >> 6) << 4);
        m = (byte_of(hdr, 8 + j) >> 4) | ((byte_of(hdr, 4 + j) >> 6) << 4);
    }
    sc = (float)s;
    mn = (float)m;
}

// x of this CTA's vector into shared memory plus its 16-element partial sums
MB_DEV void stage_x(const float *x, int cols, float *xs, float *x16)
{
    for (int i = threadIdx.x * 4; i < cols; i += kThreads * 4)
        *reinterpret_cast<float4 *>(xs + i) = *reinterpret_cast<const float4 *>(x + i);
    __syncthreads();
    for (int c = threadIdx.x; c < cols / 16; c += kThreads) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++) s += xs[c * 16 + k];
        x16[c] = s;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads)
    k_gemv_q4k(const uint8_t *__restrict__ body, int rows, int cols, const float *__restrict__ x, int x_stride,
               float *__restrict__ y, int y_stride, int accumulate)
{
    extern __shared__ __align__(16) float smem[];
    float *xs = smem, *x16 = smem + cols;
    stage_x(x + (size_t)blockIdx.y * x_stride, cols, xs, x16);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = cols / 256;
    for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    const uint8_t *rp = body + (size_t)row * nb * 144;
    float acc = 0.f;
    for (int qc = lane; qc < nb * 8; qc += 32) {
        const int blk = qc >> 3, c8 = qc & 7, part = c8 >> 1;
        const uint8_t *bp = rp + blk * 144;
        const int4 hdr = __ldg(reinterpret_cast<const int4 *>(bp));
        const int4 q = mb::ld_stream16(bp + 16 + c8 * 16);
        const float d = half_bits_to_float((uint32_t)hdr.x & 0xffffu);
        const float dmin = half_bits_to_float((uint32_t)hdr.x >> 16);
        float sc_lo, m_lo, sc_hi, m_hi;
        q4k_scale_min(hdr, 2 * part, sc_lo, m_lo);
        q4k_scale_min(hdr, 2 * part + 1, sc_hi, m_hi);
        const uint32_t w[4] = {(uint32_t)q.x, (uint32_t)q.y, (uint32_t)q.z, (uint32_t)q.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] = w[i] & 0x0F0F0F0Fu;
            hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
        const int e_lo = blk * 256 + part * 64 + (c8 & 1) * 16, e_hi = e_lo + 32;
        const float s_lo = dot16_u8(lo, xs + e_lo), s_hi = dot16_u8(hi, xs + e_hi);
        acc += (d * sc_lo) * s_lo - (dmin * m_lo) * x16[e_lo >> 4];
        acc += (d * sc_hi) * s_hi - (dmin * m_hi) * x16[e_hi >> 4];
    }
    acc = mb::warp_sum(acc);
    if (lane == 0) {
        float *out = y + (size_t)blockIdx.y * y_stride + row;
        *out = accumulate ? *out + acc : acc;
    }
    }
}

__global__ void __launch_bounds__(kThreads)
    k_gemv_q6k(const uint8_t *__restrict__ body, const uint16_t *__restrict__ dq, int rows, int cols,
               const float *__restrict__ x, int x_stride, float *__restrict__ y, int y_stride, int accumulate)
{
    extern __shared__ __align__(16) float smem[];
    float *xs = smem, *x16 = smem + cols;
    stage_x(x + (size_t)blockIdx.y * x_stride, cols, xs, x16);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = cols / 256;
    for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    float acc = 0.f;
    for (int qc = lane; qc < nb * 8; qc += 32) {
        const int blk = qc >> 3, c8 = qc & 7;
        const int half = c8 >> 2, g0 = (c8 >> 1) & 1, l0 = (c8 & 1) * 16;
        const size_t bi = (size_t)row * nb + blk;
        const uint8_t *bp = body + bi * 208;
        const int4 ql = mb::ld_stream16(bp + c8 * 16);
        const int4 qh = mb::ld_stream16(bp + 128 + half * 32 + l0);
        const int4 scv = __ldg(reinterpret_cast<const int4 *>(bp + 192));
        const float d = half_bits_to_float(__ldg(dq + bi));
        const int si = half * 8 + g0 * 2 + (l0 >> 4);
        const float sc_lo = (float)(int8_t)byte_of(scv, si), sc_hi = (float)(int8_t)byte_of(scv, si + 4);
        const uint32_t wl[4] = {(uint32_t)ql.x, (uint32_t)ql.y, (uint32_t)ql.z, (uint32_t)ql.w};
        const uint32_t wh[4] = {(uint32_t)qh.x, (uint32_t)qh.y, (uint32_t)qh.z, (uint32_t)qh.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] = (wl[i] & 0x0F0F0F0Fu) | (((wh[i] >> (2 * g0)) & 0x03030303u) << 4);
            hi[i] = ((wl[i] >> 4) & 0x0F0F0F0Fu) | (((wh[i] >> (2 * g0 + 4)) & 0x03030303u) << 4);
        }
        const int e_lo = blk * 256 + half * 128 + g0 * 32 + l0, e_hi = e_lo + 64;
        const float s_lo = dot16_u8(lo, xs + e_lo) - 32.f * x16[e_lo >> 4];
        const float s_hi = dot16_u8(hi, xs + e_hi) - 32.f * x16[e_hi >> 4];
        acc += (d * sc_lo) * s_lo + (d * sc_hi) * s_hi;
    }
    acc = mb::warp_sum(acc);
    if (lane == 0) {
        float *out = y + (size_t)blockIdx.y * y_stride + row;
        *out = accumulate ? *out + acc : acc;
    }
    }
}

__global__ void __launch_bounds__(kThreads)
    k_gemv_q80(const uint8_t *__restrict__ body, const uint16_t *__restrict__ dq, int rows, int cols,
               const float *__restrict__ x, int x_stride, float *__restrict__ y, int y_stride, int accumulate)
{
    extern __shared__ __align__(16) float smem[];
    float *xs = smem;
    for (int i = threadIdx.x * 4; i < cols; i += kThreads * 4)
        *reinterpret_cast<float4 *>(xs + i) =
            *reinterpret_cast<const float4 *>(x + (size_t)blockIdx.y * x_stride + i);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = cols / 32;
    for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
        const uint8_t *rp = body + (size_t)row * cols;
        float acc = 0.f;
        for (int c = lane; c < cols / 16; c += 32) {
            const int4 q = mb::ld_stream16(rp + c * 16);
            const float d = half_bits_to_float(__ldg(dq + (size_t)row * nb + (c >> 1)));
            acc = fmaf(d, mb::dot16_s8_f32(q, xs + c * 16), acc);
        }
        acc = mb::warp_sum(acc);
        if (lane == 0) {
            float *out = y + (size_t)blockIdx.y * y_stride + row;
            *out = accumulate ? *out + acc : acc;
        }
    }
}

// ---- fused multi-matrix GEMV for the GGUF engine -------------------------------------
//
// Up to three matrices that read the same input vector (q/k/v, gate/up) in one launch;
// optional RMSNorm of the input folded into the staging (every CTA normalises its own
// copy: sum of squares over the block, y = x * (1/sqrt(sum/cols + eps)) * gain), so the
// norm needs no launch of its own.  Rows of all matrices form one range; each warp
// dispatches on the type of the matrix its row belongs to.

// The staged input is stored swizzled: logical float e lives at 16-byte unit
// (e/4) ^ ((e/64) % 4) (an involution that permutes the four units of every aligned
// 16-float segment), so the 16-float segments that the lanes of a quarter warp read
// for Q4_K / Q6_K / Q8_0 chunks fall on different banks.
MB_DEV int swz(int e) { return ((((e >> 2) ^ ((e >> 6) & 3))) << 2) | (e & 3); }

// sum_{k<16} u_k * x[e0 + k] for a 16-aligned logical e0 of the swizzled input
MB_DEV float dot16_u8_swz(const uint32_t u[4], const float *xs, int e0)
{
    const float4 *x4 = reinterpret_cast<const float4 *>(xs + e0);
    const int k = (e0 >> 6) & 3;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 xv = x4[i ^ k];
        acc = fmaf(u8_lane(u[i], 0x7540), xv.x, acc);
        acc = fmaf(u8_lane(u[i], 0x7541), xv.y, acc);
        acc = fmaf(u8_lane(u[i], 0x7542), xv.z, acc);
        acc = fmaf(u8_lane(u[i], 0x7543), xv.w, acc);
    }
    return acc;
}

MB_DEV float dot16_s8_swz(int4 w, const float *xs, int e0)
{
    const float4 *x4 = reinterpret_cast<const float4 *>(xs + e0);
    const int k = (e0 >> 6) & 3;
    const uint32_t u[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u, (uint32_t)w.z ^ 0x80808080u,
                           (uint32_t)w.w ^ 0x80808080u};
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 xv = x4[i ^ k];
        acc = fmaf(mb::s8_lane(u[i], 0x7540), xv.x, acc);
        acc = fmaf(mb::s8_lane(u[i], 0x7541), xv.y, acc);
        acc = fmaf(mb::s8_lane(u[i], 0x7542), xv.z, acc);
        acc = fmaf(mb::s8_lane(u[i], 0x7543), xv.w, acc);
    }
    return acc;
}

MB_DEV float row_q4k(const uint8_t *rp, int nb, const float *xs, const float *x16, int lane)
{
    float acc = 0.f;
#pragma unroll 2
    for (int qc = lane; qc < nb * 8; qc += 32) {
        const int blk = qc >> 3, c8 = qc & 7, part = c8 >> 1;
        const uint8_t *bp = rp + blk * 144;
        const int4 hdr = __ldg(reinterpret_cast<const int4 *>(bp));
        const int4 q = mb::ld_stream16(bp + 16 + c8 * 16);
        const float d = half_bits_to_float((uint32_t)hdr.x & 0xffffu);
        const float dmin = half_bits_to_float((uint32_t)hdr.x >> 16);
        float sc_lo, m_lo, sc_hi, m_hi;
        q4k_scale_min(hdr, 2 * part, sc_lo, m_lo);
        q4k_scale_min(hdr, 2 * part + 1, sc_hi, m_hi);
        const uint32_t w[4] = {(uint32_t)q.x, (uint32_t)q.y, (uint32_t)q.z, (uint32_t)q.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] = w[i] & 0x0F0F0F0Fu;
            hi[i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
        const int e_lo = blk * 256 + part * 64 + (c8 & 1) * 16, e_hi = e_lo + 32;
        const float s_lo = dot16_u8_swz(lo, xs, e_lo), s_hi = dot16_u8_swz(hi, xs, e_hi);
        acc += (d * sc_lo) * s_lo - (dmin * m_lo) * x16[e_lo >> 4];
        acc += (d * sc_hi) * s_hi - (dmin * m_hi) * x16[e_hi >> 4];
    }
    return mb::warp_sum(acc);
}

MB_DEV float row_q6k(const uint8_t *body, const uint16_t *dq, int row, int nb, const float *xs, const float *x16,
                     int lane)
{
    float acc = 0.f;
#pragma unroll 2
    for (int qc = lane; qc < nb * 8; qc += 32) {
        const int blk = qc >> 3, c8 = qc & 7;
        const int half = c8 >> 2, g0 = (c8 >> 1) & 1, l0 = (c8 & 1) * 16;
        const size_t bi = (size_t)row * nb + blk;
        const uint8_t *bp = body + bi * 208;
        const int4 ql = mb::ld_stream16(bp + c8 * 16);
        const int4 qh = mb::ld_stream16(bp + 128 + half * 32 + l0);
        const int4 scv = __ldg(reinterpret_cast<const int4 *>(bp + 192));
        const float d = half_bits_to_float(__ldg(dq + bi));
        const int si = half * 8 + g0 * 2 + (l0 >> 4);
        const float sc_lo = (float)(int8_t)byte_of(scv, si), sc_hi = (float)(int8_t)byte_of(scv, si + 4);
        const uint32_t wl[4] = {(uint32_t)ql.x, (uint32_t)ql.y, (uint32_t)ql.z, (uint32_t)ql.w};
        const uint32_t wh[4] = {(uint32_t)qh.x, (uint32_t)qh.y, (uint32_t)qh.z, (uint32_t)qh.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo[i] = (wl[i] & 0x0F0F0F0Fu) | (((wh[i] >> (2 * g0)) & 0x03030303u) << 4);
            hi[i] = ((wl[i] >> 4) & 0x0F0F0F0Fu) | (((wh[i] >> (2 * g0 + 4)) & 0x03030303u) << 4);
        }
        const int e_lo = blk * 256 + half * 128 + g0 * 32 + l0, e_hi = e_lo + 64;
        const float s_lo = dot16_u8_swz(lo, xs, e_lo) - 32.f * x16[e_lo >> 4];
        const float s_hi = dot16_u8_swz(hi, xs, e_hi) - 32.f * x16[e_hi >> 4];
        acc += (d * sc_lo) * s_lo + (d * sc_hi) * s_hi;
    }
    return mb::warp_sum(acc);
}

MB_DEV float row_q80(const uint8_t *body, const uint16_t *dq, int row, int cols, const float *xs, int lane)
{
    const uint8_t *rp = body + (size_t)row * cols;
    const int nb = cols / 32;
    float acc = 0.f;
#pragma unroll 2
    for (int c = lane; c < cols / 16; c += 32) {
        const int4 q = mb::ld_stream16(rp + c * 16);
        const float d = half_bits_to_float(__ldg(dq + (size_t)row * nb + (c >> 1)));
        acc = fmaf(d, dot16_s8_swz(q, xs, c * 16), acc);
    }
    return mb::warp_sum(acc);
}

MB_DEV unsigned dev_row_bytes(int type, int cols)
{
    return type == Q4_K ? (unsigned)(cols / 256) * 144u : type == Q6_K ? (unsigned)(cols / 256) * 208u : (unsigned)cols;
}

constexpr int kMultiThreads = 512;
constexpr int kMultiWarps = kMultiThreads / 32;

__global__ void __launch_bounds__(kMultiThreads) k_gemv_multi(const MultiGemv g)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // This CTA's rows are one contiguous range; their weights do not depend on the
    // kernel ahead, so they are pulled into L2 while that kernel is still running.
    const int total = g.row_end[g.n - 1];
    const int per = (total + gridDim.x - 1) / gridDim.x;
    const int r_begin = blockIdx.x * per, r_end = min(total, r_begin + per);
    if (threadIdx.x < g.n) {
        const int i = threadIdx.x;
        const int start = i ? g.row_end[i - 1] : 0;
        const int a = max(r_begin, start), b = min(r_end, g.row_end[i]);
        if (a < b) {
            const unsigned rb = dev_row_bytes(g.m[i].type, g.cols);  // a multiple of 16
            const uint8_t *p0 = g.m[i].body + (size_t)(a - start) * rb;
            size_t left = (size_t)(b - a) * rb;
            // exactly the rows' bytes, in pieces of at most 32 KiB (skipped if unaligned)
            if (((uintptr_t)p0 & 15) == 0 && rb % 16 == 0)
                for (const uint8_t *q = p0; left > 0;) {
                    const unsigned n = (unsigned)(left < 32768 ? left : 32768);
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(n) : "memory");
                    q += n;
                    left -= n;
                }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    extern __shared__ __align__(16) float smem[];
    float *xs = smem, *x16 = smem + g.cols;
    __shared__ float red[kMultiWarps];
    const int cols = g.cols;
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < cols; i += kMultiThreads * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(g.x + i);
        *reinterpret_cast<float4 *>(xs + swz(i)) = v;
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
    if (g.gain) {
        ss = mb::warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kMultiWarps; w++) tot += red[w];
        const float sc = 1.0f / sqrtf(tot / cols + g.eps);
        for (int p = threadIdx.x; p < cols; p += kMultiThreads) xs[p] = xs[p] * sc * __ldg(g.gain + swz(p));
    }
    __syncthreads();
    // sums of 16 logical inputs: the swizzle only permutes within aligned 16-float segments
    for (int c = threadIdx.x; c < cols / 16; c += kMultiThreads) {
        float s16 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k++) s16 += xs[c * 16 + k];
        x16[c] = s16;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = r_begin + warp; r < r_end; r += kMultiWarps) {
        const int mi = r < g.row_end[0] ? 0 : (r < g.row_end[1] ? 1 : 2);
        const int row = r - (mi ? g.row_end[mi - 1] : 0);
        const DevMat &m = g.m[mi];
        float acc;
        if (m.type == Q4_K)
            acc = row_q4k(m.body + (size_t)row * (cols / 256) * 144, cols / 256, xs, x16, lane);
        else if (m.type == Q6_K)
            acc = row_q6k(m.body, m.d, row, cols / 256, xs, x16, lane);
        else
            acc = row_q80(m.body, m.d, row, cols, xs, lane);
        if (lane == 0) {
            float *out = g.y[mi] + row;
            *out = g.accumulate ? *out + acc : acc;
        }
    }
}

__global__ void k_repack_q6k(const uint8_t *__restrict__ raw, size_t nblocks, uint8_t *__restrict__ body,
                             uint16_t *__restrict__ dq)
{
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
        const uint8_t *s = raw + b * 210;
        uint8_t *t = body + b * 208;
        for (int i = 0; i < 208; i++) t[i] = s[i];
        dq[b] = (uint16_t)(s[208] | (s[209] << 8));
    }
}

__global__ void k_repack_q80(const uint8_t *__restrict__ raw, size_t nblocks, uint8_t *__restrict__ body,
                             uint16_t *__restrict__ dq)
{
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
        const uint8_t *s = raw + b * 34;
        dq[b] = (uint16_t)(s[0] | (s[1] << 8));
        for (int i = 0; i < 32; i++) body[b * 32 + i] = s[2 + i];
    }
}

// exact dequantisation, one thread per weight
__global__ void k_dequant(DevMat m, float *__restrict__ out)
{
    const size_t n = (size_t)m.rows * m.cols;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const size_t r = e / m.cols;
        const int c = (int)(e % m.cols);
        float v;
        if (m.type == Q8_0) {
            const int nb = m.cols / 32;
            const float d = half_bits_to_float(m.d[r * nb + c / 32]);
            v = __fmul_rn(d, (float)(int8_t)m.body[r * m.cols + c]);
        } else if (m.type == Q4_K) {
            const int nb = m.cols / 256, blk = c / 256, i = c & 255, j = i / 32;
            const uint8_t *p = m.body + (r * nb + blk) * 144;
            const float d = half_bits_to_float(p[0] | (p[1] << 8)), dmin = half_bits_to_float(p[2] | (p[3] << 8));
            const uint8_t *s = p + 4;
            uint32_t sc, mn;
            if (j < 4) {
                sc = s[j] & 63u;
                mn = s[j + 4] & 63u;
            } else {
                sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
                mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
            }
            uint32_t q = p[16 + (i / 64) * 32 + (i & 31)];
            q = (j & 1) ? q >> 4 : q & 15u;
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
        } else {
            const int nb = m.cols / 256, blk = c / 256, i = c & 255;
            const size_t bi = r * nb + blk;
            const uint8_t *p = m.body + bi * 208;
            const int half = i / 128, g = (i & 127) / 32, l = i & 31;
            uint32_t lo = p[half * 64 + (g & 1) * 32 + l];
            lo = g < 2 ? lo & 15u : lo >> 4;
            const uint32_t hi = (p[128 + half * 32 + l] >> (2 * g)) & 3u;
            const int q = (int)(lo | (hi << 4)) - 32;
            const int sc = (int8_t)p[192 + i / 16];
            v = __fmul_rn(__fmul_rn(half_bits_to_float(m.d[bi]), (float)sc), (float)q);
        }
        out[e] = v;
    }
}

// row `*row_index` of m, dequantised exactly (same formulas as k_dequant)
__global__ void k_dequant_row(DevMat m, const int *__restrict__ row_index, float *__restrict__ out)
{
    const size_t r = (size_t)*row_index;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < m.cols; c += gridDim.x * blockDim.x) {
        float v;
        if (m.type == Q8_0) {
            const int nb = m.cols / 32;
            v = __fmul_rn(half_bits_to_float(m.d[r * nb + c / 32]), (float)(int8_t)m.body[r * m.cols + c]);
        } else if (m.type == Q4_K) {
            const int nb = m.cols / 256, blk = c / 256, i = c & 255, j = i / 32;
            const uint8_t *p = m.body + (r * nb + blk) * 144;
            const float d = half_bits_to_float(p[0] | (p[1] << 8)), dmin = half_bits_to_float(p[2] | (p[3] << 8));
            const uint8_t *s = p + 4;
            uint32_t sc, mn;
            if (j < 4) {
                sc = s[j] & 63u;
                mn = s[j + 4] & 63u;
            } else {
                sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
                mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
            }
            uint32_t q = p[16 + (i / 64) * 32 + (i & 31)];
            q = (j & 1) ? q >> 4 : q & 15u;
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
        } else {
            const int nb = m.cols / 256, blk = c / 256, i = c & 255;
            const size_t bi = r * nb + blk;
            const uint8_t *p = m.body + bi * 208;
            const int half = i / 128, g = (i & 127) / 32, l = i & 31;
            uint32_t lo = p[half * 64 + (g & 1) * 32 + l];
            lo = g < 2 ? lo & 15u : lo >> 4;
            const uint32_t hi = (p[128 + half * 32 + l] >> (2 * g)) & 3u;
            const int q = (int)(lo | (hi << 4)) - 32;
            v = __fmul_rn(__fmul_rn(half_bits_to_float(m.d[bi]), (float)(int8_t)p[192 + i / 16]), (float)q);
        }
        out[c] = v;
    }
}

int launch_ok(const char *what)
{
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA %s: %d %s\n", what, (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

}  // namespace

DevMat make_devmat(int type, int rows, int cols, uint8_t *dst)
{
    DevMat m{type, rows, cols, dst, nullptr};
    if (type == Q6_K) m.d = reinterpret_cast<const uint16_t *>(dst + (size_t)rows * (cols / 256) * 208);
    if (type == Q8_0) m.d = reinterpret_cast<const uint16_t *>(dst + (size_t)rows * cols);
    return m;
}

int enqueue_repack(int type, const uint8_t *raw, int rows, int cols, uint8_t *dst, cudaStream_t s)
{
    const size_t bytes = dev_bytes(type, rows, cols);
    if (!bytes) return 1;
    if (type == Q4_K) {
        if (raw != dst && cudaMemcpyAsync(dst, raw, bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess) return 1;
        return 0;
    }
    DevMat m = make_devmat(type, rows, cols, dst);
    if (type == Q6_K) {
        const size_t nblocks = (size_t)rows * (cols / 256);
        k_repack_q6k<<<mb::kSMs * 4, 256, 0, s>>>(raw, nblocks, dst, const_cast<uint16_t *>(m.d));
    } else {
        const size_t nblocks = (size_t)rows * (cols / 32);
        k_repack_q80<<<mb::kSMs * 4, 256, 0, s>>>(raw, nblocks, dst, const_cast<uint16_t *>(m.d));
    }
    return launch_ok("gguf repack");
}

int enqueue_dequant_row(const DevMat &m, const int *row_index, float *out, cudaStream_t s)
{
    k_dequant_row<<<(m.cols + 255) / 256, 256, 0, s>>>(m, row_index, out);
    return launch_ok("gguf dequant row");
}

int enqueue_dequant(const DevMat &m, float *out, cudaStream_t s)
{
    k_dequant<<<mb::kSMs * 8, 256, 0, s>>>(m, out);
    return launch_ok("gguf dequant");
}

int enqueue_gemv(const DevMat &m, const float *x, int vectors, int x_stride_f, float *y, int y_stride_f,
                 cudaStream_t s, bool accumulate)
{
    if (vectors < 1 || vectors > 65535 || m.cols % 256 || m.cols <= 0 || m.rows <= 0) return 1;
    const size_t smem = (size_t)(m.cols + (m.type == Q8_0 ? 0 : m.cols / 16)) * sizeof(float);
    if (smem > 200 * 1024) return 1;
    static bool configured[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 1;
    if (!configured[dev]) {
        const int lim = 200 * 1024;
        if (cudaFuncSetAttribute(k_gemv_q4k, cudaFuncAttributeMaxDynamicSharedMemorySize, lim) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_q6k, cudaFuncAttributeMaxDynamicSharedMemorySize, lim) != cudaSuccess ||
            cudaFuncSetAttribute(k_gemv_q80, cudaFuncAttributeMaxDynamicSharedMemorySize, lim) != cudaSuccess)
            return 1;
        configured[dev] = true;
    }
    // enough CTAs to fill the GPU a few times over; each CTA stages x once and walks rows
    const int row_blocks = (m.rows + kWarps - 1) / kWarps;
    const dim3 grid(row_blocks < mb::kSMs * 8 ? row_blocks : mb::kSMs * 8, vectors);
    const int acc = accumulate ? 1 : 0;
    if (m.type == Q4_K)
        k_gemv_q4k<<<grid, kThreads, smem, s>>>(m.body, m.rows, m.cols, x, x_stride_f, y, y_stride_f, acc);
    else if (m.type == Q6_K)
        k_gemv_q6k<<<grid, kThreads, smem, s>>>(m.body, m.d, m.rows, m.cols, x, x_stride_f, y, y_stride_f, acc);
    else if (m.type == Q8_0)
        k_gemv_q80<<<grid, kThreads, smem, s>>>(m.body, m.d, m.rows, m.cols, x, x_stride_f, y, y_stride_f, acc);
    else
        return 1;
    return launch_ok("gguf gemv");
}

int enqueue_gemv_multi(const MultiGemv &g, cudaStream_t s)
{
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || g.n < 1 || g.n > 3 || g.cols <= 0 || g.cols % 256) return 1;
    for (int i = 0; i < g.n; i++)
        if (g.m[i].cols != g.cols || (i && g.row_end[i] < g.row_end[i - 1])) return 1;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(k_gemv_multi, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
            cudaSuccess)
            return 1;
        configured[dev] = true;
    }
    const int total = g.row_end[g.n - 1];
    const int blocks = (total + kMultiWarps - 1) / kMultiWarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks < mb::kSMs * 2 ? blocks : mb::kSMs * 2);
    cfg.blockDim = dim3(kMultiThreads);
    cfg.dynamicSmemBytes = sizeof(float) * (g.cols + g.cols / 16);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_gemv_multi, g) != cudaSuccess) return launch_ok("gguf fused gemv");
    return 0;
}

}  // namespace gguf
