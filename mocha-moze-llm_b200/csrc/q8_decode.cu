// Batch-1 grouped-Q8 decode step (Qwen2.5-0.5B) for B200, one kernel per phase.
//
// Phases per layer follow the reference forward (src/minimind.cu:67-113,
// src/minimind.cpp:51-82): RMSNorm -> Q/K/V GEMV + bias + split-half RoPE + KV write,
// split-K GQA attention, O GEMV + residual, RMSNorm -> gate/up GEMV + SwiGLU,
// down GEMV + residual; then final RMSNorm + tied vocabulary projection.
//
// Every phase spreads its rows over many CTAs (the reference runs the whole
// transformer in one CTA).  Weights stream from HBM with 16-byte evict-first loads,
// one warp per output row; activations stay fp32 and the int8 weights are widened
// exactly, so the only differences from the reference CPU path are summation order
// and the libm-vs-CUDA exp.  RoPE angles come from host tables computed with the
// CPU's own powf/cosf/sinf, so the rotation is bit-identical.
#include <math.h>

#include "mb_common.cuh"
#include "q8_decode.cuh"

namespace q8 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kQkvTasks = (DIM + 2 * KV) / 2;  // rows handled in RoPE pairs (i, i+32)
constexpr int kHeadBlocks = mb::kSMs * 4;

// Two grouped-Q8 row dots against the same shared-memory vector, loads of both rows
// issued before any arithmetic so each lane keeps 2*ceil(COLS/512) 16-byte loads in
// flight.  Lane l owns 16-weight chunks l, l+32, ...; each chunk lies inside one
// 64-weight scale group, so its partial dot is scaled once.
template <int COLS>
MB_DEV void row_dot2(const Mat a, int ra, const Mat b, int rb, const float *xs, int lane, float &da,
                     float &db)
{
    constexpr int CH = COLS / 16;
    constexpr int IT = (CH + 31) / 32;
    const int8_t *wa = a.w + (size_t)ra * COLS;
    const int8_t *wb = b.w + (size_t)rb * COLS;
    const float *sa = a.s + (size_t)ra * (COLS / GROUP);
    const float *sb = b.s + (size_t)rb * (COLS / GROUP);
    int4 va[IT], vb[IT];
    float ca[IT], cb[IT];
#pragma unroll
    for (int it = 0; it < IT; it++) {
        const int c = it * 32 + lane;
        if (c < CH) {
            va[it] = mb::ld_stream16(wa + c * 16);
            vb[it] = mb::ld_stream16(wb + c * 16);
            ca[it] = mb::ld_stream_f32(sa + (c >> 2));
            cb[it] = mb::ld_stream_f32(sb + (c >> 2));
        }
    }
    float acc_a = 0.f, acc_b = 0.f;
#pragma unroll
    for (int it = 0; it < IT; it++) {
        const int c = it * 32 + lane;
        if (c < CH) {
            acc_a = fmaf(mb::dot16_s8_f32(va[it], xs + c * 16), ca[it], acc_a);
            acc_b = fmaf(mb::dot16_s8_f32(vb[it], xs + c * 16), cb[it], acc_b);
        }
    }
    da = mb::warp_sum(acc_a);
    db = mb::warp_sum(acc_b);
}

template <int COLS>
MB_DEV float row_dot(const Mat a, int ra, const float *xs, int lane)
{
    constexpr int CH = COLS / 16;
    constexpr int IT = (CH + 31) / 32;
    const int8_t *wa = a.w + (size_t)ra * COLS;
    const float *sa = a.s + (size_t)ra * (COLS / GROUP);
    int4 va[IT];
    float ca[IT];
#pragma unroll
    for (int it = 0; it < IT; it++) {
        const int c = it * 32 + lane;
        if (c < CH) {
            va[it] = mb::ld_stream16(wa + c * 16);
            ca[it] = mb::ld_stream_f32(sa + (c >> 2));
        }
    }
    float acc = 0.f;
#pragma unroll
    for (int it = 0; it < IT; it++) {
        const int c = it * 32 + lane;
        if (c < CH) acc = fmaf(mb::dot16_s8_f32(va[it], xs + c * 16), ca[it], acc);
    }
    return mb::warp_sum(acc);
}

// y = (x * s) * g with s = 1/sqrt(sum(x^2)/DIM + eps), as src/minimind.cpp:47-50; the
// sum uses a fixed tree so every CTA derives the same bits.
MB_DEV void block_rmsnorm(const float *xs, const float *gain, float *ys, float *red)
{
    float ss = 0.f;
    for (int i = threadIdx.x; i < DIM; i += kThreads) ss = fmaf(xs[i], xs[i], ss);
    const float sum = mb::block_sum<kThreads>(ss, red);
    const float s = 1.0f / sqrtf(sum / DIM + RMS_EPS);
    for (int i = threadIdx.x; i < DIM; i += kThreads) ys[i] = xs[i] * s * __ldg(gain + i);
    __syncthreads();
}

MB_DEV void load_vec(float *dst, const float *src, int n)
{
    for (int i = threadIdx.x * 4; i < n; i += kThreads * 4)
        *reinterpret_cast<float4 *>(dst + i) = mb::ld_cg4(reinterpret_cast<const float4 *>(src + i));
    __syncthreads();
}

MB_DEV size_t kv_index(int layer, int kvh, int pos)
{
    return (((size_t)layer * KV_HEADS + kvh) * CONTEXT + pos) * HEAD_DIM;
}

// RMSNorm -> Q/K/V rows -> bias -> RoPE -> q buffer / KV cache.  Layer 0 also
// dequantises the embedding row of the input token (src/minimind.cu:70).
__global__ void __launch_bounds__(kThreads) k_qkv(const Model *__restrict__ M, Buffers b, int layer)
{
    __shared__ __align__(16) float xs[DIM];
    __shared__ __align__(16) float ns[DIM];
    __shared__ float red[kWarps];
    const Layer &L = M->layer[layer];
    const int pos = b.st->pos;
    if (layer == 0) {
        const int token = b.st->token;
        const int8_t *e = M->embed.w + (size_t)token * DIM;
        const float *es = M->embed.s + (size_t)token * (DIM / GROUP);
        for (int i = threadIdx.x; i < DIM; i += kThreads) {
            const float v = (float)e[i] * __ldg(es + i / GROUP);
            xs[i] = v;
            if (blockIdx.x == 0) b.x[i] = v;
        }
        __syncthreads();
    } else {
        load_vec(xs, b.x, DIM);
    }
    block_rmsnorm(xs, L.attn_norm, ns, red);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int task = blockIdx.x * kWarps + warp;
    if (task >= kQkvTasks) return;
    int kind, t;
    Mat m;
    const float *bias;
    if (task < DIM / 2) { kind = 0; t = task; m = L.q; bias = L.bq; }
    else if (task < DIM / 2 + KV / 2) { kind = 1; t = task - DIM / 2; m = L.k; bias = L.bk; }
    else { kind = 2; t = task - DIM / 2 - KV / 2; m = L.v; bias = L.bv; }
    const int head = t / 32, i = t % 32, r0 = head * HEAD_DIM + i;
    float d0, d1;
    row_dot2<DIM>(m, r0, m, r0 + 32, ns, lane, d0, d1);
    if (lane == 0) {
        d0 += __ldg(bias + r0);
        d1 += __ldg(bias + r0 + 32);
        if (kind == 2) {
            float *v = b.vc + kv_index(layer, head, pos);
            v[i] = d0;
            v[i + 32] = d1;
        } else {
            const float cs = __ldg(b.rope_cos + pos * 32 + i), sn = __ldg(b.rope_sin + pos * 32 + i);
            // unfused products, as the reference CPU evaluates them (src/minimind.cpp:64-66)
            const float lo = __fsub_rn(__fmul_rn(d0, cs), __fmul_rn(d1, sn));
            const float hi = __fadd_rn(__fmul_rn(d1, cs), __fmul_rn(d0, sn));
            if (kind == 0) {
                b.q[r0] = lo;
                b.q[r0 + 32] = hi;
            } else {
                float *k = b.kc + kv_index(layer, head, pos);
                k[i] = lo;
                k[i + 32] = hi;
            }
        }
    }
}

// Split-K GQA attention: CTA (chunk, kv head) scores ATTN_CHUNK positions for the
// seven query heads sharing the KV head and writes per-head (max, sum, acc[64]).
__global__ void __launch_bounds__(kThreads) k_attn(Buffers b, int layer)
{
    const int chunk = blockIdx.x, kvh = blockIdx.y;
    const int pos = b.st->pos;
    const int p0 = chunk * ATTN_CHUNK;
    if (p0 > pos) return;
    const int np = min(ATTN_CHUNK, pos + 1 - p0);
    __shared__ __align__(16) float qs[GQA][HEAD_DIM];
    __shared__ float ks[ATTN_CHUNK][HEAD_DIM + 1];
    __shared__ __align__(16) float vs[ATTN_CHUNK][HEAD_DIM];
    const float *kb = b.kc + kv_index(layer, kvh, p0);
    const float *vb = b.vc + kv_index(layer, kvh, p0);
    for (int i = threadIdx.x; i < GQA * HEAD_DIM; i += kThreads)
        qs[i / HEAD_DIM][i % HEAD_DIM] = mb::ld_cg(b.q + kvh * GQA * HEAD_DIM + i);
    for (int i = threadIdx.x; i < np * HEAD_DIM; i += kThreads) {
        ks[i / HEAD_DIM][i % HEAD_DIM] = mb::ld_cg(kb + i);
        vs[i / HEAD_DIM][i % HEAD_DIM] = mb::ld_cg(vb + i);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp >= GQA) return;
    float s = -INFINITY;
    if (lane < np) {
        float z = 0.f;
#pragma unroll 16
        for (int i = 0; i < HEAD_DIM; i++) z = fmaf(qs[warp][i], ks[lane][i], z);
        s = z * 0.125f;
    }
    const float m = mb::warp_max(s);
    const float e = lane < np ? expf(s - m) : 0.f;
    const float l = mb::warp_sum(e);
    float a0 = 0.f, a1 = 0.f;
    for (int p = 0; p < np; p++) {
        const float w = __shfl_sync(0xffffffffu, e, p);
        a0 = fmaf(w, vs[p][lane], a0);
        a1 = fmaf(w, vs[p][lane + 32], a1);
    }
    float *out = b.partial + ((size_t)(kvh * ATTN_MAX_CHUNKS + chunk) * GQA + warp) * ATTN_PARTIAL;
    if (lane == 0) {
        out[0] = m;
        out[1] = l;
    }
    out[2 + lane] = a0;
    out[2 + lane + 32] = a1;
}

// Combine the attention partials into the 896-wide head output, then O GEMV with the
// residual add (src/minimind.cu:107, add=true).
__global__ void __launch_bounds__(kThreads) k_oproj(const Model *__restrict__ M, Buffers b, int layer)
{
    __shared__ __align__(16) float os[DIM];
    const int pos = b.st->pos;
    const int nch = pos / ATTN_CHUNK + 1;
    constexpr int cstride = GQA * ATTN_PARTIAL;
    for (int idx = threadIdx.x; idx < DIM; idx += kThreads) {
        const int h = idx / HEAD_DIM, d = idx % HEAD_DIM, kvh = h / GQA, j = h % GQA;
        const float *p = b.partial + ((size_t)kvh * ATTN_MAX_CHUNKS * GQA + j) * ATTN_PARTIAL;
        float mx = -INFINITY;
        for (int c = 0; c < nch; c++) mx = fmaxf(mx, mb::ld_cg(p + c * cstride));
        float lsum = 0.f, acc = 0.f;
        for (int c = 0; c < nch; c++) {
            const float w = expf(mb::ld_cg(p + c * cstride) - mx);
            lsum = fmaf(w, mb::ld_cg(p + c * cstride + 1), lsum);
            acc = fmaf(w, mb::ld_cg(p + c * cstride + 2 + d), acc);
        }
        os[idx] = acc / lsum;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarps + warp;
    const float d = row_dot<DIM>(M->layer[layer].o, row, os, lane);
    if (lane == 0) b.x[row] = mb::ld_cg(b.x + row) + d;
}

// RMSNorm -> gate/up rows -> SwiGLU (src/minimind.cpp:76-77).
__global__ void __launch_bounds__(kThreads) k_gateup(const Model *__restrict__ M, Buffers b, int layer)
{
    __shared__ __align__(16) float xs[DIM];
    __shared__ __align__(16) float ns[DIM];
    __shared__ float red[kWarps];
    const Layer &L = M->layer[layer];
    load_vec(xs, b.x, DIM);
    block_rmsnorm(xs, L.ffn_norm, ns, red);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarps + warp;
    float g, u;
    row_dot2<DIM>(L.gate, row, L.up, row, ns, lane, g, u);
    if (lane == 0) b.h[row] = (g / (1.0f + expf(-g))) * u;
}

// down GEMV + residual (src/minimind.cu:109).
__global__ void __launch_bounds__(kThreads) k_down(const Model *__restrict__ M, Buffers b, int layer)
{
    __shared__ __align__(16) float hs[HIDDEN];
    load_vec(hs, b.h, HIDDEN);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarps + warp;
    const float d = row_dot<HIDDEN>(M->layer[layer].down, row, hs, lane);
    if (lane == 0) b.x[row] = mb::ld_cg(b.x + row) + d;
}

// Final RMSNorm (when NORM) and tied vocabulary projection, two rows per warp step.
template <bool NORM>
__global__ void __launch_bounds__(kThreads)
    k_head(Mat embed, const float *final_norm, const float *in, float *hidden, float *logits, int rows)
{
    __shared__ __align__(16) float xs[DIM];
    __shared__ __align__(16) float ns[DIM];
    __shared__ float red[kWarps];
    if (NORM) {
        load_vec(xs, in, DIM);
        block_rmsnorm(xs, final_norm, ns, red);
        if (blockIdx.x == 0)
            for (int i = threadIdx.x; i < DIM; i += kThreads) hidden[i] = ns[i];
    } else {
        load_vec(ns, in, DIM);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stride = gridDim.x * kWarps;
    int row = blockIdx.x * kWarps + warp;
    for (; row + stride < rows; row += 2 * stride) {
        float d0, d1;
        row_dot2<DIM>(embed, row, embed, row + stride, ns, lane, d0, d1);
        if (lane == 0) {
            logits[row] = d0;
            logits[row + stride] = d1;
        }
    }
    if (row < rows) {
        const float d = row_dot<DIM>(embed, row, ns, lane);
        if (lane == 0) logits[row] = d;
    }
}

}  // namespace

int forward_launches(bool project) { return LAYERS * 5 + (project ? 1 : 0); }

int enqueue_forward(const Model *dm, const Model &hm, const Buffers &b, bool project, cudaStream_t s)
{
    for (int l = 0; l < LAYERS; l++) {
        k_qkv<<<(kQkvTasks + kWarps - 1) / kWarps, kThreads, 0, s>>>(dm, b, l);
        k_attn<<<dim3(ATTN_MAX_CHUNKS, KV_HEADS), kThreads, 0, s>>>(b, l);
        k_oproj<<<DIM / kWarps, kThreads, 0, s>>>(dm, b, l);
        k_gateup<<<HIDDEN / kWarps, kThreads, 0, s>>>(dm, b, l);
        k_down<<<DIM / kWarps, kThreads, 0, s>>>(dm, b, l);
    }
    if (project)
        k_head<true><<<kHeadBlocks, kThreads, 0, s>>>(hm.embed, hm.final_norm, b.x, b.hidden, b.logits, VOCAB);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA forward launch: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

int enqueue_head_only(const Mat &embed, const float *hidden, float *logits, int rows, cudaStream_t s)
{
    k_head<false><<<kHeadBlocks, kThreads, 0, s>>>(embed, nullptr, hidden, nullptr, logits, rows);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA head launch: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

void fill_rope_tables(float *cos_table, float *sin_table, int context, int half, float theta)
{
    for (int pos = 0; pos < context; pos++) {
        for (int i = 0; i < half; i++) {
            const float angle = pos * powf(theta, -2.f * i / (2 * half));
            cos_table[pos * half + i] = cosf(angle);
            sin_table[pos * half + i] = sinf(angle);
        }
    }
}

}  // namespace q8
