// Persistent batch-1 decode step for the grouped-Q8 model on B200.
//
// One cooperative launch of 148 CTAs (one per SM) runs the whole token:
//   * warp 0 of every CTA streams that CTA's weights -- laid out at set-up as one
//     contiguous region per CTA, in the order the CTA consumes them -- through a
//     5-slot shared-memory ring with cp.async.bulk copies completed on mbarriers.
//     Weights do not depend on activations, so the stream runs ahead of the
//     dependency chain by up to the ring depth (~1.7 layers).
//   * warps 1..8 walk the token's phases: per layer QKV(+bias, RoPE, KV write),
//     split-K attention (last unit per KV head combines), O + residual,
//     RMSNorm -> gate/up + SwiGLU, down + residual; then the final norm, the tied
//     vocabulary head fused with the repetition penalty, control mask and per-CTA
//     top-k, and -- in the last CTA to finish -- the merge and the token draw.
//   * phases are separated by epoch-tagged global counters; every wait is bounded
//     (about two seconds of clock cycles) and sets an error word instead of hanging.
// The arithmetic is the reference's (src/minimind.cu:67-123, src/minimind.cpp:51-82):
// fp32 activations, int8 weights widened exactly, one fp32 scale per 64 weights.
#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "mb_common.cuh"
#include "q8_persistent.cuh"
#include "sampling_dev.cuh"

namespace q8p {
namespace {

using namespace q8;
constexpr int kNT = kConsumerWarps * 32;
constexpr long long kTimeoutCycles = 4000000000LL;
constexpr int kMaxChunks = CONTEXT / kAttnChunk;
constexpr int kQkvPairs = (DIM + 2 * KV) / 2;  // 576
constexpr int kGateupPerChunk = 19;            // pairs (38 rows of 896)
constexpr int kHeadPerChunk = 38;              // rows
constexpr int kHeadSlice = 1040;               // >= ceil(VOCAB / kCTAs)

struct Smem {
    uint8_t ring[kSlots][kSlotBytes];
    __align__(16) float xs[DIM];
    __align__(16) float ns[DIM];
    union __align__(16) {
        float hs[HIDDEN];
        struct {
            float q[GQA][HEAD_DIM];
            float k[kAttnChunk][HEAD_DIM + 1];
            float v[kAttnChunk][HEAD_DIM];
        } att;
        float hl[kHeadSlice];
    } u;
    float red[kConsumerWarps][8];
    unsigned long long full[kSlots], empty[kSlots];
    int flag;
    int token, pos;
    volatile int issued;         // chunks the producer has started copying
    volatile int producer_done;  // the producer has left its loop
};

// ---- low-level primitives --------------------------------------------------

MB_DEV uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

MB_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kNT) : "memory"); }

MB_DEV void mbar_init(unsigned long long *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

MB_DEV void mbar_expect_tx(unsigned long long *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

MB_DEV void mbar_arrive(unsigned long long *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

MB_DEV bool mbar_test(unsigned long long *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

MB_DEV unsigned ld_acquire(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

MB_DEV unsigned ld_volatile(const unsigned *p) { return *(const volatile unsigned *)p; }

MB_DEV void fail(Sync *sy, unsigned *host_error, unsigned code)
{
    atomicCAS(&sy->error, 0u, code);
    *(volatile unsigned *)host_error = code;
    __threadfence_system();
}

// Bounded wait on an mbarrier phase; false (and the error word set) on timeout or
// when another CTA already failed.
MB_DEV bool mbar_wait(unsigned long long *bar, uint32_t parity, Sync *sy, unsigned *host_error)
{
    if (mbar_test(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_test(bar, parity)) return true;
        if (ld_volatile(&sy->error)) return false;
        if (clock64() - t0 > kTimeoutCycles) {
            fail(sy, host_error, 2);
            return false;
        }
    }
}

MB_DEV void bulk_load(void *dst, const void *src, uint32_t bytes, unsigned long long *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(mb::evict_first_policy())
        : "memory");
}

// ---- consumer-side helpers --------------------------------------------------

struct Ctx {
    Smem &S;
    Sync *sy;
    unsigned *host_error;
    int ct, cw, lane;
    unsigned target;
};

// all consumer threads return the same verdict
MB_DEV bool gwait(Ctx &c, const unsigned *cnt)
{
    if (c.ct == 0) {
        int ok = 1;
        if (ld_acquire(cnt) < c.target) {
            const long long t0 = clock64();
            while (ld_acquire(cnt) < c.target) {
                if (ld_volatile(&c.sy->error)) { ok = 0; break; }
                if (clock64() - t0 > kTimeoutCycles) {
                    fail(c.sy, c.host_error, 1);
                    ok = 0;
                    break;
                }
            }
        }
        c.S.flag = ok;
    }
    cbar();
    return c.S.flag != 0;
}

MB_DEV void gsignal(Ctx &c, unsigned *cnt)
{
    cbar();
    if (c.ct == 0) {
        __threadfence();
        atomicAdd(cnt, 1u);
    }
}

MB_DEV void load_vec_cg(float *dst, const float *src, int n, int ct)
{
    for (int i = ct * 4; i < n; i += kNT * 4)
        *reinterpret_cast<float4 *>(dst + i) = __ldcg(reinterpret_cast<const float4 *>(src + i));
}

// y = (x * s) * g, s = 1/sqrt(sum(x^2)/DIM + eps); identical bits in every CTA
MB_DEV void rmsnorm(Ctx &c, const float *xs, const float *gain, float *ns)
{
    float ss = 0.f;
    for (int i = c.ct; i < DIM; i += kNT) ss = fmaf(xs[i], xs[i], ss);
    ss = mb::warp_sum(ss);
    if (c.lane == 0) c.S.red[c.cw][0] = ss;
    cbar();
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) sum += c.S.red[w][0];
    const float s = 1.0f / sqrtf(sum / DIM + RMS_EPS);
    for (int i = c.ct; i < DIM; i += kNT) ns[i] = xs[i] * s * __ldg(gain + i);
    cbar();
}

// 16 int8 weights (smem) . 16 fp32 inputs held in registers
MB_DEV float dot16r(const int4 w, const float *xr)
{
    const uint32_t u[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u, (uint32_t)w.z ^ 0x80808080u,
                           (uint32_t)w.w ^ 0x80808080u};
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        acc = fmaf(mb::s8_lane(u[i], 0x7540), xr[4 * i + 0], acc);
        acc = fmaf(mb::s8_lane(u[i], 0x7541), xr[4 * i + 1], acc);
        acc = fmaf(mb::s8_lane(u[i], 0x7542), xr[4 * i + 2], acc);
        acc = fmaf(mb::s8_lane(u[i], 0x7543), xr[4 * i + 3], acc);
    }
    return acc;
}

// A 896-wide row: lane owns 16-weight chunks lane and lane+32 (< 56); its 32 inputs
// live in registers for every row of the phase.
MB_DEV void load_x896(const float *ns, int lane, float *xr)
{
#pragma unroll
    for (int i = 0; i < 16; i++) xr[i] = ns[lane * 16 + i];
#pragma unroll
    for (int i = 0; i < 16; i++) xr[16 + i] = lane < 24 ? ns[(lane + 32) * 16 + i] : 0.f;
}

MB_DEV float row896(const uint8_t *w_row, const float *s_row, const float *xr, int lane)
{
    const int4 a = *reinterpret_cast<const int4 *>(w_row + lane * 16);
    float acc = dot16r(a, xr) * s_row[lane >> 2];
    if (lane < 24) {
        const int4 b = *reinterpret_cast<const int4 *>(w_row + (lane + 32) * 16);
        acc = fmaf(dot16r(b, xr + 16), s_row[(lane + 32) >> 2], acc);
    }
    return mb::warp_sum(acc);
}

MB_DEV size_t kv_index(int layer, int kvh, int pos)
{
    return (((size_t)layer * KV_HEADS + kvh) * CONTEXT + pos) * HEAD_DIM;
}

// ---- the kernel ---------------------------------------------------------------

struct Args {
    const Model *M;
    const Plan *P;
    Buffers b;
    Sync *sy;
    Scratch scr;
    int mode;
    const sampling::Params *prm;
    sampling::SeqState *seq;
    int *out_ring, *out_count;
    const int *prompt;
    unsigned *host_error;
};

struct Cursor {
    uint32_t i, end, k;
};

// Wait for the next chunk of the stream; returns its slot data or null on failure.
MB_DEV const uint8_t *take(Ctx &c, const Args &a, Cursor &cur, uint32_t kind, const Chunk *&ch)
{
    if (cur.i >= cur.end) {
        if (c.ct == 0) fail(c.sy, c.host_error, 3);
        return nullptr;
    }
    ch = &a.P->chunks[cur.i];
    if (ch->kind != kind) {
        if (c.ct == 0) fail(c.sy, c.host_error, 4);
        return nullptr;
    }
    const uint32_t slot = cur.k % kSlots, use = cur.k / kSlots;
    if (!mbar_wait(&c.S.full[slot], use & 1, c.sy, c.host_error)) return nullptr;
    return c.S.ring[slot];
}

MB_DEV void give_back(Ctx &c, Cursor &cur)
{
    cbar();
    if (c.ct == 0) mbar_arrive(&c.S.empty[cur.k % kSlots]);
    cur.i++;
    cur.k++;
}

MB_DEV bool next_is(const Args &a, const Cursor &cur, uint32_t kind, uint32_t layer)
{
    if (cur.i >= cur.end) return false;
    const Chunk &ch = a.P->chunks[cur.i];
    return ch.kind == kind && ch.layer == layer;
}

MB_DEV void attention_unit(Ctx &c, const Args &a, int layer, int pos, int nch, int unit)
{
    Smem &S = c.S;
    const int kvh = unit / nch, ch = unit % nch;
    const int p0 = ch * kAttnChunk, np = min(kAttnChunk, pos + 1 - p0);
    const float *kb = a.b.kc + kv_index(layer, kvh, p0);
    const float *vb = a.b.vc + kv_index(layer, kvh, p0);
    for (int i = c.ct; i < GQA * HEAD_DIM; i += kNT)
        S.u.att.q[i / HEAD_DIM][i % HEAD_DIM] = __ldcg(a.b.q + kvh * GQA * HEAD_DIM + i);
    for (int i = c.ct; i < np * HEAD_DIM; i += kNT) {
        S.u.att.k[i / HEAD_DIM][i % HEAD_DIM] = __ldcg(kb + i);
        S.u.att.v[i / HEAD_DIM][i % HEAD_DIM] = __ldcg(vb + i);
    }
    cbar();
    if (c.cw < GQA) {
        const int j = c.cw, lane = c.lane;
        float s = -INFINITY;
        if (lane < np) {
            float z = 0.f;
#pragma unroll 16
            for (int i = 0; i < HEAD_DIM; i++) z = fmaf(S.u.att.q[j][i], S.u.att.k[lane][i], z);
            s = z * 0.125f;
        }
        const float m = mb::warp_max(s);
        const float e = lane < np ? expf(s - m) : 0.f;
        const float l = mb::warp_sum(e);
        float a0 = 0.f, a1 = 0.f;
        for (int p = 0; p < np; p++) {
            const float w = __shfl_sync(0xffffffffu, e, p);
            a0 = fmaf(w, S.u.att.v[p][lane], a0);
            a1 = fmaf(w, S.u.att.v[p][lane + 32], a1);
        }
        float *out = a.scr.partial + ((size_t)(kvh * kMaxChunks + ch) * GQA + j) * ATTN_PARTIAL;
        if (lane == 0) {
            out[0] = m;
            out[1] = l;
        }
        out[2 + lane] = a0;
        out[2 + lane + 32] = a1;
    }
    cbar();
    if (c.ct == 0) {
        __threadfence();
        const unsigned t = atomicAdd(&c.sy->tickets[layer][kvh], 1u);
        S.flag = t == (unsigned)(nch - 1);
        if (S.flag) atomicExch(&c.sy->tickets[layer][kvh], 0u);
    }
    cbar();
    if (S.flag) {
        __threadfence();
        constexpr int cstride = GQA * ATTN_PARTIAL;
        for (int idx = c.ct; idx < GQA * HEAD_DIM; idx += kNT) {
            const int j = idx / HEAD_DIM, d = idx % HEAD_DIM;
            const float *p = a.scr.partial + ((size_t)kvh * kMaxChunks * GQA + j) * ATTN_PARTIAL;
            float mx = -INFINITY;
            for (int q = 0; q < nch; q++) mx = fmaxf(mx, __ldcg(p + q * cstride));
            float lsum = 0.f, acc = 0.f;
            for (int q = 0; q < nch; q++) {
                const float w = expf(__ldcg(p + q * cstride) - mx);
                lsum = fmaf(w, __ldcg(p + q * cstride + 1), lsum);
                acc = fmaf(w, __ldcg(p + q * cstride + 2 + d), acc);
            }
            a.scr.o[kvh * GQA * HEAD_DIM + idx] = acc / lsum;
        }
    }
    cbar();
}

// descending bitonic sort of n (power of two) keys by the consumer threads
MB_DEV void bitonic_desc(unsigned long long *keys, int n, int ct)
{
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = ct; t < n / 2; t += kNT) {
                const int i = 2 * t - (t & (stride - 1)), j = i + stride;
                const unsigned long long x = keys[i], y = keys[j];
                if (((i & size) == 0) ? (x < y) : (x > y)) {
                    keys[i] = y;
                    keys[j] = x;
                }
            }
            cbar();
        }
    }
}

MB_DEV unsigned long long block_max(Ctx &c, unsigned long long v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    unsigned long long *r = reinterpret_cast<unsigned long long *>(&c.S.red[0][0]);
    if (c.lane == 0) r[c.cw] = v;
    cbar();
    unsigned long long best = 0ull;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) best = r[w] > best ? r[w] : best;
    cbar();
    return best;
}

// Error exit of the consumers: wait (bounded) until the producer has stopped and
// every bulk copy it started into this CTA's ring has landed, so no copy is still
// writing shared memory when the CTA exits.
MB_DEV void drain(Ctx &c, const Cursor &cur)
{
    if (c.ct == 0) {
        const long long t0 = clock64();
        while (!c.S.producer_done && clock64() - t0 < kTimeoutCycles) {
        }
        const int issued = c.S.issued;
        for (int k = (int)cur.k; k < issued; k++) {
            const long long t1 = clock64();
            while (!mbar_test(&c.S.full[k % kSlots], (k / kSlots) & 1) && clock64() - t1 < kTimeoutCycles) {
            }
        }
    }
    cbar();
}

__global__ void __launch_bounds__(kThreads, 1) k_step(Args a)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem &S = *reinterpret_cast<Smem *>(smem_raw);
    const int cta = blockIdx.x;
    const unsigned epoch = ld_volatile(&a.sy->epoch);
    const bool project = a.mode == FORWARD_PROJECT || a.mode == DECODE;
    const bool decode = a.mode == DECODE;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.token = ld_volatile((const unsigned *)&a.b.st->token);
        S.pos = ld_volatile((const unsigned *)&a.b.st->pos);
        S.issued = 0;
        S.producer_done = 0;
        S.flag = 0;
        const bool bad = S.token < 0 || S.token >= VOCAB || S.pos < 0 || S.pos >= CONTEXT ||
                         (a.mode == PREFILL && S.pos + 1 >= CONTEXT);
        if (bad) {
            fail(a.sy, a.host_error, 5);
            S.flag = -1;
        }
    }
    __syncthreads();
    if (S.flag < 0) return;  // invalid token / position: nothing was issued
    const uint32_t c0 = a.P->chunk_begin[cta], c1 = a.P->chunk_begin[cta + 1];

    if (threadIdx.x < 32) {  // ---- producer warp: stream this CTA's weights
        if (threadIdx.x == 0) {
            uint32_t k = 0;
            for (uint32_t i = c0; i < c1 && S.flag >= 0; i++) {
                const Chunk ch = a.P->chunks[i];
                if (ch.kind == HEAD && !project) continue;
                const uint32_t slot = k % kSlots, use = k / kSlots;
                if (use > 0 && !mbar_wait(&S.empty[slot], (use - 1) & 1, a.sy, a.host_error)) break;
                if (ld_volatile(&a.sy->error)) break;
                mbar_expect_tx(&S.full[slot], ch.bytes);
                bulk_load(S.ring[slot], a.P->stream + ch.off, ch.bytes, &S.full[slot]);
                k++;
                S.issued = (int)k;
            }
            __threadfence_block();
            S.producer_done = 1;
        }
        return;
    }

    Ctx c{S, a.sy, a.host_error, (int)threadIdx.x - 32, ((int)threadIdx.x - 32) >> 5, (int)threadIdx.x & 31,
          (epoch + 1) * kCTAs};
    const int pos = S.pos;
    Cursor cur{c0, c1, 0};
    const Model *M = a.M;
    float xr[32];

    for (int l = 0; l < LAYERS; l++) {
        const Layer &L = M->layer[l];
        // ---- QKV + bias + RoPE + KV write
        if (l == 0) {
            const int token = S.token;
            const int8_t *e = M->embed.w + (size_t)token * DIM;
            const float *es = M->embed.s + (size_t)token * (DIM / GROUP);
            for (int i = c.ct; i < DIM; i += kNT) {
                const float v = (float)e[i] * __ldg(es + i / GROUP);
                S.xs[i] = v;
                if (cta == 0) a.b.x[i] = v;
            }
        } else {
            if (!gwait(c, &a.sy->counters[l - 1][PH_DOWN])) return drain(c, cur);
            load_vec_cg(S.xs, a.b.x, DIM, c.ct);
        }
        cbar();
        rmsnorm(c, S.xs, L.attn_norm, S.ns);
        {
            const Chunk *ch;
            const uint8_t *w = take(c, a, cur, QKV, ch);
            if (!w) return drain(c, cur);
            const int npair = ch->count;
            const float *sc = reinterpret_cast<const float *>(w + (size_t)2 * npair * DIM);
            if (c.cw < npair) {
                load_x896(S.ns, c.lane, xr);
                const int pair = ch->first + c.cw;
                const float d0 = row896(w + (size_t)(2 * c.cw) * DIM, sc + (2 * c.cw) * 14, xr, c.lane);
                const float d1 = row896(w + (size_t)(2 * c.cw + 1) * DIM, sc + (2 * c.cw + 1) * 14, xr, c.lane);
                if (c.lane == 0) {
                    int kind, t;
                    const float *bias;
                    if (pair < DIM / 2) { kind = 0; t = pair; bias = L.bq; }
                    else if (pair < DIM / 2 + KV / 2) { kind = 1; t = pair - DIM / 2; bias = L.bk; }
                    else { kind = 2; t = pair - DIM / 2 - KV / 2; bias = L.bv; }
                    const int head = t / 32, i = t % 32, r0 = head * HEAD_DIM + i;
                    const float v0 = d0 + __ldg(bias + r0), v1 = d1 + __ldg(bias + r0 + 32);
                    if (kind == 2) {
                        float *v = a.b.vc + kv_index(l, head, pos);
                        v[i] = v0;
                        v[i + 32] = v1;
                    } else {
                        const float cs = __ldg(a.b.rope_cos + pos * 32 + i), sn = __ldg(a.b.rope_sin + pos * 32 + i);
                        const float lo = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
                        const float hi = __fadd_rn(__fmul_rn(v1, cs), __fmul_rn(v0, sn));
                        if (kind == 0) {
                            a.b.q[r0] = lo;
                            a.b.q[r0 + 32] = hi;
                        } else {
                            float *k = a.b.kc + kv_index(l, head, pos);
                            k[i] = lo;
                            k[i + 32] = hi;
                        }
                    }
                }
            }
            give_back(c, cur);
        }
        gsignal(c, &a.sy->counters[l][PH_QKV]);

        // ---- split-K attention; the last unit of each KV head combines
        if (!gwait(c, &a.sy->counters[l][PH_QKV])) return drain(c, cur);
        {
            const int nch = pos / kAttnChunk + 1;
            if (cta < KV_HEADS * nch) attention_unit(c, a, l, pos, nch, cta);
        }
        gsignal(c, &a.sy->counters[l][PH_ATTN]);

        // ---- O projection + residual
        if (!gwait(c, &a.sy->counters[l][PH_ATTN])) return drain(c, cur);
        load_vec_cg(S.ns, a.scr.o, DIM, c.ct);
        cbar();
        {
            const Chunk *ch;
            const uint8_t *w = take(c, a, cur, OPROJ, ch);
            if (!w) return drain(c, cur);
            const int nrow = ch->count;
            const float *sc = reinterpret_cast<const float *>(w + (size_t)nrow * DIM);
            if (c.cw < nrow) {
                load_x896(S.ns, c.lane, xr);
                const int row = ch->first + c.cw;
                const float d = row896(w + (size_t)c.cw * DIM, sc + c.cw * 14, xr, c.lane);
                if (c.lane == 0) a.b.x[row] = __ldcg(a.b.x + row) + d;
            }
            give_back(c, cur);
        }
        gsignal(c, &a.sy->counters[l][PH_O]);

        // ---- RMSNorm -> gate/up -> SwiGLU
        if (!gwait(c, &a.sy->counters[l][PH_O])) return drain(c, cur);
        load_vec_cg(S.xs, a.b.x, DIM, c.ct);
        cbar();
        rmsnorm(c, S.xs, L.ffn_norm, S.ns);
        load_x896(S.ns, c.lane, xr);
        while (next_is(a, cur, GATEUP, l)) {
            const Chunk *ch;
            const uint8_t *w = take(c, a, cur, GATEUP, ch);
            if (!w) return drain(c, cur);
            const int npair = ch->count;
            const float *sc = reinterpret_cast<const float *>(w + (size_t)2 * npair * DIM);
            for (int p = c.cw; p < npair; p += kConsumerWarps) {
                const float g = row896(w + (size_t)(2 * p) * DIM, sc + (2 * p) * 14, xr, c.lane);
                const float u = row896(w + (size_t)(2 * p + 1) * DIM, sc + (2 * p + 1) * 14, xr, c.lane);
                if (c.lane == 0) a.b.h[ch->first + p] = (g / (1.0f + expf(-g))) * u;
            }
            give_back(c, cur);
        }
        gsignal(c, &a.sy->counters[l][PH_GATEUP]);

        // ---- down + residual: the CTA's threads own column chunks, rows reduced
        if (!gwait(c, &a.sy->counters[l][PH_GATEUP])) return drain(c, cur);
        load_vec_cg(S.u.hs, a.b.h, HIDDEN, c.ct);
        cbar();
        {
            const Chunk *ch;
            const uint8_t *w = take(c, a, cur, DOWN, ch);
            if (!w) return drain(c, cur);
            const int nrow = ch->count;
            constexpr int CH = HIDDEN / 16;  // 304 chunks of 16
            const float *sc = reinterpret_cast<const float *>(w + (size_t)nrow * HIDDEN);
            const int c1i = c.ct, c2i = c.ct + kNT;
#pragma unroll
            for (int i = 0; i < 16; i++) xr[i] = S.u.hs[c1i * 16 + i];
#pragma unroll
            for (int i = 0; i < 16; i++) xr[16 + i] = c2i < CH ? S.u.hs[c2i * 16 + i] : 0.f;
            for (int r = 0; r < nrow; r++) {
                const uint8_t *wr = w + (size_t)r * HIDDEN;
                const float *sr = sc + r * (HIDDEN / GROUP);
                float p = dot16r(*reinterpret_cast<const int4 *>(wr + c1i * 16), xr) * sr[c1i >> 2];
                if (c2i < CH) p = fmaf(dot16r(*reinterpret_cast<const int4 *>(wr + c2i * 16), xr + 16), sr[c2i >> 2], p);
                p = mb::warp_sum(p);
                if (c.lane == 0) S.red[c.cw][r] = p;
            }
            cbar();
            if (c.ct < nrow) {
                float sum = 0.f;
#pragma unroll
                for (int w8 = 0; w8 < kConsumerWarps; w8++) sum += S.red[w8][c.ct];
                const int row = ch->first + c.ct;
                a.b.x[row] = __ldcg(a.b.x + row) + sum;
            }
            give_back(c, cur);
        }
        gsignal(c, &a.sy->counters[l][PH_DOWN]);
    }

    if (project) {
        // ---- final norm + tied head, logits kept in shared memory for selection
        if (!gwait(c, &a.sy->counters[LAYERS - 1][PH_DOWN])) return drain(c, cur);
        load_vec_cg(S.xs, a.b.x, DIM, c.ct);
        cbar();
        rmsnorm(c, S.xs, M->final_norm, S.ns);
        if (cta == 0)
            for (int i = c.ct; i < DIM; i += kNT) a.b.hidden[i] = S.ns[i];
        load_x896(S.ns, c.lane, xr);
        const int lo = a.P->head_lo[cta], n = a.P->head_lo[cta + 1] - lo;
        while (next_is(a, cur, HEAD, LAYERS)) {
            const Chunk *ch;
            const uint8_t *w = take(c, a, cur, HEAD, ch);
            if (!w) return drain(c, cur);
            const int nrow = ch->count;
            const float *sc = reinterpret_cast<const float *>(w + (size_t)nrow * DIM);
            for (int r = c.cw; r < nrow; r += kConsumerWarps) {
                const float d = row896(w + (size_t)r * DIM, sc + r * 14, xr, c.lane);
                if (c.lane == 0) {
                    a.b.logits[ch->first + r] = d;
                    S.u.hl[ch->first + r - lo] = d;
                }
            }
            give_back(c, cur);
        }
        if (decode) {
            // penalty (distinct ids of the history window) and control mask on this
            // CTA's vocabulary slice, then the slice's top k as ordered keys
            const sampling::Params prm = *a.prm;
            if (c.cw == 0) {
                const int count = min(max(a.seq->history_count, 0), sampling::kHistory);
                for (int j = c.lane; j < count; j += 32) {
                    const int id = a.seq->history[j];
                    bool dup = false;
                    for (int t = 0; t < j; t++) dup |= a.seq->history[t] == id;
                    if (!dup && id >= lo && id < lo + n) {
                        const float v = S.u.hl[id - lo];
                        S.u.hl[id - lo] = v < 0 ? v * prm.penalty : v / prm.penalty;
                    }
                }
            }
            cbar();
            const int k = min(max(prm.top_k, 1), sampling::kMaxK);
            unsigned long long *keys = reinterpret_cast<unsigned long long *>(S.ring[0]);
            unsigned long long best = 0ull;
            for (int i = c.ct; i < 2048; i += kNT) {
                unsigned long long key = 0ull;
                if (i < n) {
                    const int id = lo + i;
                    float v = S.u.hl[i];
                    if (id >= prm.control_first && id != prm.eos) v = -1e30f;
                    key = mb::rank_key(v, id);
                }
                keys[i] = key;
                best = key > best ? key : best;
            }
            if (k == 1) {
                best = block_max(c, best);
                if (c.ct == 0) a.scr.cand[cta * sampling::kMaxK] = best;
            } else {
                cbar();
                bitonic_desc(keys, 2048, c.ct);
                for (int j = c.ct; j < k; j += kNT) a.scr.cand[cta * sampling::kMaxK + j] = keys[j];
            }
        }
    }

    // ---- end of step: the last CTA finishes the token
    cbar();
    if (c.ct == 0) {
        __threadfence();
        const unsigned t = atomicAdd(&a.sy->done, 1u);
        S.flag = t == c.target - 1;
    }
    cbar();
    if (!S.flag) return;
    __threadfence();
    if (decode) {
        const sampling::Params prm = *a.prm;
        const int k = min(max(prm.top_k, 1), sampling::kMaxK);
        unsigned long long *keys = reinterpret_cast<unsigned long long *>(S.ring[0]);
        if (k == 1) {
            unsigned long long best = 0ull;
            for (int i = c.ct; i < kCTAs; i += kNT) {
                const unsigned long long v = __ldcg(a.scr.cand + i * sampling::kMaxK);
                best = v > best ? v : best;
            }
            best = block_max(c, best);
            if (c.ct == 0) keys[0] = best;
        } else {
            const int nin = kCTAs * k;
            int n = 1;
            while (n < nin) n <<= 1;
            for (int i = c.ct; i < n; i += kNT)
                keys[i] = i < nin ? __ldcg(a.scr.cand + (i / k) * sampling::kMaxK + (i % k)) : 0ull;
            cbar();
            bitonic_desc(keys, n, c.ct);
        }
        cbar();
        if (c.ct == 0) {
            uint32_t seed = a.seq->seed;
            int token = sampling::draw_token(keys, prm, seed);
            a.seq->seed = seed;
            if (token < 0 || token >= prm.vocab) token = prm.eos;
            sampling::record_token(token, prm, a.seq, a.out_ring, a.out_count);
            a.b.st->token = token;
            a.b.st->pos = pos + 1;
        }
    } else if (a.mode == PREFILL) {
        if (c.ct == 0) {
            a.b.st->pos = pos + 1;
            a.b.st->token = a.prompt[pos + 1];
        }
    }
    if (c.ct == 0) {
        a.b.st->steps++;
        __threadfence();
        atomicExch(&a.sy->epoch, epoch + 1);
    }
}

// host: balanced split of n items over parts
inline void split(int n, int parts, int i, int &lo, int &hi)
{
    lo = (int)((long long)n * i / parts);
    hi = (int)((long long)n * (i + 1) / parts);
}

}  // namespace

size_t smem_bytes() { return sizeof(Smem); }

int init_device()
{
    const cudaError_t e = cudaFuncSetAttribute(k_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem));
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA persistent decode init: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k_step, kThreads, sizeof(Smem)) != cudaSuccess ||
        blocks < 1) {
        fprintf(stderr, "MOCHA_B200: persistent decode kernel does not fit on an SM\n");
        return 1;
    }
    return 0;
}

int build_plan(const FileHeader *hdr, const unsigned char *hfile, Plan *hplan, Chunk **dchunks, uint8_t **dstream,
               size_t *stream_bytes, cudaStream_t s)
{
    std::vector<Chunk> chunks;
    std::vector<uint8_t> stream;
    stream.reserve((size_t)540 << 20);
    const FileTensor *t = hdr->t;
    auto align16 = [](size_t v) { return (v + 15) & ~(size_t)15; };
    // append rows (as (tensor, row) pairs) as one chunk: int8 rows, then fp32 scales
    auto emit = [&](uint32_t kind, uint32_t layer, uint32_t first, uint32_t count,
                    const std::vector<std::pair<const FileTensor *, int>> &rows) {
        Chunk ch{};
        ch.off = stream.size();
        ch.kind = kind;
        ch.layer = layer;
        ch.first = first;
        ch.count = count;
        for (auto &r : rows) {
            const uint8_t *src = hfile + r.first->data + (size_t)r.second * r.first->cols;
            stream.insert(stream.end(), src, src + r.first->cols);
        }
        for (auto &r : rows) {
            const size_t g = r.first->cols / GROUP;
            const uint8_t *src = hfile + r.first->scales + (size_t)r.second * g * 4;
            stream.insert(stream.end(), src, src + g * 4);
        }
        stream.resize(align16(stream.size()), 0);
        ch.bytes = (uint32_t)(stream.size() - ch.off);
        if (ch.bytes > (uint32_t)kSlotBytes) return false;
        chunks.push_back(ch);
        return true;
    };
    for (int c = 0; c < kCTAs; c++) {
        hplan->chunk_begin[c] = (uint32_t)chunks.size();
        for (int l = 0; l < LAYERS; l++) {
            const FileTensor *lt = t + 1 + l * STRIDE;
            int lo, hi;
            std::vector<std::pair<const FileTensor *, int>> rows;
            split(kQkvPairs, kCTAs, c, lo, hi);
            for (int p = lo; p < hi; p++) {
                const FileTensor *m;
                int tt;
                if (p < DIM / 2) { m = &lt[WQ]; tt = p; }
                else if (p < DIM / 2 + KV / 2) { m = &lt[WK]; tt = p - DIM / 2; }
                else { m = &lt[WV]; tt = p - DIM / 2 - KV / 2; }
                const int r0 = (tt / 32) * HEAD_DIM + tt % 32;
                rows.push_back({m, r0});
                rows.push_back({m, r0 + 32});
            }
            if (!emit(QKV, l, lo, hi - lo, rows)) return 1;
            rows.clear();
            split(DIM, kCTAs, c, lo, hi);
            for (int r = lo; r < hi; r++) rows.push_back({&lt[WO], r});
            if (!emit(OPROJ, l, lo, hi - lo, rows)) return 1;
            split(HIDDEN, kCTAs, c, lo, hi);
            for (int p0 = lo; p0 < hi; p0 += kGateupPerChunk) {
                const int p1 = p0 + kGateupPerChunk < hi ? p0 + kGateupPerChunk : hi;
                rows.clear();
                for (int p = p0; p < p1; p++) {
                    rows.push_back({&lt[WGATE], p});
                    rows.push_back({&lt[WUP], p});
                }
                if (!emit(GATEUP, l, p0, p1 - p0, rows)) return 1;
            }
            rows.clear();
            split(DIM, kCTAs, c, lo, hi);
            for (int r = lo; r < hi; r++) rows.push_back({&lt[WDOWN], r});
            if (!emit(DOWN, l, lo, hi - lo, rows)) return 1;
        }
        int lo, hi;
        split(VOCAB, kCTAs, c, lo, hi);
        hplan->head_lo[c] = lo;
        if (hi - lo > kHeadSlice) return 1;
        for (int r0 = lo; r0 < hi; r0 += kHeadPerChunk) {
            const int r1 = r0 + kHeadPerChunk < hi ? r0 + kHeadPerChunk : hi;
            std::vector<std::pair<const FileTensor *, int>> rows;
            for (int r = r0; r < r1; r++) rows.push_back({&t[0], r});
            if (!emit(HEAD, LAYERS, r0, r1 - r0, rows)) return 1;
        }
    }
    hplan->chunk_begin[kCTAs] = (uint32_t)chunks.size();
    hplan->head_lo[kCTAs] = VOCAB;
    if (cudaMalloc(dstream, stream.size()) != cudaSuccess ||
        cudaMalloc(dchunks, chunks.size() * sizeof(Chunk)) != cudaSuccess ||
        cudaMemcpyAsync(*dstream, stream.data(), stream.size(), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(*dchunks, chunks.data(), chunks.size() * sizeof(Chunk), cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        fprintf(stderr, "MOCHA_B200: persistent plan upload failed\n");
        return 1;
    }
    hplan->stream = *dstream;
    hplan->chunks = *dchunks;
    *stream_bytes = stream.size();
    return 0;
}

int enqueue_step(const Model *dm, const Plan *dplan, const Buffers &b, Sync *sync, const Scratch &scr, int mode,
                 const sampling::Params *prm, sampling::SeqState *seq, int *out_ring, int *out_count,
                 const int *prompt, unsigned *host_error, cudaStream_t s)
{
    Args a{dm, dplan, b, sync, scr, mode, prm, seq, out_ring, out_count, prompt, host_error};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCTAs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(Smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_step, a);
    if (e != cudaSuccess) {
        fprintf(stderr, "CUDA persistent decode launch: %d %s\n", (int)e, cudaGetErrorString(e));
        return 1;
    }
    return 0;
}

}  // namespace q8p
