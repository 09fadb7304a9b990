// Persistent batch-1 decode step for the grouped-Q8 model on B200.
//
// One cooperative launch of 148 CTAs (one per SM) runs the whole token.
//
// Weights: warp 0 of every CTA streams that CTA's weights -- laid out at set-up as
// one contiguous region per CTA, in consumption order -- through a 4-slot
// shared-memory ring with cp.async.bulk copies completed on mbarriers.  Each chunk
// carries a 16-byte header (kind, layer, row range) and its rows' biases; chunks that
// start a normalised phase also receive the RMSNorm gain by a second bulk copy (an
// L2 hit: every CTA reads the same gain).  Weights do not depend on activations, so
// the stream runs ahead of the dependency chain by up to the ring depth.
//
// Activations: the 16 consumer warps exchange every cross-CTA value as a 64-bit data
// word (float | tag << 32, tag = epoch << 8 | layer << 3 | phase) written with one
// relaxed store and polled directly by its readers.  There are no counters, fences or
// second loads between phases; each reader waits exactly for the words it needs.
// Per layer: QKV (+bias, split-half RoPE, KV write) -> attention split over the
// positions of each query head (K/V of past positions are prefetched with cp.async
// before the query exists) -> O + residual -> RMSNorm -> gate/up + SwiGLU ->
// down + residual.  The vocabulary head is fused with the repetition penalty, the
// control mask and a per-CTA top-k; the last CTA to finish (one atomic ticket)
// merges the candidates, draws the token and advances the epoch.
//
// Every wait is bounded (~2 s of clock cycles); on expiry the kernel records an
// error word (device and mapped host memory), drains its own bulk copies and exits.
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
constexpr int kNT = kConsumerWarps * 32;  // consumer threads
constexpr long long kTimeoutCycles = 4000000000LL;
constexpr int kQkvPairs = (DIM + 2 * KV) / 2;  // 576
constexpr int kGateupPerChunk = 17;            // pairs: 34 rows of 896 + header < kGainOff
constexpr int kHeadPerChunk = 34;              // rows
constexpr int kHeadSlice = 1040;               // >= ceil(VOCAB / kCTAs)
constexpr int kPartWords = HEADS * kMaxSplit * ATTN_PARTIAL;

enum Phase { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_H = 3, PH_X = 4 };

struct Smem {
    uint8_t ring[kSlots][kSlotBytes];
    __align__(16) float xs[DIM];  // residual (x_in, then x_mid) of the current layer
    __align__(16) float ns[DIM];  // normalised input / attention output
    union __align__(16) {
        float hs[HIDDEN];          // down-projection input
        float part[kPartWords];    // gathered attention partials
        struct {
            float k[kAttnLenMax][HEAD_DIM];
            float v[kAttnLenMax][HEAD_DIM];
            float q[HEAD_DIM];
            float e[kAttnLenMax + 1];
        } att;
        float hl[kHeadSlice];      // this CTA's slice of the logits
    } u;
    float red[kConsumerWarps][8];
    float rc[HEAD_DIM / 2], rs[HEAD_DIM / 2];  // RoPE cos/sin at pos
    Chunk desc[kMaxChunksPerCta];  // this CTA's chunk descriptors (producer)
    unsigned long long full[kSlots], empty[kSlots];
    int flag;
    int iters;  // poll iterations of the last traced gather
    int token, pos;
    volatile int issued;         // chunks the producer has started copying
    volatile int producer_done;  // the producer has left its loop
};

// ---- low-level primitives --------------------------------------------------

MB_DEV uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

MB_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kNT) : "memory"); }

// consumer barrier that also ANDs a predicate over the consumer threads
MB_DEV int cbar_and(int v)
{
    int r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.s32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.s32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(v), "n"(kNT)
        : "memory");
    return r;
}

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

MB_DEV unsigned ld_volatile(const unsigned *p) { return *(const volatile unsigned *)p; }

MB_DEV void fail(Sync *sy, unsigned *host_error, unsigned code)
{
    atomicCAS(&sy->error, 0u, code);
    *(volatile unsigned *)host_error = code;
    __threadfence_system();
}

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

MB_DEV void bulk_load(void *dst, const void *src, uint32_t bytes, unsigned long long *bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

MB_DEV void bulk_load_plain(void *dst, const void *src, uint32_t bytes, unsigned long long *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

MB_DEV void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
MB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// data words
MB_DEV void dw_store(unsigned long long *p, float v, uint32_t tag)
{
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

MB_DEV unsigned long long dw_load(const unsigned long long *p)
{
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

MB_DEV uint32_t make_tag(uint32_t epoch, int layer, int phase) { return (epoch << 8) | (layer << 3) | phase; }

// ---- consumer-side helpers --------------------------------------------------

struct Ctx {
    Smem &S;
    Sync *sy;
    unsigned *host_error;
    int ct, cw, lane;
};

// 32-byte relaxed load of four data words (one L2 request instead of four)
MB_DEV void dw_load4(const unsigned long long *p, unsigned long long (&v)[4])
{
    asm volatile("ld.relaxed.gpu.global.v4.u64 {%0,%1,%2,%3}, [%4];"
                 : "=l"(v[0]), "=l"(v[1]), "=l"(v[2]), "=l"(v[3])
                 : "l"(p)
                 : "memory");
}

// Poll the data words src[0..n) (n a multiple of 4, src 32-byte aligned) that `want`
// selects until each carries `tag`, storing their floats to dst.  Thread ct owns the
// 4-word groups ct, ct+kNT, ...; each request covers a whole group, only groups with
// missing words are polled again, and a short sleep between rounds keeps 148 CTAs
// from saturating the L2 slices that hold the words.  Every consumer thread returns
// the same verdict.
template <int E, typename Want>
MB_DEV bool gather_if(Ctx &c, const unsigned long long *src, int n, uint32_t tag, float *dst, Want want,
                      int *iters = nullptr)
{
    const int ng = n >> 2;
    unsigned need[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        const int g = c.ct + e * kNT;
        need[e] = 0;
        if (g < ng)
#pragma unroll
            for (int j = 0; j < 4; j++) need[e] |= want(4 * g + j) ? (1u << j) : 0u;
    }
    int ok = 1, it = 0;
    long long t0 = 0;
    for (;;) {
        unsigned missing = 0;
#pragma unroll
        for (int e = 0; e < E; e++) {
            if (!need[e]) continue;
            const int g = c.ct + e * kNT;
            unsigned long long v[4];
            dw_load4(src + 4 * g, v);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if ((need[e] >> j & 1u) && (uint32_t)(v[j] >> 32) == tag) {
                    dst[4 * g + j] = __uint_as_float((uint32_t)v[j]);
                    need[e] &= ~(1u << j);
                }
            }
            missing |= need[e];
        }
        if (!missing) break;
        it++;
        if (t0 == 0) {
            t0 = clock64();
        } else if (clock64() - t0 > kTimeoutCycles) {
            fail(c.sy, c.host_error, 1);
            ok = 0;
            break;
        }
        if (ld_volatile(&c.sy->error)) {
            ok = 0;
            break;
        }
        __nanosleep(64);
    }
    if (iters) atomicMax(iters, it);
    return cbar_and(ok) != 0;
}

struct All {
    MB_DEV bool operator()(int) const { return true; }
};

template <int E>
MB_DEV bool gather(Ctx &c, const unsigned long long *src, int n, uint32_t tag, float *dst, int *iters = nullptr)
{
    return gather_if<E>(c, src, n, tag, dst, All{}, iters);
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
    for (int i = c.ct; i < DIM; i += kNT) ns[i] = xs[i] * s * gain[i];
    cbar();
}

// 16 int8 weights . 16 fp32 inputs held in registers (two accumulation chains)
MB_DEV float dot16r(const int4 w, const float *xr)
{
    const uint32_t u[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u, (uint32_t)w.z ^ 0x80808080u,
                           (uint32_t)w.w ^ 0x80808080u};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        a0 = fmaf(mb::s8_lane(u[i], 0x7540), xr[4 * i + 0], a0);
        a1 = fmaf(mb::s8_lane(u[i], 0x7541), xr[4 * i + 1], a1);
        a0 = fmaf(mb::s8_lane(u[i], 0x7542), xr[4 * i + 2], a0);
        a1 = fmaf(mb::s8_lane(u[i], 0x7543), xr[4 * i + 3], a1);
    }
    return a0 + a1;
}

// A 896-wide row: lane owns 16-weight chunks lane and lane+32 (< 56); its 32 inputs
// live in registers for every row of the phase.
MB_DEV void load_x896(const float *ns, int lane, float *xr)
{
    const float4 *n4 = reinterpret_cast<const float4 *>(ns);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 v = n4[lane * 4 + i];
        xr[4 * i] = v.x;
        xr[4 * i + 1] = v.y;
        xr[4 * i + 2] = v.z;
        xr[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 v = lane < 24 ? n4[(lane + 32) * 4 + i] : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[16 + 4 * i] = v.x;
        xr[16 + 4 * i + 1] = v.y;
        xr[16 + 4 * i + 2] = v.z;
        xr[16 + 4 * i + 3] = v.w;
    }
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
    unsigned long long *trace;  // optional [kCTAs][kTraceStamps] %globaltimer stamps
};

MB_DEV void stamp(const Args &a, int cta, int ct, int point)
{
    if (a.trace && ct == 0 && point < kTraceStamps) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[cta * kTraceStamps + point] = t;
    }
}

MB_DEV void stamp_value(const Args &a, int cta, int ct, int point, unsigned long long v)
{
    if (a.trace && ct == 0 && point < kTraceStamps) a.trace[cta * kTraceStamps + point] = v;
}

struct Cursor {
    uint32_t k;  // chunks consumed
};

// Wait for the next chunk; returns the slot (header first) or null on failure.
MB_DEV const uint8_t *take(Ctx &c, Cursor &cur, uint32_t kind)
{
    const uint32_t slot = cur.k % kSlots, use = cur.k / kSlots;
    if (!mbar_wait(&c.S.full[slot], use & 1, c.sy, c.host_error)) return nullptr;
    const uint8_t *w = c.S.ring[slot];
    if (reinterpret_cast<const ChunkHdr *>(w)->kind != kind) {
        if (c.ct == 0) fail(c.sy, c.host_error, 4);
        return nullptr;
    }
    return w;
}

MB_DEV void give_back(Ctx &c, Cursor &cur)
{
    cbar();
    if (c.ct == 0) mbar_arrive(&c.S.empty[cur.k % kSlots]);
    cur.k++;
}

// Is the next chunk of `kind` in `layer`?  (waits for it to land, then reads its
// header; -1 on failure)
MB_DEV int next_is(Ctx &c, const Cursor &cur, int remaining, uint32_t kind, uint32_t layer)
{
    if (remaining <= 0) return 0;
    const uint32_t slot = cur.k % kSlots, use = cur.k / kSlots;
    if (!mbar_wait(&c.S.full[slot], use & 1, c.sy, c.host_error)) return -1;
    const ChunkHdr *h = reinterpret_cast<const ChunkHdr *>(c.S.ring[slot]);
    return h->kind == kind && h->layer == layer ? 1 : 0;
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
    cp_async_wait_all();
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

// attention split of one query head: positions [p0, p0+np)
struct AttnUnit {
    int head, split, p0, np;
};

struct UsedSplit {
    int splits;
    MB_DEV bool operator()(int i) const { return (i / ATTN_PARTIAL) % kMaxSplit < splits; }
};

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
        const bool bad = S.token < 0 || S.token >= VOCAB || S.pos < 0 || S.pos >= CONTEXT || epoch == 0 ||
                         epoch >= (1u << 24) || (a.mode == PREFILL && S.pos + 1 >= CONTEXT) ||
                         a.P->chunk_begin[cta + 1] - a.P->chunk_begin[cta] > (uint32_t)kMaxChunksPerCta;
        if (bad) {
            fail(a.sy, a.host_error, 5);
            S.flag = -1;
        }
    }
    __syncthreads();
    if (S.flag < 0) return;  // invalid token / position: nothing was issued
    const uint32_t c0 = a.P->chunk_begin[cta], c1 = a.P->chunk_begin[cta + 1];

    const uint32_t c_end = project ? c1 : a.P->head_begin[cta];  // head chunks only when projecting
    if (threadIdx.x < 32) {  // ---- producer warp: stream this CTA's weights
        for (uint32_t j = threadIdx.x; j < c_end - c0 && j < (uint32_t)kMaxChunksPerCta; j += 32)
            S.desc[j] = a.P->chunks[c0 + j];
        __syncwarp();
        if (threadIdx.x == 0) {
            const uint64_t policy = mb::evict_first_policy();
            uint32_t k = 0;
            for (uint32_t i = 0; i < c_end - c0; i++) {
                const Chunk ch = S.desc[i];
                const uint32_t slot = k % kSlots, use = k / kSlots;
                if (use > 0 && !mbar_wait(&S.empty[slot], (use - 1) & 1, a.sy, a.host_error)) break;
                if (ld_volatile(&a.sy->error)) break;
                mbar_expect_tx(&S.full[slot], ch.bytes + (ch.gain_off ? kGainBytes : 0));
                bulk_load(S.ring[slot], a.P->stream + ch.off, ch.bytes, &S.full[slot], policy);
                if (ch.gain_off)
                    bulk_load_plain(S.ring[slot] + kGainOff, a.P->blob + ch.gain_off, kGainBytes, &S.full[slot]);
                k++;
                S.issued = (int)k;
            }
            __threadfence_block();
            S.producer_done = 1;
        }
        return;
    }

    Ctx c{S, a.sy, a.host_error, (int)threadIdx.x - 32, ((int)threadIdx.x - 32) >> 5, (int)threadIdx.x & 31};
    const int pos = S.pos;
    Cursor cur{0};
    int remaining = (int)(c_end - c0);  // chunks this CTA still has to take
    const Model *M = a.M;
    const Scratch &scr = a.scr;
    float xr[32];
    stamp(a, cta, c.ct, 0);

    // per-step constants: RoPE at pos, the attention split owned by this CTA
    if (c.ct < HEAD_DIM / 2) {
        S.rc[c.ct] = __ldg(a.b.rope_cos + pos * 32 + c.ct);
        S.rs[c.ct] = __ldg(a.b.rope_sin + pos * 32 + c.ct);
    }
    const int splits = min(kMaxSplit, (pos + kAttnTarget) / kAttnTarget);
    const int span = (pos + splits) / splits;  // ceil((pos+1)/splits) <= kAttnLenMax
    AttnUnit unit{-1, 0, 0, 0};
    if (cta < HEADS * splits) {
        unit.head = cta / splits;
        unit.split = cta % splits;
        unit.p0 = unit.split * span;
        unit.np = min(span, pos + 1 - unit.p0);
    }
    // layer-0 input: the token's embedding row (src/minimind.cu:70)
    {
        const int8_t *e = M->embed.w + (size_t)S.token * DIM;
        const float *es = M->embed.s + (size_t)S.token * (DIM / GROUP);
        for (int i = c.ct; i < DIM; i += kNT) S.xs[i] = (float)e[i] * __ldg(es + i / GROUP);
    }
    cbar();

    for (int l = 0; l < LAYERS; l++) {
        // K/V of past positions for this CTA's attention split: no dependency on this
        // step, copied asynchronously while the QKV phase runs
        if (unit.head >= 0) {
            const int kvh = unit.head / GQA;
            const int past = min(unit.np, pos - unit.p0);  // rows < pos
            const float *kb = a.b.kc + kv_index(l, kvh, unit.p0);
            const float *vb = a.b.vc + kv_index(l, kvh, unit.p0);
            for (int i = c.ct; i < past * (HEAD_DIM / 4); i += kNT) {
                const int p = i / (HEAD_DIM / 4), q4 = i % (HEAD_DIM / 4);
                cp_async16(&S.u.att.k[p][q4 * 4], kb + p * HEAD_DIM + q4 * 4);
                cp_async16(&S.u.att.v[p][q4 * 4], vb + p * HEAD_DIM + q4 * 4);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        // ---- QKV + bias + RoPE + KV write
        if (l > 0 && !gather<1>(c, scr.xin, DIM, make_tag(epoch, l - 1, PH_X), S.xs)) return drain(c, cur);
        stamp(a, cta, c.ct, 2 + l * 12 + 0);
        {
            const uint8_t *w = take(c, cur, QKV);
            if (!w) return drain(c, cur);
            const ChunkHdr hd = *reinterpret_cast<const ChunkHdr *>(w);
            rmsnorm(c, S.xs, reinterpret_cast<const float *>(w + kGainOff), S.ns);
            const int npair = hd.count;
            const uint8_t *rows = w + sizeof(ChunkHdr);
            const float *sc = reinterpret_cast<const float *>(rows + (size_t)2 * npair * DIM);
            const float *bias = sc + 2 * npair * (DIM / GROUP);
            if (c.cw < npair) {
                load_x896(S.ns, c.lane, xr);
                const int pair = hd.first + c.cw;
                const float d0 = row896(rows + (size_t)(2 * c.cw) * DIM, sc + (2 * c.cw) * 14, xr, c.lane);
                const float d1 = row896(rows + (size_t)(2 * c.cw + 1) * DIM, sc + (2 * c.cw + 1) * 14, xr, c.lane);
                if (c.lane == 0) {
                    const uint32_t tag = make_tag(epoch, l, PH_QKV);
                    int kind, t;
                    if (pair < DIM / 2) { kind = 0; t = pair; }
                    else if (pair < DIM / 2 + KV / 2) { kind = 1; t = pair - DIM / 2; }
                    else { kind = 2; t = pair - DIM / 2 - KV / 2; }
                    const int head = t / 32, i = t % 32, r0 = head * HEAD_DIM + i;
                    const float v0 = d0 + bias[2 * c.cw], v1 = d1 + bias[2 * c.cw + 1];
                    if (kind == 2) {
                        float *v = a.b.vc + kv_index(l, head, pos);
                        v[i] = v0;
                        v[i + 32] = v1;
                        dw_store(scr.kv + (head * 2 + 1) * HEAD_DIM + i, v0, tag);
                        dw_store(scr.kv + (head * 2 + 1) * HEAD_DIM + i + 32, v1, tag);
                    } else {
                        const float cs = S.rc[i], sn = S.rs[i];
                        // unfused products, as the reference CPU evaluates them (src/minimind.cpp:64-66)
                        const float lo = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
                        const float hi = __fadd_rn(__fmul_rn(v1, cs), __fmul_rn(v0, sn));
                        if (kind == 0) {
                            dw_store(scr.q + r0, lo, tag);
                            dw_store(scr.q + r0 + 32, hi, tag);
                        } else {
                            float *k = a.b.kc + kv_index(l, head, pos);
                            k[i] = lo;
                            k[i + 32] = hi;
                            dw_store(scr.kv + (head * 2) * HEAD_DIM + i, lo, tag);
                            dw_store(scr.kv + (head * 2) * HEAD_DIM + i + 32, hi, tag);
                        }
                    }
                }
            }
            give_back(c, cur);
            remaining--;
        }
        stamp(a, cta, c.ct, 2 + l * 12 + 1);

        // ---- attention: one split of one query head per CTA
        if (unit.head >= 0) {
            const uint32_t tag = make_tag(epoch, l, PH_QKV);
            const int h = unit.head, kvh = h / GQA, np = unit.np;
            const bool has_cur = unit.p0 + np == pos + 1;
            const unsigned long long ready = (unsigned long long)tag << 32;
            // the query of this head, and this position's K/V when the split holds it
            int ok = 1;
            if (c.ct < HEAD_DIM) {
                const unsigned long long *qa = scr.q + h * HEAD_DIM + c.ct;
                const unsigned long long *ka = scr.kv + (kvh * 2) * HEAD_DIM + c.ct;
                const unsigned long long *va = scr.kv + (kvh * 2 + 1) * HEAD_DIM + c.ct;
                unsigned long long w = dw_load(qa);
                unsigned long long wk = has_cur ? dw_load(ka) : ready;
                unsigned long long wv = has_cur ? dw_load(va) : ready;
                const long long t0 = clock64();
                while ((uint32_t)(w >> 32) != tag || (uint32_t)(wk >> 32) != tag || (uint32_t)(wv >> 32) != tag) {
                    if ((uint32_t)(w >> 32) != tag) w = dw_load(qa);
                    if ((uint32_t)(wk >> 32) != tag) wk = dw_load(ka);
                    if ((uint32_t)(wv >> 32) != tag) wv = dw_load(va);
                    if (ld_volatile(&c.sy->error)) {
                        ok = 0;
                        break;
                    }
                    if (clock64() - t0 > kTimeoutCycles) {
                        fail(c.sy, c.host_error, 1);
                        ok = 0;
                        break;
                    }
                }
                S.u.att.q[c.ct] = __uint_as_float((uint32_t)w);
                if (has_cur) {
                    S.u.att.k[np - 1][c.ct] = __uint_as_float((uint32_t)wk);
                    S.u.att.v[np - 1][c.ct] = __uint_as_float((uint32_t)wv);
                }
            }
            cp_async_wait_all();
            if (!cbar_and(ok)) return drain(c, cur);
            // scores: warp per position, lanes over the 64 dims
            for (int p = c.cw; p < np; p += kConsumerWarps) {
                float z = S.u.att.q[c.lane] * S.u.att.k[p][c.lane];
                z = fmaf(S.u.att.q[c.lane + 32], S.u.att.k[p][c.lane + 32], z);
                z = mb::warp_sum(z);
                if (c.lane == 0) S.u.att.e[p] = z * 0.125f;
            }
            cbar();
            if (c.cw == 0) {
                float m = -INFINITY;
                for (int p = c.lane; p < np; p += 32) m = fmaxf(m, S.u.att.e[p]);
                m = mb::warp_max(m);
                float lsum = 0.f;
                for (int p = c.lane; p < np; p += 32) {
                    const float e = expf(S.u.att.e[p] - m);
                    S.u.att.e[p] = e;
                    lsum += e;
                }
                lsum = mb::warp_sum(lsum);
                if (c.lane == 0) {
                    S.red[0][0] = m;
                    S.red[0][1] = lsum;
                }
            }
            cbar();
            if (c.ct < HEAD_DIM) {
                float acc = 0.f;
                for (int p = 0; p < np; p++) acc = fmaf(S.u.att.e[p], S.u.att.v[p][c.ct], acc);
                const uint32_t ptag = make_tag(epoch, l, PH_ATTN);
                unsigned long long *out = scr.part + ((size_t)h * kMaxSplit + unit.split) * ATTN_PARTIAL;
                dw_store(out + 2 + c.ct, acc, ptag);
                if (c.ct == 0) {
                    dw_store(out, S.red[0][0], ptag);
                    dw_store(out + 1, S.red[0][1], ptag);
                }
            }
            cbar();
        }
        stamp(a, cta, c.ct, 2 + l * 12 + 2);

        // ---- O projection + residual: combine every head's splits, then the rows
        if (!gather_if<(kPartWords / 4 + kNT - 1) / kNT>(c, scr.part, kPartWords, make_tag(epoch, l, PH_ATTN), S.u.part,
                                                       UsedSplit{splits}))
            return drain(c, cur);
        for (int idx = c.ct; idx < DIM; idx += kNT) {
            const int h = idx / HEAD_DIM, d = idx % HEAD_DIM;
            const float *p = S.u.part + (size_t)h * kMaxSplit * ATTN_PARTIAL;
            float mx = -INFINITY;
            for (int s = 0; s < splits; s++) mx = fmaxf(mx, p[s * ATTN_PARTIAL]);
            float lsum = 0.f, acc = 0.f;
            for (int s = 0; s < splits; s++) {
                const float wgt = expf(p[s * ATTN_PARTIAL] - mx);
                lsum = fmaf(wgt, p[s * ATTN_PARTIAL + 1], lsum);
                acc = fmaf(wgt, p[s * ATTN_PARTIAL + 2 + d], acc);
            }
            S.ns[idx] = acc / lsum;
        }
        cbar();
        stamp(a, cta, c.ct, 2 + l * 12 + 3);
        {
            const uint8_t *w = take(c, cur, OPROJ);
            if (!w) return drain(c, cur);
            const ChunkHdr hd = *reinterpret_cast<const ChunkHdr *>(w);
            const int nrow = hd.count;
            const uint8_t *rows = w + sizeof(ChunkHdr);
            const float *sc = reinterpret_cast<const float *>(rows + (size_t)nrow * DIM);
            if (c.cw < nrow) {
                load_x896(S.ns, c.lane, xr);
                const int row = hd.first + c.cw;
                const float d = row896(rows + (size_t)c.cw * DIM, sc + c.cw * 14, xr, c.lane);
                if (c.lane == 0) dw_store(scr.xmid + row, S.xs[row] + d, make_tag(epoch, l, PH_O));
            }
            give_back(c, cur);
            remaining--;
        }
        stamp(a, cta, c.ct, 2 + l * 12 + 4);

        // ---- RMSNorm -> gate/up -> SwiGLU
        if (c.ct == 0) S.iters = 0;
        cbar();
        if (!gather<1>(c, scr.xmid, DIM, make_tag(epoch, l, PH_O), S.xs, &S.iters)) return drain(c, cur);
        stamp(a, cta, c.ct, 2 + l * 12 + 5);
        stamp_value(a, cta, c.ct, 2 + l * 12 + 11, (unsigned long long)S.iters);
        {
            bool first = true;
            for (;;) {
                const int more = next_is(c, cur, remaining, GATEUP, l);
                if (more < 0) return drain(c, cur);
                if (!more) break;
                const uint8_t *w = take(c, cur, GATEUP);
                if (!w) return drain(c, cur);
                if (first) {
                    stamp(a, cta, c.ct, 2 + l * 12 + 9);
                    rmsnorm(c, S.xs, reinterpret_cast<const float *>(w + kGainOff), S.ns);
                    load_x896(S.ns, c.lane, xr);
                    first = false;
                    stamp(a, cta, c.ct, 2 + l * 12 + 10);
                }
                const ChunkHdr hd = *reinterpret_cast<const ChunkHdr *>(w);
                const int npair = hd.count;
                const uint8_t *rows = w + sizeof(ChunkHdr);
                const float *sc = reinterpret_cast<const float *>(rows + (size_t)2 * npair * DIM);
                const uint32_t tag = make_tag(epoch, l, PH_H);
                for (int p = c.cw; p < npair; p += kConsumerWarps) {
                    const float g = row896(rows + (size_t)(2 * p) * DIM, sc + (2 * p) * 14, xr, c.lane);
                    const float u = row896(rows + (size_t)(2 * p + 1) * DIM, sc + (2 * p + 1) * 14, xr, c.lane);
                    if (c.lane == 0) dw_store(scr.h + hd.first + p, (g / (1.0f + expf(-g))) * u, tag);
                }
                give_back(c, cur);
                remaining--;
            }
        }
        stamp(a, cta, c.ct, 2 + l * 12 + 6);

        // ---- down + residual: the CTA's threads own column chunks, rows reduced
        if (!gather<(HIDDEN / 4 + kNT - 1) / kNT>(c, scr.h, HIDDEN, make_tag(epoch, l, PH_H), S.u.hs))
            return drain(c, cur);
        stamp(a, cta, c.ct, 2 + l * 12 + 7);
        {
            const uint8_t *w = take(c, cur, DOWN);
            if (!w) return drain(c, cur);
            const ChunkHdr hd = *reinterpret_cast<const ChunkHdr *>(w);
            const int nrow = hd.count;
            constexpr int CH = HIDDEN / 16;  // 304 chunks of 16
            const uint8_t *rows = w + sizeof(ChunkHdr);
            const float *sc = reinterpret_cast<const float *>(rows + (size_t)nrow * HIDDEN);
            const int ci = c.ct;
            if (ci < CH) {
                const float4 *h4 = reinterpret_cast<const float4 *>(S.u.hs + ci * 16);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float4 v = h4[i];
                    xr[4 * i] = v.x;
                    xr[4 * i + 1] = v.y;
                    xr[4 * i + 2] = v.z;
                    xr[4 * i + 3] = v.w;
                }
            }
            for (int r = 0; r < nrow; r++) {
                float p = 0.f;
                if (ci < CH)
                    p = dot16r(*reinterpret_cast<const int4 *>(rows + (size_t)r * HIDDEN + ci * 16), xr) *
                        sc[r * (HIDDEN / GROUP) + (ci >> 2)];
                p = mb::warp_sum(p);
                if (c.lane == 0) S.red[c.cw][r] = p;
            }
            cbar();
            if (c.ct < nrow) {
                float sum = 0.f;
#pragma unroll
                for (int w16 = 0; w16 < kConsumerWarps; w16++) sum += S.red[w16][c.ct];
                const int row = hd.first + c.ct;
                dw_store(scr.xin + row, S.xs[row] + sum, make_tag(epoch, l, PH_X));
            }
            give_back(c, cur);
            remaining--;
        }
        stamp(a, cta, c.ct, 2 + l * 12 + 8);
    }

    if (project) {
        // ---- final norm + tied head, logits kept in shared memory for selection
        if (!gather<1>(c, scr.xin, DIM, make_tag(epoch, LAYERS - 1, PH_X), S.xs)) return drain(c, cur);
        stamp(a, cta, c.ct, 300);
        const int lo = a.P->head_lo[cta], n = a.P->head_lo[cta + 1] - lo;
        bool first = true;
        for (;;) {
            const int more = next_is(c, cur, remaining, HEAD, LAYERS);
            if (more < 0) return drain(c, cur);
            if (!more) break;
            const uint8_t *w = take(c, cur, HEAD);
            if (!w) return drain(c, cur);
            if (first) {
                rmsnorm(c, S.xs, reinterpret_cast<const float *>(w + kGainOff), S.ns);
                if (cta == 0)
                    for (int i = c.ct; i < DIM; i += kNT) a.b.hidden[i] = S.ns[i];
                load_x896(S.ns, c.lane, xr);
                first = false;
            }
            const ChunkHdr hd = *reinterpret_cast<const ChunkHdr *>(w);
            const int nrow = hd.count;
            const uint8_t *rows = w + sizeof(ChunkHdr);
            const float *sc = reinterpret_cast<const float *>(rows + (size_t)nrow * DIM);
            for (int r = c.cw; r < nrow; r += kConsumerWarps) {
                const float d = row896(rows + (size_t)r * DIM, sc + r * 14, xr, c.lane);
                if (c.lane == 0) {
                    a.b.logits[hd.first + r] = d;
                    S.u.hl[hd.first + r - lo] = d;
                }
            }
            give_back(c, cur);
            remaining--;
        }
        cbar();
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
    stamp(a, cta, c.ct, 301);
    cbar();
    if (c.ct == 0) {
        __threadfence();
        const unsigned t = atomicAdd(&a.sy->done, 1u);
        S.flag = t == (unsigned)kCTAs - 1;
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
    stamp(a, cta, c.ct, 302);
    if (c.ct == 0) {
        a.b.st->steps++;
        a.sy->done = 0;
        const unsigned next = epoch + 1 >= (1u << 24) ? 1u : epoch + 1;
        __threadfence();
        atomicExch(&a.sy->epoch, next);
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

size_t scratch_words() { return (size_t)DIM + 2 * KV + kPartWords + DIM + DIM + HIDDEN; }

void carve_scratch(unsigned long long *base, Scratch *scr)
{
    scr->q = base;
    scr->kv = scr->q + DIM;
    scr->part = scr->kv + 2 * KV;
    scr->xmid = scr->part + kPartWords;
    scr->xin = scr->xmid + DIM;
    scr->h = scr->xin + DIM;
}

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

int build_plan(const FileHeader *hdr, const unsigned char *hfile, const unsigned char *dfile, Plan *hplan,
               Chunk **dchunks, uint8_t **dstream, size_t *stream_bytes, cudaStream_t s)
{
    std::vector<Chunk> chunks;
    std::vector<uint8_t> stream;
    stream.reserve((size_t)560 << 20);
    const FileTensor *t = hdr->t;
    auto align16 = [](size_t v) { return (v + 15) & ~(size_t)15; };
    // one chunk: header, int8 rows, fp32 scales, optional fp32 extras (biases)
    auto emit = [&](uint32_t kind, uint32_t layer, uint32_t first, uint32_t count,
                    const std::vector<std::pair<const FileTensor *, int>> &rows, const std::vector<float> &extra,
                    uint32_t gain_off) {
        Chunk ch{};
        ch.off = stream.size();
        ch.gain_off = gain_off;
        const ChunkHdr hd{kind, layer, first, count};
        const uint8_t *hb = reinterpret_cast<const uint8_t *>(&hd);
        stream.insert(stream.end(), hb, hb + sizeof hd);
        for (auto &r : rows) {
            const uint8_t *src = hfile + r.first->data + (size_t)r.second * r.first->cols;
            stream.insert(stream.end(), src, src + r.first->cols);
        }
        for (auto &r : rows) {
            const size_t g = r.first->cols / GROUP;
            const uint8_t *src = hfile + r.first->scales + (size_t)r.second * g * 4;
            stream.insert(stream.end(), src, src + g * 4);
        }
        const uint8_t *eb = reinterpret_cast<const uint8_t *>(extra.data());
        stream.insert(stream.end(), eb, eb + extra.size() * 4);
        stream.resize(align16(stream.size()), 0);
        ch.bytes = (uint32_t)(stream.size() - ch.off);
        const uint32_t limit = gain_off ? (uint32_t)kGainOff : (uint32_t)kSlotBytes;
        if (ch.bytes > limit || (gain_off && gain_off % 16)) return false;
        chunks.push_back(ch);
        return true;
    };
    for (int c = 0; c < kCTAs; c++) {
        hplan->chunk_begin[c] = (uint32_t)chunks.size();
        for (int l = 0; l < LAYERS; l++) {
            const FileTensor *lt = t + 1 + l * STRIDE;
            int lo, hi;
            std::vector<std::pair<const FileTensor *, int>> rows;
            std::vector<float> bias;
            split(kQkvPairs, kCTAs, c, lo, hi);
            for (int p = lo; p < hi; p++) {
                const FileTensor *m, *b;
                int tt;
                if (p < DIM / 2) { m = &lt[WQ]; b = &lt[BQ]; tt = p; }
                else if (p < DIM / 2 + KV / 2) { m = &lt[WK]; b = &lt[BK]; tt = p - DIM / 2; }
                else { m = &lt[WV]; b = &lt[BV]; tt = p - DIM / 2 - KV / 2; }
                const int r0 = (tt / 32) * HEAD_DIM + tt % 32;
                rows.push_back({m, r0});
                rows.push_back({m, r0 + 32});
                const float *bv = reinterpret_cast<const float *>(hfile + b->data);
                bias.push_back(bv[r0]);
                bias.push_back(bv[r0 + 32]);
            }
            if (!emit(QKV, l, lo, hi - lo, rows, bias, lt[ATTN_NORM].data)) return 1;
            rows.clear();
            split(DIM, kCTAs, c, lo, hi);
            for (int r = lo; r < hi; r++) rows.push_back({&lt[WO], r});
            if (!emit(OPROJ, l, lo, hi - lo, rows, {}, 0)) return 1;
            split(HIDDEN, kCTAs, c, lo, hi);
            for (int p0 = lo; p0 < hi; p0 += kGateupPerChunk) {
                const int p1 = p0 + kGateupPerChunk < hi ? p0 + kGateupPerChunk : hi;
                rows.clear();
                for (int p = p0; p < p1; p++) {
                    rows.push_back({&lt[WGATE], p});
                    rows.push_back({&lt[WUP], p});
                }
                if (!emit(GATEUP, l, p0, p1 - p0, rows, {}, p0 == lo ? lt[FFN_NORM].data : 0)) return 1;
            }
            rows.clear();
            split(DIM, kCTAs, c, lo, hi);
            for (int r = lo; r < hi; r++) rows.push_back({&lt[WDOWN], r});
            if (!emit(DOWN, l, lo, hi - lo, rows, {}, 0)) return 1;
        }
        int lo, hi;
        split(VOCAB, kCTAs, c, lo, hi);
        hplan->head_lo[c] = lo;
        hplan->head_begin[c] = (uint32_t)chunks.size();
        if (hi - lo > kHeadSlice) return 1;
        for (int r0 = lo; r0 < hi; r0 += kHeadPerChunk) {
            const int r1 = r0 + kHeadPerChunk < hi ? r0 + kHeadPerChunk : hi;
            std::vector<std::pair<const FileTensor *, int>> rows;
            for (int r = r0; r < r1; r++) rows.push_back({&t[0], r});
            if (!emit(HEAD, LAYERS, r0, r1 - r0, rows, {}, r0 == lo ? t[TENSORS - 1].data : 0)) return 1;
        }
    }
    hplan->chunk_begin[kCTAs] = (uint32_t)chunks.size();
    hplan->head_lo[kCTAs] = VOCAB;
    for (int c = 0; c < kCTAs; c++)
        if (hplan->chunk_begin[c + 1] - hplan->chunk_begin[c] > (uint32_t)kMaxChunksPerCta) return 1;
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
    hplan->blob = dfile;
    *stream_bytes = stream.size();
    return 0;
}

int enqueue_step(const Model *dm, const Plan *dplan, const Buffers &b, Sync *sync, const Scratch &scr, int mode,
                 const sampling::Params *prm, sampling::SeqState *seq, int *out_ring, int *out_count,
                 const int *prompt, unsigned *host_error, cudaStream_t s, unsigned long long *trace)
{
    Args a{dm, dplan, b, sync, scr, mode, prm, seq, out_ring, out_count, prompt, host_error, trace};
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
