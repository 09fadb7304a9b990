// Persistent batch-1 decode step for the grouped-Q8 model on B200.
//
// One cooperative launch of 148 CTAs (one per SM) runs the whole token.
//
// Weights: every CTA streams its own weights -- laid out at set-up as one contiguous
// region per CTA, in consumption order -- through a 4-slot shared-memory ring with
// cp.async.bulk copies completed on mbarriers; thread 0 starts the copy of chunk
// k + 4 as soon as the consumers give slot k back (the first four at the start).  Each chunk
// carries a 16-byte header (kind, layer, range) and its rows' scales and biases;
// chunks that start a normalised phase also receive the RMSNorm gain by a second bulk
// copy (an L2 hit: every CTA reads the same gain).  Weights do not depend on
// activations, so the stream runs ahead of the dependency chain by up to the ring
// depth.
//
// Matrix-vector products run on the int8 tensor cores (mma.sync m16n8k32): the
// stream stores every matrix as 16-row tiles already in the A-fragment order of that
// instruction (a lane's 16 bytes per 32-column step), and the activation enters as
// three int8 limbs per 64-column group, x = s (a0 + a1/254 + a2/254^2) with
// s = max|x| / 127 -- the B fragment's columns 0..2.  The int32 products of one group
// are exact; they are combined as (254 D0 + D1 + D2/254) * s/254 and scaled by the
// weight group's fp32 scale.  The (tile, group) units of a chunk are split evenly over
// the 16 consumer warps and the per-warp row sums added in warp order.
//
// Activations: the 16 warps exchange every cross-CTA value as a 64-bit data
// word (float | tag << 32, tag = epoch << 8 | layer << 3 | phase) written with one
// relaxed store and polled directly by its readers; words read by every CTA are
// written to four replicas.  There are no counters, fences or second loads between
// phases; each reader waits exactly for the words it needs.
// Per layer: QKV (+bias, split-half RoPE, KV write) -> attention split over the
// positions of each query head (K/V of past positions are prefetched with cp.async
// before the query exists); each split projects its unnormalised output through the
// head's 64 columns of O, the splits of a head exchange their (max, sum of weights)
// and scale their projection to the head's softmax, and the 896 rows are all-reduced
// like the down projection below -> x_mid in every CTA -> RMSNorm -> gate/up + SwiGLU on this
// CTA's own slice of the hidden units -> the down projection of that slice for all
// 896 rows (split-K), added into one accumulator per row as 64-bit fixed point
// (value * 2^32, red.add: integer sums do not depend on the order of arrival, so
// the result is deterministic) whose low byte counts the additions -> every CTA polls
// the 896 accumulators until each holds all 148 additions and adds the sums to its
// own copy of x_mid: the next layer's input, with no gather.
// The vocabulary head is fused with the repetition penalty, the control mask and a
// per-CTA top-k; the last CTA to finish (one atomic ticket) merges the candidates,
// draws the token and advances the epoch.
//
// Every wait is bounded (~2 s of clock cycles); on expiry the kernel records an
// error word (device and mapped host memory), drains its own bulk copies and exits.
// The arithmetic follows the reference (src/minimind.cu:67-123, src/minimind.cpp:51-82):
// fp32 activations between the matrix products, int8 weights, one fp32 scale per 64
// weights; the products themselves use the exact integer limb form above.
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
constexpr long long kErrorPollCycles = 50000;  // spin before a wait starts reading the error flag
constexpr int kQkvPairs = (DIM + 2 * KV) / 2;  // 576
constexpr int kSteps = DIM / 32;               // 32-column MMA steps of a 896-wide row
constexpr int kGroups = DIM / GROUP;           // 14 scale groups of a 896-wide row
constexpr int kTileBytes = kSteps * 32 * 16;   // one 16-row tile of a 896-wide matrix
constexpr int kHalfBytes = kSteps * 32 * 8;    // one 8-row tile (rows 8..15 absent)
constexpr int kGateupPerChunk = 16;            // hidden units per gate/up chunk (two tiles)
constexpr int kHeadPerChunk = 32;              // vocabulary rows per head chunk (two tiles)
constexpr int kHeadSlice = 1040;               // >= ceil(VOCAB / kCTAs)
constexpr int kDownTiles = DIM / 16;           // 56 row tiles of the down projection
constexpr int kPartWords = HEADS * kMaxSplit * 2;   // (max, sum of weights) of every attention split
constexpr int kOStepBytes = kDownTiles * 512;        // one 32-column step of a head's O columns, all 896 rows
constexpr int kOHeadBytes = 2 * kOStepBytes;
constexpr int kGpStride = kConsumerWarps + 1;  // padded: conflict-free row sums
// The thread that starts the ring's bulk copies in the layer loop: lane 0 of the last
// warp, which has the least work on the critical path (warp 0 merges and quantizes;
// warps 14 and 15 sit out the grouped matrix-vector products).
constexpr int kIssuer = kNT - 32;
constexpr int kKStride = HEAD_DIM + 4;         // cached key row in shared memory: conflict-free float4 reads
constexpr int kMaxAttnWarps = (kAttnLenMax + 7) / 8;  // warps holding positions of a split (8 each)
static_assert(kMaxAttnWarps <= kConsumerWarps, "attention warps");
constexpr int kStrideKv = replica_stride(2 * KV);
constexpr float kMagic = 12582912.0f;          // 1.5 * 2^23: v + kMagic rounds v to an integer (|v| < 2^22)
static_assert(DIM % 64 == 0 && kCTAs % 4 == 0, "layout");

enum Phase { PH_QKV = 0, PH_ATTN = 1 };
constexpr float kFixInv = 1.0f / 4294967296.0f;  // partial sums as fixed point, scaled by 2^32 ...
// ... in bits 8..63 of an accumulator word; bits 0..7 count the additions (< 256), so a
// reader sees from the word alone when every contributor's addition has landed.  Each
// addition is (q << 8) + 1, q = rint(v * 2^32): the low byte only ever gains the +1s,
// and the sum is the word shifted right arithmetically by 8 (|sum| < 2^23 fits).
// Every accumulator has kAccRep copies and writer w adds into copy w % kAccRep: the L2
// slice that owns a line serves its red operations one by one, and 148 writers on one
// copy queue behind each other; readers add the copies' integer sums (exact, so the
// result does not depend on the split).  Two copies measured best: each further copy
// costs the 148 readers one more 32-byte poll per round.
constexpr int kAccRep = 2;
// Each 32-byte sector of four accumulator words gets its own 128-byte line
// (kSecPerLine sectors per line): the red operations on a line are served one by one,
// and a reader's poll is one sector either way.
constexpr int kSecPerLine = 1;
constexpr int kAccCopyWords = (DIM / 4 / kSecPerLine) * 16;  // one copy of DIM sums, padded
__host__ __device__ inline int acc_word(int row)
{
    const int sec = row >> 2;
    return (sec / kSecPerLine) * 16 + (sec % kSecPerLine) * 4 + (row & 3);
}

struct Smem {
    uint8_t ring[kSlots][kSlotBytes];
    __align__(16) float xs[DIM];  // residual (x_in, then x_mid) of the current layer
    __align__(16) float ns[DIM];  // normalised input / attention output
    union __align__(16) {
        struct {
            float k[kAttnLenMax][kKStride];
            float v[kAttnLenMax][HEAD_DIM];
            float q[HEAD_DIM];
            float wp[kConsumerWarps][HEAD_DIM + 4];  // per-warp partials: max, sum of weights, -, -, 64 accumulators
        } att;
        float hl[kHeadSlice];      // this CTA's slice of the logits
    } u;
    __align__(16) uint2 bf[kSteps][32];  // B fragments of the current 896-wide input (lanes 12..31 zero)
    __align__(16) uint2 bfh[2][32];      // B fragments of the SwiGLU slice (lanes 12..31 zero)
    __align__(16) uint2 bfo[2][32];      // B fragments of this split's attention output (64 dims)
    float so;                            // its scale / 254
    float att_m, att_l, att_w;           // this split's max and sum of weights; its weight in the head
    float gp[5 * 16][kGpStride];   // per-group partial row sums of the current job (<= 5 tiles)
    float sxs[kGroups];            // input scale / 254 per group
    __align__(16) float hst[2][32];  // SwiGLU outputs: the block's at column unit % 32, the piece's at 0..7
    float sh[2];                   // their scale / 254, per down step
    __align__(16) float red[kConsumerWarps][8];  // also read as 64-bit keys (block_max)
    float rc[HEAD_DIM / 2], rs[HEAD_DIM / 2];  // RoPE cos/sin at pos
    Chunk desc[kMaxChunksPerCta];  // this CTA's chunk descriptors
    // pointers the layer loop needs, copied from global memory once: a pointer load from
    // global memory feeding a second load puts two L2 round trips on the path
    const float *gain[2][LAYERS];  // RMSNorm gains: [0] attention, [1] FFN
    const float *final_gain;       // the final norm's
    const uint8_t *ofrag;          // the plan's O-by-head fragments and scales
    const float *oscale;
    unsigned long long full[kSlots];
    int flag;
    int token, pos;
    int issued;                  // chunks whose bulk copy has been started
    int slot_done[kSlots];       // head phase: tiles of the slot's chunk finished
    int slot_fill[kSlots];       // the chunk last issued into each slot
};
static_assert(sizeof(Smem) <= 232448, "shared memory per CTA");

// Hidden units whose gate/up rows and down-projection columns CTA c owns: the
// 32-unit block [32c, 32c + 32) and, for the last 16 CTAs, an 8-unit piece of the four
// spare blocks, [4736 + 8j, 4736 + 8j + 8) for CTA 132 + j (4864 = 148 * 32 + 16 * 8).
// Down-projection step 0 covers the CTA's block (its own chunk); the piece's 8 down
// columns ride in the piece's gate/up chunk, after its tile, so the CTA never waits
// for a second down chunk: its three gate/up chunks and its down chunk fill the ring
// together.
constexpr int kSpareFirst = kCTAs - (HIDDEN - 32 * kCTAs) / 8;  // 132
static_assert(32 * kCTAs + 8 * (kCTAs - kSpareFirst) == HIDDEN, "hidden slices");
__host__ __device__ inline bool has_spare(int c) { return c >= kSpareFirst; }
__host__ __device__ inline int spare_lo(int c) { return 32 * kCTAs + 8 * (c - kSpareFirst); }
// The piece's down columns in its gate/up chunk, after the tile and the tile rows'
// scales: [kDownTiles][16][8 B] -- registers a0 and a1 of lanes 4 g + tig, tig < 2, of a
// 32-column step whose columns 0..7 are the piece's units (the rest zero) -- then the
// 896 rows' scales of the piece's 64-column group.
constexpr int kSpareDownOff = kTileBytes + 16 * kGroups * 4;
constexpr int kSpareDownBytes = kDownTiles * 16 * 8;

// ---- low-level primitives --------------------------------------------------

// Error paths (a wait that has spun for a long time, a failed check) are kept out of
// line: they never run on the hot path, and inlined copies of them would crowd the
// per-layer loop out of the instruction caches.
#define Q8P_COLD __device__ __noinline__

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

Q8P_COLD void fail(Sync *sy, unsigned *host_error, unsigned code)
{
    atomicCAS(&sy->error, 0u, code);
    *(volatile unsigned *)host_error = code;
    __threadfence_system();
}

// A wait that has spun for `spun` cycles gives up when another CTA has recorded an
// error -- read only once the wait is long, since the flag costs an L2 round trip --
// or when the bound expires (recorded here with `code`).
Q8P_COLD bool give_up_slow(Sync *sy, unsigned *host_error, long long spun, unsigned code)
{
    if (spun > kTimeoutCycles) {
        fail(sy, host_error, code);
        return true;
    }
    return ld_volatile(&sy->error) != 0;
}

MB_DEV bool give_up(Sync *sy, unsigned *host_error, long long spun, unsigned code)
{
    if (spun < kErrorPollCycles) return false;
    return give_up_slow(sy, host_error, spun, code);
}

MB_DEV bool mbar_wait(unsigned long long *bar, uint32_t parity, Sync *sy, unsigned *host_error)
{
    if (mbar_test(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_test(bar, parity)) return true;
        if (give_up(sy, host_error, clock64() - t0, 2)) return false;
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

// the same word into every replica of an array whose copies are `stride` words apart
MB_DEV void dw_store_rep(unsigned long long *p, int stride, float v, uint32_t tag)
{
#pragma unroll
    for (int r = 0; r < kReplicas; r++) dw_store(p + r * stride, v, tag);
}

MB_DEV unsigned long long dw_load(const unsigned long long *p)
{
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// One counted fixed-point addition (the result is not returned: a reduction in L2).
// rint(v * 2^32) from two 32-bit conversions, which issue faster than one 64-bit one:
// hi = rint(v * 2^8), then the remainder v * 2^8 - hi (exact, |.| <= 1/2) scaled by 2^24;
// hi * 2^24 is even, so rint(hi * 2^24 + r * 2^24) = hi * 2^24 + rint(r * 2^24), ties
// included.  Exact for |v| < 2^23, the format's range.
MB_DEV void fix_add(unsigned long long *p, float v)
{
    const float x = v * 256.f;
    const int hi = __float2int_rn(x);
    const int lo = __float2int_rn((x - (float)hi) * 16777216.f);
    const unsigned long long q = (unsigned long long)(((long long)hi << 24) + lo);
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"((q << 8) + 1ull) : "memory");
}

MB_DEV uint32_t make_tag(uint32_t epoch, int layer, int phase) { return (epoch << 8) | (layer << 3) | phase; }

// ---- consumer-side helpers --------------------------------------------------

struct Ctx {
    Smem &S;
    Sync *sy;
    unsigned *host_error;
    int ct, cw, lane;
    int rep;                        // replica this CTA reads
    const uint8_t *stream, *blob;   // this step's weight stream and the model file (gains)
    uint32_t nchunks;               // chunks this CTA streams in this step
    uint64_t policy;                // L2 evict-first for the stream
};

// 32-byte relaxed load of four data words (one L2 request instead of four)
MB_DEV void dw_load4(const unsigned long long *p, unsigned long long (&v)[4])
{
    asm volatile("ld.relaxed.gpu.global.v4.u64 {%0,%1,%2,%3}, [%4];"
                 : "=l"(v[0]), "=l"(v[1]), "=l"(v[2]), "=l"(v[3])
                 : "l"(p)
                 : "memory");
}

// ---- int8 tensor-core matrix-vector products ------------------------------------

MB_DEV void mma_s8(int (&d)[4], const uint4 &a, const uint2 &b)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y));
}

// The three int8 limbs of four values already multiplied by 127 / max|x|, packed one
// limb per word: q = a0 + a1/254 + a2/254^2 + e, |e| <= 1/(2*254^2).  Rounding is to
// nearest even through kMagic; |q| <= 127 (to within rounding) keeps every limb in
// [-127, 127].
MB_DEV void limbs4(const float (&q)[4], uint32_t &p0, uint32_t &p1, uint32_t &p2)
{
    uint32_t b[3][4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float t0 = __fadd_rn(q[j], kMagic);
        const float a0 = __fsub_rn(t0, kMagic);
        const float r1 = __fmul_rn(__fsub_rn(q[j], a0), 254.f);
        const float t1 = __fadd_rn(r1, kMagic);
        const float a1 = __fsub_rn(t1, kMagic);
        const float r2 = __fmul_rn(__fsub_rn(r1, a1), 254.f);
        const float t2 = __fadd_rn(r2, kMagic);
        b[0][j] = __float_as_uint(t0);
        b[1][j] = __float_as_uint(t1);
        b[2][j] = __float_as_uint(t2);
    }
    // low byte of each word (two's complement of the integer), four per word
    p0 = __byte_perm(__byte_perm(b[0][0], b[0][1], 0x0040), __byte_perm(b[0][2], b[0][3], 0x0040), 0x5410);
    p1 = __byte_perm(__byte_perm(b[1][0], b[1][1], 0x0040), __byte_perm(b[1][2], b[1][3], 0x0040), 0x5410);
    p2 = __byte_perm(__byte_perm(b[2][0], b[2][1], 0x0040), __byte_perm(b[2][2], b[2][3], 0x0040), 0x5410);
}

// Column block of quantizer thread t < 224 of a 896-wide input: step ks = t >> 3, lane
// column tig = (t >> 1) & 3, half h = t & 1 own columns 32 ks + 16 h + 4 tig + {0..3},
// which are B-fragment register h of lanes 4n + tig (limb n).  The 16 threads of a
// 64-column group form an aligned 16-lane block.
MB_DEV int quant_col(int t) { return 32 * (t >> 3) + 16 * (t & 1) + 4 * ((t >> 1) & 3); }

// Four values n[] of thread t (group max m already reduced over its 16 lanes) -> limbs
// into S.bf and, from the group's first thread, the group scale / 254.  127 / m comes
// from the fast divide (within 2 ulp: |q| stays <= 127 to within rounding), so the
// values the limbs stand for are off by about 1e-7 relative, the order of the limbs'
// own resolution; an IEEE division here cost two of them per quantization on the
// critical path.
MB_DEV void put_limbs(Smem &S, int t, const float (&n)[4], float m)
{
    const int ks = t >> 3, tig = (t >> 1) & 3, h = t & 1;
    const float inv = m > 0.f ? __fdividef(127.f, m) : 0.f;
    const float q[4] = {n[0] * inv, n[1] * inv, n[2] * inv, n[3] * inv};
    uint32_t p0, p1, p2;
    limbs4(q, p0, p1, p2);
    if ((t & 15) == 0) S.sxs[ks >> 1] = m * (1.0f / (127.f * 254.f));
    uint32_t *b = reinterpret_cast<uint32_t *>(&S.bf[ks][0]);
    b[2 * tig + h] = p0;
    b[2 * (4 + tig) + h] = p1;
    b[2 * (8 + tig) + h] = p2;
}

// Maximum of m >= 0 over each aligned 16-lane half of the warp (two whole-warp reduxes,
// each seeing the other half as zeros).
MB_DEV float group_max16(float m)
{
    const bool lo = (threadIdx.x & 16) == 0;
    const float a = mb::warp_max(lo ? m : 0.f), b = mb::warp_max(lo ? 0.f : m);
    return lo ? a : b;
}

// The four gain values of thread ct's columns (see norm_quantize), loaded ahead of use.
MB_DEV float4 load_gain(int ct, const float *gain)
{
    return ct < 256 ? __ldg(reinterpret_cast<const float4 *>(gain + quant_col(min(ct, 223))))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
}

// RMSNorm with the gain g, in the reference's form ((x * s) * g, s = 1/sqrt(sum x^2 /
// DIM + eps)) with s from the hardware reciprocal square root (within 2 ulp of the
// rounded 1/sqrtf), quantized straight into S.bf / S.sxs.  Thread ct < 224 (warps 0..6)
// owns columns quant_col(ct) .. + 3 of x and g (g from load_gain).  In two halves around
// a consumer barrier, so that the first can be fused into the reduction that produces x.

// First half: the warp sums of x^2 into S.red and pm = the 16-lane group max of |x * g|.
// Warps 0..6, all lanes.
MB_DEV void norm_sums(Smem &S, int ct, float4 g, float4 x, float &pm)
{
    float ss = fmaf(x.w, x.w, fmaf(x.z, x.z, fmaf(x.y, x.y, x.x * x.x)));
    pm = fmaxf(fmaxf(fabsf(x.x * g.x), fabsf(x.y * g.y)), fmaxf(fabsf(x.z * g.z), fabsf(x.w * g.w)));
    ss = mb::warp_sum(ss);
    pm = group_max16(pm);
    if ((ct & 31) == 0) S.red[ct >> 5][0] = ss;
}

// Second half, after the barrier: s from the seven warp sums, the limbs of (x * s) * g
// (with keep also the values into S.ns); every consumer thread calls it (one barrier).
MB_DEV void norm_finish(Smem &S, int ct, float4 g, float4 x, float pm, int keep)
{
    if (ct < DIM / 4) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < 7; w++) sum += S.red[w][0];
        const float s = rsqrtf(sum * (1.0f / DIM) + RMS_EPS);
        const float n[4] = {(x.x * s) * g.x, (x.y * s) * g.y, (x.z * s) * g.z, (x.w * s) * g.w};
        if (keep) *reinterpret_cast<float4 *>(S.ns + quant_col(ct)) = make_float4(n[0], n[1], n[2], n[3]);
        put_limbs(S, ct, n, pm * s);
    }
    cbar();
}

// The whole norm of S.xs; every consumer thread calls it (two barriers).
MB_DEV void norm_quantize(Smem *Sp, int ct, float4 g, int keep)
{
    Smem &S = *Sp;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    float pm = 0.f;
    if (ct < DIM / 4) {
        x = *reinterpret_cast<const float4 *>(S.xs + quant_col(ct));
        norm_sums(S, ct, g, x, pm);
    }
    cbar();
    norm_finish(S, ct, g, x, pm, keep);
}

// D fragments of one group -> the limb combination (254 D0 + D1 + D2/254) of rows g
// (v0) and g + 8 (v1); valid in lanes with tig == 0 (limb 2 comes from lane + 1).
MB_DEV void combine(const int (&d)[4], float &v0, float &v1)
{
    const int e0 = __shfl_down_sync(0xffffffffu, d[0], 1), e2 = __shfl_down_sync(0xffffffffu, d[2], 1);
    v0 = fmaf((float)e0, 1.f / 254.f, (float)(d[0] * 254 + d[1]));
    v1 = fmaf((float)e2, 1.f / 254.f, (float)(d[2] * 254 + d[3]));
}

// The 16-row tiles of up to three chunks of 896-wide rows: tile t is tile t & 1 of
// chunk t >> 1 (fragments [tile][kSteps][32 lanes][16 B], then the tile rows' scales
// [16][kGroups] per tile), or, when half, the one 8-row tile of chunk 0 ([kSteps][32][8 B],
// registers a0 and a2; scales [8][kGroups]).
struct Tiles {
    const uint8_t *frag[3];
    const float *sc[3];
    int T, half;
};

// Tiles x groups: warp w < kGroups takes group w (k-steps 2w, 2w + 1) of every tile, so
// it loads its two B fragments and its input scale once and reuses them across the tiles
// (shared-memory bandwidth, not latency, bounds this loop); its row sums go to
// S.gp[row][w] and row_sum() adds the 14 groups of a row in order.  MAXT >= T; an
// iteration t >= T repeats tile T - 1 (no branch around the loads) and stores nothing.
template <int MAXT>
MB_DEV void gemv_mma(Smem *Sp, int cw, int lane, Tiles tl)
{
    Smem &S = *Sp;
    if (cw >= kGroups) return;
    const int g = lane >> 2, tig = lane & 3, grp = cw;
    const uint2 b0 = S.bf[2 * grp][lane], b1 = S.bf[2 * grp + 1][lane];
    const float f = S.sxs[grp];
    // every tile's first MMA, then every second one, then the combines: each tile's
    // MMA -> MMA -> shuffle -> convert chain is about 90 cycles, paid once, not per tile
    int d[MAXT][4];
#pragma unroll
    for (int k = 0; k < 2; k++)
#pragma unroll
        for (int i = 0; i < MAXT; i++) {
            const int t = min(i, tl.T - 1), ch = t >> 1;
            const uint8_t *fr = (ch == 0 ? tl.frag[0] : ch == 1 ? tl.frag[1] : tl.frag[2]) + (t & 1) * kTileBytes;
            uint4 a;
            if (tl.half) {
                const uint2 x = *reinterpret_cast<const uint2 *>(fr + ((size_t)(2 * grp + k) * 32 + lane) * 8);
                a = make_uint4(x.x, 0u, x.y, 0u);
            } else {
                a = *reinterpret_cast<const uint4 *>(fr + ((size_t)(2 * grp + k) * 32 + lane) * 16);
            }
            if (k == 0) {
#pragma unroll
                for (int j = 0; j < 4; j++) d[i][j] = 0;
            }
            mma_s8(d[i], a, k == 0 ? b0 : b1);
        }
#pragma unroll
    for (int i = 0; i < MAXT; i++) {
        const int t = min(i, tl.T - 1), ch = t >> 1;
        const float *sc = (ch == 0 ? tl.sc[0] : ch == 1 ? tl.sc[1] : tl.sc[2]) + (t & 1) * 16 * kGroups;
        float v0, v1;
        combine(d[i], v0, v1);
        // (a half tile has 8 rows of scales: row g stands in for the absent row g + 8)
        const float s0 = sc[g * kGroups + grp], s1 = sc[(tl.half ? g : g + 8) * kGroups + grp];
        if (tig == 0 && i < tl.T) {
            S.gp[16 * t + g][cw] = v0 * (s0 * f);
            if (!tl.half) S.gp[16 * t + g + 8][cw] = v1 * (s1 * f);
        }
    }
}

// Row `row` of the current job: its 14 group partials in group order (after a
// consumer barrier).
MB_DEV float row_sum(const Ctx &c, int row)
{
    const float *v = c.S.gp[row];
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kGroups; w++) s += v[w];
    return s;
}

// Down projection, one 32-column step of this CTA's hidden units for all 896 rows
// ([kDownTiles][32 lanes][16 B]; a spare piece's 8-column form [kDownTiles][16][8 B]:
// registers a0, a1 of lanes with tig < 2): warp cw's tiles [56 cw/16, 56 (cw+1)/16); the
// step's partials (v * weight scale * input scale sx) are added to acc[tile][row g |
// row g + 8].  A warp with three tiles also multiplies a fourth (the next warp's first)
// into an acc entry its caller ignores: no branch around the loads.
// The block's down step and, WithPiece, the piece's step in one pass over the warp's
// tiles (the two MMAs of a tile are independent): each acc entry adds the block's
// product, then the piece's (the order of two separate passes).
template <bool WithPiece>
MB_DEV void down_steps(Ctx &c, const uint8_t *frag, const float *sw, const uint2 (&bf0)[32], float sx0,
                       const uint8_t *pfrag, const float *psw, const uint2 (&bf1)[32], float sx1, float (&acc)[4][2])
{
    const int t0 = kDownTiles * c.cw / kConsumerWarps;
    const uint2 b0 = bf0[c.lane], b1 = bf1[c.lane];
    const int g = c.lane >> 2, tig = c.lane & 3;
    // every MMA of the warp is issued before the first combine: a tile's MMA -> shuffle
    // -> convert chain is about 70 cycles, and tile after tile it would be paid four times
    int d[4][4], e[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = min(t0 + i, kDownTiles - 1);
#pragma unroll
        for (int j = 0; j < 4; j++) d[i][j] = e[i][j] = 0;
        mma_s8(d[i], *reinterpret_cast<const uint4 *>(frag + ((size_t)t * 32 + c.lane) * 16), b0);
        if (WithPiece) {
            uint4 a = make_uint4(0u, 0u, 0u, 0u);
            const uint2 v = *reinterpret_cast<const uint2 *>(pfrag + ((size_t)t * 16 + 2 * g + (tig & 1)) * 8);
            if (tig < 2) {
                a.x = v.x;
                a.y = v.y;
            }
            mma_s8(e[i], a, b1);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = min(t0 + i, kDownTiles - 1);
        float v0, v1;
        combine(d[i], v0, v1);
        const int r0 = 16 * t + g;
        acc[i][0] = fmaf(v0, sw[r0] * sx0, acc[i][0]);
        acc[i][1] = fmaf(v1, sw[r0 + 8] * sx0, acc[i][1]);
        if (WithPiece) {
            float w0, w1;
            combine(e[i], w0, w1);
            acc[i][0] = fmaf(w0, psw[r0] * sx1, acc[i][0]);
            acc[i][1] = fmaf(w1, psw[r0 + 8] * sx1, acc[i][1]);
        }
    }
}

MB_DEV size_t kv_index(int layer, int kvh, int pos)
{
    return (((size_t)layer * KV_HEADS + kvh) * CONTEXT + pos) * HEAD_DIM;
}

// S.xs += the 896 counted fixed-point sums at acc once they hold `count` additions in
// all: writer w adds to copy w % kAccRep (copies kAccCopyWords apart), so copy r waits for
// ceil((count - r) / kAccRep) of them.  Thread t < 224 polls its four words of every
// copy (one 32-byte request per copy and round).  Every consumer thread returns the
// same verdict (ends with a barrier).
MB_DEV bool add_sums(Ctx &c, const unsigned long long *acc, unsigned count)
{
    int ok = 1;
    if (c.ct < DIM / 4) {
        unsigned long long v[kAccRep][4];
        unsigned need[kAccRep];
#pragma unroll
        for (int r = 0; r < kAccRep; r++) {
            need[r] = (count + kAccRep - 1 - r) / kAccRep;
            dw_load4(acc + r * kAccCopyWords + acc_word(4 * c.ct), v[r]);
        }
        long long t0 = 0;
        for (;;) {
            bool done = true;
#pragma unroll
            for (int r = 0; r < kAccRep; r++)
#pragma unroll
                for (int j = 0; j < 4; j++) done = done && (unsigned)(v[r][j] & 0xFFu) == need[r];
            if (done) break;
            if (t0 == 0) {
                t0 = clock64();
            } else if (give_up(c.sy, c.host_error, clock64() - t0, 1)) {
                ok = 0;
                break;
            }
#pragma unroll
            for (int r = 0; r < kAccRep; r++) dw_load4(acc + r * kAccCopyWords + acc_word(4 * c.ct), v[r]);
        }
        long long s[4] = {0, 0, 0, 0};
#pragma unroll
        for (int r = 0; r < kAccRep; r++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[j] += (long long)v[r][j] >> 8;
        float4 x = *reinterpret_cast<const float4 *>(c.S.xs + 4 * c.ct);
        x.x += __ll2float_rn(s[0]) * kFixInv;
        x.y += __ll2float_rn(s[1]) * kFixInv;
        x.z += __ll2float_rn(s[2]) * kFixInv;
        x.w += __ll2float_rn(s[3]) * kFixInv;
        *reinterpret_cast<float4 *>(c.S.xs + 4 * c.ct) = x;
    }
    return cbar_and(ok) != 0;
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

struct Cursor {
    uint32_t k;  // chunks consumed
};

// add_sums for the reductions that feed a norm: thread t < 224 polls the words of its
// norm columns quant_col(t) .. + 3 (32 bytes per copy), adds them to S.xs and to x, and
// runs the norm's first half on x (pm as norm_sums gives it) before the barrier that the
// reduction ends with anyway; meanwhile the threads t >= 224, idle here, run side()
// and the issuer thread (one of them) check() -- the next phase's chunks: landed,
// headers valid -- whose verdict joins the barrier's.  The caller finishes with
// norm_finish.
template <typename Check, typename Side>
MB_DEV bool add_sums_norm(Ctx &c, const unsigned long long *acc, unsigned count, float4 g, float4 &x, float &pm,
                          Check check, Side side)
{
    int ok = 1;
    x = make_float4(0.f, 0.f, 0.f, 0.f);
    pm = 0.f;
    if (c.ct < DIM / 4) {
        const int col = quant_col(c.ct);
        unsigned long long v[kAccRep][4];
        unsigned need[kAccRep];
#pragma unroll
        for (int r = 0; r < kAccRep; r++) {
            need[r] = (count + kAccRep - 1 - r) / kAccRep;
            dw_load4(acc + r * kAccCopyWords + acc_word(col), v[r]);
        }
        long long t0 = 0;
        for (;;) {
            bool done = true;
#pragma unroll
            for (int r = 0; r < kAccRep; r++)
#pragma unroll
                for (int j = 0; j < 4; j++) done = done && (unsigned)(v[r][j] & 0xFFu) == need[r];
            if (done) break;
            if (t0 == 0) {
                t0 = clock64();
            } else if (give_up(c.sy, c.host_error, clock64() - t0, 1)) {
                ok = 0;
                break;
            }
#pragma unroll
            for (int r = 0; r < kAccRep; r++) dw_load4(acc + r * kAccCopyWords + acc_word(col), v[r]);
        }
        long long s4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int r = 0; r < kAccRep; r++)
#pragma unroll
            for (int j = 0; j < 4; j++) s4[j] += (long long)v[r][j] >> 8;
        x = *reinterpret_cast<const float4 *>(c.S.xs + col);
        x.x += __ll2float_rn(s4[0]) * kFixInv;
        x.y += __ll2float_rn(s4[1]) * kFixInv;
        x.z += __ll2float_rn(s4[2]) * kFixInv;
        x.w += __ll2float_rn(s4[3]) * kFixInv;
        *reinterpret_cast<float4 *>(c.S.xs + col) = x;
        norm_sums(c.S, c.ct, g, x, pm);
    }
    if (c.ct == kIssuer && !check()) ok = 0;
    if (c.ct >= DIM / 4) side();
    return cbar_and(ok) != 0;
}

// attention split of one query head: positions [p0, p0+np)
struct AttnUnit {
    int head, split, p0, np;
};

// Threads [t0, t0 + nt): start the asynchronous copy of the past K/V rows of layer l for
// this CTA's attention split into shared memory (they do not depend on this step), and
// (thread t0) the L2 prefetch of the head's O columns and scales, wanted after the
// attention.
MB_DEV void attn_prefetch(Ctx &c, const Args &a, const AttnUnit &unit, int l, int pos, int t0, int nt)
{
    const int kvh = unit.head / GQA;
    const int past = min(unit.np, pos - unit.p0);  // rows < pos
    const float *kb = a.b.kc + kv_index(l, kvh, unit.p0);
    const float *vb = a.b.vc + kv_index(l, kvh, unit.p0);
    for (int i = c.ct - t0; i < past * (HEAD_DIM / 4); i += nt) {
        const int p = i / (HEAD_DIM / 4), q4 = i % (HEAD_DIM / 4);
        cp_async16(&c.S.u.att.k[p][q4 * 4], kb + p * HEAD_DIM + q4 * 4);
        cp_async16(&c.S.u.att.v[p][q4 * 4], vb + p * HEAD_DIM + q4 * 4);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (c.ct == t0) {
        const uint8_t *of = c.S.ofrag + (size_t)(l * HEADS + unit.head) * kOHeadBytes;
        const float *os = c.S.oscale + (size_t)(l * HEADS + unit.head) * DIM;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(of), "r"(kOHeadBytes) : "memory");
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(os), "r"(DIM * 4) : "memory");
    }
}

// Issuer-side checks of the chunks the next phase reads without waiting.  The QKV job of
// layer l at the cursor: landed, a QKV header of layer l with 1..4 pairs.
MB_DEV bool qkv_ready(Ctx &c, const Cursor &cur, int remaining, int l)
{
    const uint32_t slot = cur.k % kSlots;
    if (remaining < 1) {
        fail(c.sy, c.host_error, 4);
        return false;
    }
    if (!mbar_wait(&c.S.full[slot], (cur.k / kSlots) & 1, c.sy, c.host_error)) return false;
    const ChunkHdr *h = reinterpret_cast<const ChunkHdr *>(c.S.ring[slot]);
    if (h->kind != QKV || h->layer != (uint32_t)l || h->count < 1 || h->count > 4) {
        fail(c.sy, c.host_error, 4);
        return false;
    }
    return true;
}

// Layer l's FFN chunks from the cursor: ngu gate/up chunks (two of 16 units, then the
// 8-unit piece if the CTA has one) and the first down chunk after them (ngu + 1 <=
// kSlots: all resident together).
MB_DEV bool ffn_ready(Ctx &c, const Cursor &cur, int remaining, int l, int ngu)
{
    if (remaining < ngu + 1) {
        fail(c.sy, c.host_error, 4);
        return false;
    }
    bool ok = true;
    for (int i = 0; i <= ngu; i++) {
        const uint32_t k = cur.k + (uint32_t)i;
        if (!mbar_wait(&c.S.full[k % kSlots], (k / kSlots) & 1, c.sy, c.host_error)) return false;
        const ChunkHdr *h = reinterpret_cast<const ChunkHdr *>(c.S.ring[k % kSlots]);
        if (i < ngu)
            ok = ok && h->kind == GATEUP && h->layer == (uint32_t)l && h->count == (i < 2 ? 16u : 8u);
        else
            ok = ok && h->kind == DOWN && h->layer == (uint32_t)l && h->first == 0 && h->count == 1;
    }
    if (!ok) fail(c.sy, c.host_error, 4);
    return ok;
}


// Wait for the next chunk; returns the slot (header first) or null on failure.
// Every chunk's range is checked against the bounds its consumers assume.
MB_DEV const uint8_t *take(Ctx &c, Cursor &cur, uint32_t kind)
{
    const uint32_t slot = cur.k % kSlots, use = cur.k / kSlots;
    if (!mbar_wait(&c.S.full[slot], use & 1, c.sy, c.host_error)) return nullptr;
    const uint8_t *w = c.S.ring[slot];
    const ChunkHdr *h = reinterpret_cast<const ChunkHdr *>(w);
    bool ok = h->kind == kind && h->count >= 1;
    if (kind == QKV) ok = ok && h->count <= 4;
    if (kind == GATEUP) ok = ok && (h->count == 8 || h->count == (uint32_t)kGateupPerChunk);
    if (kind == HEAD) ok = ok && h->count <= (uint32_t)kHeadPerChunk;
    if (kind == DOWN) ok = ok && h->count == 1 && h->first == 0;
    if (!ok) {
        if (c.ct == 0) fail(c.sy, c.host_error, 4);
        return nullptr;
    }
    return w;
}

// The chunk `ahead` places past the cursor (ahead < kSlots: its copy was started when
// the chunk before the cursor was given back), after it has landed.
MB_DEV const uint8_t *peek(Ctx &c, const Cursor &cur, int ahead)
{
    const uint32_t k = cur.k + (uint32_t)ahead, slot = k % kSlots, use = k / kSlots;
    if (!mbar_wait(&c.S.full[slot], use & 1, c.sy, c.host_error)) return nullptr;
    return c.S.ring[slot];
}

// The issuing thread, after a consumer barrier: start the bulk copy of chunk k (if any)
// into slot k % kSlots, whose previous chunk every consumer has finished reading.
MB_DEV void issue(Ctx &c, uint32_t k, bool shared_issuers = false)
{
    if (k >= c.nchunks) return;
    const Chunk ch = c.S.desc[k];
    const uint32_t slot = k % kSlots;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(&c.S.full[slot], ch.bytes + (ch.gain_off ? kGainBytes : 0));
    bulk_load(c.S.ring[slot], c.stream + ch.off, ch.bytes, &c.S.full[slot], c.policy);
    if (ch.gain_off) bulk_load_plain(c.S.ring[slot] + kGainOff, c.blob + ch.gain_off, kGainBytes, &c.S.full[slot]);
    if (shared_issuers) {
        atomicMax(&c.S.issued, (int)k + 1);
        *(volatile int *)&c.S.slot_fill[slot] = (int)k;
    } else {
        c.S.issued = (int)k + 1;
    }
}

// Release the chunk at the cursor and refill its slot with the chunk kSlots ahead.
MB_DEV void give_back(Ctx &c, Cursor &cur)
{
    cbar();
    if (c.ct == kIssuer) issue(c, cur.k + kSlots);
    cur.k++;
}

// Error exit: wait (bounded) until every bulk copy started into this CTA's ring has
// landed, so no copy is still writing shared memory when the CTA exits.
MB_DEV void drain(Ctx &c, const Cursor &cur)
{
    if (c.ct == kIssuer) {  // the thread that recorded S.issued
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
            S.slot_done[s] = 0;
            S.slot_fill[s] = -1;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.token = ld_volatile((const unsigned *)&a.b.st->token);
        S.pos = ld_volatile((const unsigned *)&a.b.st->pos);
        S.issued = 0;
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
    for (uint32_t j = threadIdx.x; j < c_end - c0 && j < (uint32_t)kMaxChunksPerCta; j += kThreads)
        S.desc[j] = a.P->chunks[c0 + j];
    if (threadIdx.x < 2 * LAYERS) {
        const q8::Layer &ly = a.M->layer[threadIdx.x >> 1];
        S.gain[threadIdx.x & 1][threadIdx.x >> 1] = (threadIdx.x & 1) ? ly.ffn_norm : ly.attn_norm;
    }
    if (threadIdx.x == 2 * LAYERS) {
        S.ofrag = a.P->ofrag;
        S.oscale = a.P->oscale;
        S.final_gain = a.M->final_norm;
    }
    __syncthreads();
    Ctx c{S,
          a.sy,
          a.host_error,
          (int)threadIdx.x,
          (int)threadIdx.x >> 5,
          (int)threadIdx.x & 31,
          cta % kReplicas,
          a.P->stream,
          a.P->blob,
          c_end - c0,
          mb::evict_first_policy()};
    // the first kSlots chunks; every later one is started when a slot is given back
    if (c.ct == kIssuer)
        for (uint32_t k = 0; k < (uint32_t)kSlots; k++) issue(c, k);
    const int pos = S.pos;
    Cursor cur{0};
    int remaining = (int)(c_end - c0);  // chunks this CTA still has to take
    const Model *M = a.M;
    const Scratch &scr = a.scr;
    // the copies of the broadcast arrays this CTA reads
    const unsigned long long *kv_r = scr.kv + c.rep * kStrideKv;
    const int nks = has_spare(cta) ? 2 : 1;  // down-projection steps of this CTA
    // the down-projection accumulators of this step (set epoch & 1); this CTA clears its
    // share of the other set, which the next step uses (the last step that used it has
    // finished: it was the previous launch on this stream)
    const int set = (int)(epoch & 1u);
    unsigned long long *dacc = scr.dacc + (size_t)set * kAccRep * LAYERS * kAccCopyWords;
    unsigned long long *xacc = scr.xacc + (size_t)set * kAccRep * LAYERS * kAccCopyWords;
    {
        unsigned long long *od = scr.dacc + (size_t)(set ^ 1) * kAccRep * LAYERS * kAccCopyWords;
        unsigned long long *ox = scr.xacc + (size_t)(set ^ 1) * kAccRep * LAYERS * kAccCopyWords;
        const int lo = kAccRep * LAYERS * DIM * cta / kCTAs, hi = kAccRep * LAYERS * DIM * (cta + 1) / kCTAs;
        for (int i = lo + (int)threadIdx.x; i < hi; i += kThreads) {
            const size_t w = (size_t)(i / DIM) * kAccCopyWords + acc_word(i % DIM);  // (copy, row) -> word
            od[w] = 0ull;
            ox[w] = 0ull;
        }
    }
    // B-fragment columns 3..7 stay zero; columns 0..2 are rewritten by every quantize
    for (int i = c.ct; i < kSteps * 32; i += kNT) S.bf[i >> 5][i & 31] = make_uint2(0u, 0u);
    for (int i = c.ct; i < 2 * 32; i += kNT) {
        S.bfh[i >> 5][i & 31] = make_uint2(0u, 0u);
        S.hst[i >> 5][i & 31] = 0.f;  // columns 8..31 of the piece's step stay zero
    }
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

    // the RMSNorm gains are loaded a layer ahead and carried in registers (a load placed
    // next to its use would put two dependent L2 round trips on the critical path)
    float4 g_attn = load_gain(c.ct, S.gain[0][0]), g_ffn = load_gain(c.ct, S.gain[1][0]);
    for (int l = 0; l < LAYERS; l++) {
        // layer 0's past K/V for this CTA's attention split (every later layer's were
        // started by the idle threads of the previous layer's x_out reduction)
        if (l == 0 && unit.head >= 0) attn_prefetch(c, a, unit, 0, pos, 0, kNT);
        // ---- QKV + bias + RoPE + KV write
        stamp(a, cta, c.ct, 2 + l * kTraceLayer + 0);
        {
            // layer 0's norm here; every later layer's ran inside the previous layer's
            // x_out reduction, which also checked this QKV chunk
            if (l == 0) norm_quantize(&S, c.ct, g_attn, 0);
            g_attn = load_gain(c.ct, S.gain[0][min(l + 1, LAYERS - 1)]);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 12);
            const uint8_t *w = l == 0 ? take(c, cur, QKV) : S.ring[cur.k % kSlots];
            if (!w) return drain(c, cur);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 11);
            const ChunkHdr hd = *reinterpret_cast<const ChunkHdr *>(w);
            const int npair = hd.count;
            const uint8_t *frag = w + sizeof(ChunkHdr);
            const float *sc = reinterpret_cast<const float *>(frag + kHalfBytes);
            const float *bias = sc + 8 * kGroups;
            gemv_mma<1>(&S, c.cw, c.lane, Tiles{{frag, frag, frag}, {sc, sc, sc}, 1, 1});
            cbar();
            if (c.ct < npair) {
                stamp(a, cta, c.ct, 2 + l * kTraceLayer + 13);
                const int pair = hd.first + c.ct;
                const uint32_t tag = make_tag(epoch, l, PH_QKV);
                int kind, t;
                if (pair < DIM / 2) { kind = 0; t = pair; }
                else if (pair < DIM / 2 + KV / 2) { kind = 1; t = pair - DIM / 2; }
                else { kind = 2; t = pair - DIM / 2 - KV / 2; }
                const int head = t / 32, i = t % 32, r0 = head * HEAD_DIM + i;
                const float v0 = row_sum(c, 2 * c.ct) + bias[2 * c.ct];
                const float v1 = row_sum(c, 2 * c.ct + 1) + bias[2 * c.ct + 1];
                if (kind == 2) {
                    float *v = a.b.vc + kv_index(l, head, pos);
                    v[i] = v0;
                    v[i + 32] = v1;
                    dw_store_rep(scr.kv + (head * 2 + 1) * HEAD_DIM + i, kStrideKv, v0, tag);
                    dw_store_rep(scr.kv + (head * 2 + 1) * HEAD_DIM + i + 32, kStrideKv, v1, tag);
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
                        dw_store_rep(scr.kv + (head * 2) * HEAD_DIM + i, kStrideKv, lo, tag);
                        dw_store_rep(scr.kv + (head * 2) * HEAD_DIM + i + 32, kStrideKv, hi, tag);
                    }
                }
            }
            give_back(c, cur);
            remaining--;
        }
        stamp(a, cta, c.ct, 2 + l * kTraceLayer + 1);

        // ---- attention: one split of one query head per CTA
        if (unit.head >= 0) {
            const uint32_t tag = make_tag(epoch, l, PH_QKV);
            const int h = unit.head, kvh = h / GQA, np = unit.np;
            const bool has_cur = unit.p0 + np == pos + 1;
            const unsigned long long ready = (unsigned long long)tag << 32;
            // this warp's tiles of the head's O columns (both 32-column steps) and their
            // rows' scales, loaded now so the projection after the softmax waits for nothing
            const int ot0 = kDownTiles * c.cw / kConsumerWarps, otn = kDownTiles * (c.cw + 1) / kConsumerWarps - ot0;
            uint4 ofr[2][4];
            float osc[4][2];
            {
                const uint8_t *of = S.ofrag + (size_t)(l * HEADS + h) * kOHeadBytes;
                const float *os = S.oscale + (size_t)(l * HEADS + h) * DIM;
                const int g = c.lane >> 2;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int ti = min(ot0 + i, kDownTiles - 1);
#pragma unroll
                    for (int ks = 0; ks < 2; ks++)
                        ofr[ks][i] = __ldcg(reinterpret_cast<const uint4 *>(of + ks * kOStepBytes +
                                                                            ((size_t)ti * 32 + c.lane) * 16));
                    osc[i][0] = __ldcg(os + 16 * ti + g);
                    osc[i][1] = __ldcg(os + 16 * ti + g + 8);
                }
            }
            // the query of this head, and this position's K/V when the split holds it
            int ok = 1;
            if (c.ct < HEAD_DIM) {
                const unsigned long long *qa = scr.q + h * HEAD_DIM + c.ct;
                const unsigned long long *ka = kv_r + (kvh * 2) * HEAD_DIM + c.ct;
                const unsigned long long *va = kv_r + (kvh * 2 + 1) * HEAD_DIM + c.ct;
                unsigned long long w = dw_load(qa);
                unsigned long long wk = has_cur ? dw_load(ka) : ready;
                unsigned long long wv = has_cur ? dw_load(va) : ready;
                const long long t0 = clock64();
                while ((uint32_t)(w >> 32) != tag || (uint32_t)(wk >> 32) != tag || (uint32_t)(wv >> 32) != tag) {
                    if ((uint32_t)(w >> 32) != tag) w = dw_load(qa);
                    if ((uint32_t)(wk >> 32) != tag) wk = dw_load(ka);
                    if ((uint32_t)(wv >> 32) != tag) wv = dw_load(va);
                    if (give_up(c.sy, c.host_error, clock64() - t0, 1)) {
                        ok = 0;
                        break;
                    }
                }
                S.u.att.q[c.ct] = __uint_as_float((uint32_t)w);
                stamp(a, cta, c.ct, 2 + l * kTraceLayer + 14);
                if (has_cur) {
                    S.u.att.k[np - 1][c.ct] = __uint_as_float((uint32_t)wk);
                    S.u.att.v[np - 1][c.ct] = __uint_as_float((uint32_t)wv);
                }
            }
            cp_async_wait_all();
            if (!cbar_and(ok)) return drain(c, cur);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 15);
            // Online softmax per warp: warp cw owns positions 8 cw .. 8 cw + 7 (lane & 7
            // picks the position, lane >> 3 the quarter of the 64 dims of its score); it
            // keeps its own max, sum of weights and 64 accumulators, and 64 threads merge
            // the warp partials.  Key rows are kKStride floats apart so the eight lanes of
            // a phase hit distinct banks.
            const int nw = (np + 7) / 8;  // warps holding positions (np <= 128)
            if (c.cw < nw) {
                const int p = 8 * c.cw + (c.lane & 7), qd = c.lane >> 3;
                const bool valid = p < np;
                float z = 0.f;
                if (valid) {
                    const float4 *k4 = reinterpret_cast<const float4 *>(S.u.att.k[p]);
                    const float4 *q4 = reinterpret_cast<const float4 *>(S.u.att.q);
#pragma unroll
                    for (int m = 0; m < 4; m++) {
                        const float4 kk = k4[4 * m + qd], qq = q4[4 * m + qd];
                        z = fmaf(qq.x, kk.x, z);
                        z = fmaf(qq.y, kk.y, z);
                        z = fmaf(qq.z, kk.z, z);
                        z = fmaf(qq.w, kk.w, z);
                    }
                }
                z += __shfl_xor_sync(0xffffffffu, z, 8);
                z += __shfl_xor_sync(0xffffffffu, z, 16);
                const float sc = valid ? z * 0.125f : -INFINITY;
                const float m = mb::warp_max(sc);
                // the hardware exponential (__expf: within 2 + 1.2|x| ulp by CUDA's own
                // bound, arguments <= 0 here) for every softmax weight, merge factor and
                // split weight: the full-precision expf put about 150 more cycles on each
                // of these chains; the weights are normalised by their own sums
                const float e = valid ? __expf(sc - m) : 0.f;
                // the warp's sum of weights comes with the P.V shuffles (every lane sees
                // the 8 weights in order)
                float lw = 0.f, a0 = 0.f, a1 = 0.f;
                const float *vb = S.u.att.v[8 * c.cw];
                // rows past np read the next rows of the buffer (or, for row 8 * 12 + 7 =
                // kAttnLenMax, the query after it) and enter as zeros: no branch around
                // the loads
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float ej = __shfl_sync(0xffffffffu, e, j);  // lane j holds position 8 cw + j
                    lw += ej;
                    const bool in = 8 * c.cw + j < np;
                    const float x0 = vb[j * HEAD_DIM + c.lane], x1 = vb[j * HEAD_DIM + 32 + c.lane];
                    a0 = fmaf(ej, in ? x0 : 0.f, a0);
                    a1 = fmaf(ej, in ? x1 : 0.f, a1);
                }
                float *wp = S.u.att.wp[c.cw];
                wp[4 + c.lane] = a0;
                wp[4 + 32 + c.lane] = a1;
                if (c.lane == 0) {
                    wp[0] = m;
                    wp[1] = lw;
                }
            }
            cbar();
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 16);
            // Warp 0 merges the warps' partials at the split's max and quantizes the
            // result straight into S.bfo: lane t (t = lane % 16; both halves compute the
            // same) owns dims 32 ks + 16 hh + 4 tig + {0..3}, ks = t >> 3, tig = (t >> 1) & 3,
            // hh = t & 1 -- its limbs' place in the B fragments, as in put_limbs.
            // Lane w < nw holds warp w's max and its factor exp(m_w - max) (one expf per
            // lane); the sums run over w in order with the factors shuffled in, and rows
            // of idle warps enter as zeros (no branch around the loads).
            if (c.cw == 0) {
                const float mw = c.lane < nw ? S.u.att.wp[c.lane][0] : -INFINITY;
                const float mx = mb::warp_max(mw);
                const float fw = c.lane < nw ? __expf(mw - mx) : 0.f;
                const int t = c.lane & 15, ks = t >> 3, tig = (t >> 1) & 3, hh = t & 1;
                const int d0 = 32 * ks + 16 * hh + 4 * tig;
                // lanes 0..15 sum warps [0, kHalf), lanes 16..31 warps [kHalf, 2 kHalf); the
                // halves are then added (both lanes of a pair get the same sum)
                constexpr int kHalf = (kMaxAttnWarps + 1) / 2;
                float lsum = 0.f;
                float o[4] = {0.f, 0.f, 0.f, 0.f};
                const int wb = (c.lane >> 4) * kHalf;
#pragma unroll
                for (int i = 0; i < kHalf; i++) {
                    const int w = wb + i;
                    const float f = __shfl_sync(0xffffffffu, fw, w);
                    const bool in = w < nw;
                    const float lw = S.u.att.wp[min(w, kConsumerWarps - 1)][1];
                    const float4 p = *reinterpret_cast<const float4 *>(&S.u.att.wp[min(w, kConsumerWarps - 1)][4 + d0]);
                    lsum = fmaf(f, in ? lw : 0.f, lsum);
                    o[0] = fmaf(f, in ? p.x : 0.f, o[0]);
                    o[1] = fmaf(f, in ? p.y : 0.f, o[1]);
                    o[2] = fmaf(f, in ? p.z : 0.f, o[2]);
                    o[3] = fmaf(f, in ? p.w : 0.f, o[3]);
                }
                lsum += __shfl_xor_sync(0xffffffffu, lsum, 16);
#pragma unroll
                for (int j = 0; j < 4; j++) o[j] += __shfl_xor_sync(0xffffffffu, o[j], 16);
                if (c.lane == 0) {
                    S.att_m = mx;
                    S.att_l = lsum;
                    if (splits > 1) {  // for the other splits of this head
                        const uint32_t ptag = make_tag(epoch, l, PH_ATTN);
                        unsigned long long *ml = scr.part + 2 * ((size_t)h * kMaxSplit + unit.split);
                        dw_store(ml, mx, ptag);
                        dw_store(ml + 1, lsum, ptag);
                    }
                }
                const float m = mb::warp_max(fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3]))));
                const float inv = m > 0.f ? __fdividef(127.f, m) : 0.f;
                const float q[4] = {o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv};
                uint32_t p0, p1, p2;
                limbs4(q, p0, p1, p2);
                if (c.lane < 16) {
                    uint32_t *b = reinterpret_cast<uint32_t *>(&S.bfo[ks][0]);
                    b[2 * tig + hh] = p0;
                    b[2 * (4 + tig) + hh] = p1;
                    b[2 * (8 + tig) + hh] = p2;
                }
                if (c.lane == 0) S.so = m * (1.0f / (127.f * 254.f));
            }
            cbar();
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 3);
            // warp 0 starts reading the splits' (max, sum) before the products
            const uint32_t ptag = make_tag(epoch, l, PH_ATTN);
            const unsigned long long *ml = scr.part + 2 * ((size_t)h * kMaxSplit + min(c.lane, splits - 1));
            unsigned long long w0 = 0, w1 = 0;
            if (c.cw == 0 && splits > 1) {
                w0 = dw_load(ml);
                w1 = dw_load(ml + 1);
            }
            // the unnormalised output through O's 64 columns of this head: P = O_h acc
            // (a warp with three tiles also multiplies a copy of its last; unused)
            float pacc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
            const uint2 bo[2] = {S.bfo[0][c.lane], S.bfo[1][c.lane]};
            {
                // The head's 64 columns are one scale group of O's rows and one
                // quantization of the output: both 32-column steps add into one int32 sum
                // per tile (|D| <= 2 * 32 * 128 * 127), combined once.  Every tile's first
                // MMA, then every second one, then the combines (as in gemv_mma).
                int d[4][4];
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        if (ks == 0) {
#pragma unroll
                            for (int j = 0; j < 4; j++) d[i][j] = 0;
                        }
                        mma_s8(d[i], ofr[ks][i], bo[ks]);
                    }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    float v0, v1;
                    combine(d[i], v0, v1);
                    pacc[i][0] = v0 * osc[i][0];
                    pacc[i][1] = v1 * osc[i][1];
                }
            }
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 4);
            // this split's weight in the head's softmax: exp(m - M) / L over the splits
            if (c.cw == 0) {
                float wgt = 0.f;
                if (splits == 1) {
                    wgt = 1.0f / S.att_l;
                } else {
                    if (c.lane < splits && ((uint32_t)(w0 >> 32) != ptag || (uint32_t)(w1 >> 32) != ptag)) {
                        const long long t0 = clock64();
                        while ((uint32_t)(w0 >> 32) != ptag || (uint32_t)(w1 >> 32) != ptag) {
                            if ((uint32_t)(w0 >> 32) != ptag) w0 = dw_load(ml);
                            if ((uint32_t)(w1 >> 32) != ptag) w1 = dw_load(ml + 1);
                            if (give_up(c.sy, c.host_error, clock64() - t0, 1)) {
                                ok = 0;
                                break;
                            }
                        }
                    }
                    const float m = c.lane < splits ? __uint_as_float((uint32_t)w0) : -INFINITY;
                    const float lv = c.lane < splits ? __uint_as_float((uint32_t)w1) : 0.f;
                    const float M = mb::warp_max(m);
                    const float L = mb::warp_sum(c.lane < splits ? __expf(m - M) * lv : 0.f);
                    wgt = __fdividef(__expf(S.att_m - M), L);
                }
                if (c.lane == 0) S.att_w = wgt;
            }
            if (!cbar_and(ok)) return drain(c, cur);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 23);
            {
                const float f = S.so * S.att_w;
                const int g = c.lane >> 2;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (i < otn && (c.lane & 3) == 0) {
                        const int r0 = 16 * (ot0 + i) + g, r1 = r0 + 8;
                        fix_add(xacc + (size_t)(kAccRep * l + cta % kAccRep) * kAccCopyWords + acc_word(r0), pacc[i][0] * f);
                        fix_add(xacc + (size_t)(kAccRep * l + cta % kAccRep) * kAccCopyWords + acc_word(r1), pacc[i][1] * f);
                    }
                }
            }
            cbar();
        }
        stamp(a, cta, c.ct, 2 + l * kTraceLayer + 2);

        // ---- x_mid = x_in + the attention block, all-reduced over the attention CTAs
        // (with the FFN norm's first half, and the issuer checking the FFN chunks)
        const int ngu = has_spare(cta) ? 3 : 2, T = has_spare(cta) ? 5 : 4;  // gate/up chunks, tiles
        {
            float4 x;
            float pm;
            if (!add_sums_norm(c, xacc + (size_t)kAccRep * l * kAccCopyWords, (unsigned)(HEADS * splits), g_ffn, x, pm,
                               [&]() { return ffn_ready(c, cur, remaining, l, ngu); }, []() {}))
                return drain(c, cur);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 5);
            norm_finish(S, c.ct, g_ffn, x, pm, 0);
        }

        // ---- RMSNorm -> gate/up -> SwiGLU
        {
            // (after the last layer: the final norm's gain, for the head)
            g_ffn = load_gain(c.ct, l + 1 < LAYERS ? S.gain[1][l + 1] : S.final_gain);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 10);
            // this layer's gate/up chunks, resident together in slots cur.k .. cur.k + ngu - 1,
            // and the first down chunk after them: checked during the x_mid reduction
            const uint32_t s0 = cur.k % kSlots, s1 = (cur.k + 1) % kSlots, s2 = (cur.k + (ngu > 2 ? 2 : 0)) % kSlots;
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 9);
            Tiles tl{{S.ring[s0] + sizeof(ChunkHdr), S.ring[s1] + sizeof(ChunkHdr), S.ring[s2] + sizeof(ChunkHdr)},
                     {nullptr, nullptr, nullptr},
                     T,
                     0};
            // chunk i holds tiles 2i, 2i + 1 (the last chunk may hold one)
            tl.sc[0] = reinterpret_cast<const float *>(tl.frag[0] + (size_t)min(2, T) * kTileBytes);
            tl.sc[1] = reinterpret_cast<const float *>(tl.frag[1] + (size_t)max(1, min(2, T - 2)) * kTileBytes);
            tl.sc[2] = reinterpret_cast<const float *>(tl.frag[2] + (size_t)max(1, min(2, T - 4)) * kTileBytes);
            if (T > 4)
                gemv_mma<5>(&S, c.cw, c.lane, tl);
            else
                gemv_mma<4>(&S, c.cw, c.lane, tl);
            cbar();
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 18);
            // the products are in S.gp: the block's gate/up chunks go back at once; a
            // piece's chunk stays at the cursor until its down columns have been used
            if (c.ct == kIssuer)
                for (int i = 0; i < 2; i++) issue(c, cur.k + i + kSlots);
            cur.k += 2;
            remaining -= 2;
            // h = silu(gate) * up, each down step's 32 columns in one warp, quantized there
            // with the step's own scale (no block barrier between SwiGLU and limbs): warp 0
            // the CTA's block, unit 32 cta + lane at column lane (tile lane / 8 holds its
            // gate row 16 t + lane % 8 and its up row 8 below); warp 1, for a CTA with a
            // piece, the piece's 8 units from tile 4 at columns 0..7 of its step
            if (c.cw < nks) {
                const int t = c.cw == 0 ? c.lane >> 3 : 4, j = c.lane & 7;
                const bool live = c.cw == 0 || c.lane < 8;
                const int col = c.cw == 0 ? c.lane : j;
                float hv = 0.f;
                if (live) {
                    const float g = row_sum(c, 16 * t + j), u = row_sum(c, 16 * t + 8 + j);
                    hv = __fdividef(g, 1.0f + expf(-g)) * u;
                    S.hst[c.cw][col] = hv;
                }
                __syncwarp();
                const float m = mb::warp_max(fabsf(hv));
                if (c.lane < 8) {  // columns 16 h + 4 tig + {0..3}: B-fragment register h of lanes 4 n + tig
                    const int tig = c.lane >> 1, h = c.lane & 1;
                    const float4 v = *reinterpret_cast<const float4 *>(&S.hst[c.cw][16 * h + 4 * tig]);
                    const float inv = m > 0.f ? __fdividef(127.f, m) : 0.f;
                    const float q[4] = {v.x * inv, v.y * inv, v.z * inv, v.w * inv};
                    uint32_t p0, p1, p2;
                    limbs4(q, p0, p1, p2);
                    uint32_t *b = reinterpret_cast<uint32_t *>(&S.bfh[c.cw][0]);
                    b[2 * tig + h] = p0;
                    b[2 * (4 + tig) + h] = p1;
                    b[2 * (8 + tig) + h] = p2;
                }
                if (c.lane == 0) S.sh[c.cw] = m * (1.0f / (127.f * 254.f));
            }
            cbar();
        }
        stamp(a, cta, c.ct, 2 + l * kTraceLayer + 7);
        stamp(a, cta, c.ct, 2 + l * kTraceLayer + 19);
        {
            // the block's down step (checked with the gate/up chunks; after a kept piece
            // chunk), then the piece's 8 columns from that chunk
            const int keep = nks - 1;
            float pacc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
            const uint8_t *frag = S.ring[(cur.k + keep) % kSlots] + sizeof(ChunkHdr);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 20);
            const float *sw = reinterpret_cast<const float *>(frag + (size_t)kDownTiles * 512);
            const uint8_t *pf = S.ring[cur.k % kSlots] + sizeof(ChunkHdr) + kSpareDownOff;
            const float *psw = reinterpret_cast<const float *>(pf + kSpareDownBytes);
            if (keep)
                down_steps<true>(c, frag, sw, S.bfh[0], S.sh[0], pf, psw, S.bfh[1], S.sh[1], pacc);
            else
                down_steps<false>(c, frag, sw, S.bfh[0], S.sh[0], pf, psw, S.bfh[1], S.sh[1], pacc);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 21);
            // rows 16 t + g and 16 t + g + 8 of the warp's tiles: this CTA's partial
            {
                const int t0 = kDownTiles * c.cw / kConsumerWarps;
                const int n = kDownTiles * (c.cw + 1) / kConsumerWarps - t0;
                const int g = c.lane >> 2;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (i < n && (c.lane & 3) == 0) {
                        const int r0 = 16 * (t0 + i) + g, r1 = r0 + 8;
                        fix_add(dacc + (size_t)(kAccRep * l + cta % kAccRep) * kAccCopyWords + acc_word(r0), pacc[i][0]);
                        fix_add(dacc + (size_t)(kAccRep * l + cta % kAccRep) * kAccCopyWords + acc_word(r1), pacc[i][1]);
                    }
                }
            }
            cbar();
            if (c.ct == kIssuer)
                for (int i = 0; i <= keep; i++) issue(c, cur.k + i + kSlots);
            cur.k += 1 + keep;
            remaining -= 1 + keep;
        }
        stamp(a, cta, c.ct, 2 + l * kTraceLayer + 6);
        // all-reduce: once all 148 CTAs' additions are complete every CTA adds the sums
        // to its x_mid -- the next layer's input -- fused with that layer's QKV norm (first
        // half) while the issuer checks its QKV chunk
        if (l + 1 < LAYERS) {
            float4 x;
            float pm;
            if (!add_sums_norm(c, dacc + (size_t)kAccRep * l * kAccCopyWords, kCTAs, g_attn, x, pm,
                               [&]() { return qkv_ready(c, cur, remaining, l + 1); },
                               [&]() {
                                   if (unit.head >= 0) attn_prefetch(c, a, unit, l + 1, pos, DIM / 4, kNT - DIM / 4);
                               }))
                return drain(c, cur);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 8);
            norm_finish(S, c.ct, g_attn, x, pm, 0);
        } else {
            if (!add_sums(c, dacc + (size_t)kAccRep * l * kAccCopyWords, kCTAs)) return drain(c, cur);
            stamp(a, cta, c.ct, 2 + l * kTraceLayer + 8);
        }
    }

    if (project) {
        // ---- final norm + tied head, logits kept in shared memory for selection
        stamp(a, cta, c.ct, kTraceHead);
        const int lo = a.P->head_lo[cta], n = a.P->head_lo[cta + 1] - lo;
        // the rest of this CTA's stream is its head chunks: 32 vocabulary rows (two
        // tiles) each, the last one shorter
        const int nhc = remaining;
        if (nhc <= 0 || !peek(c, cur, 0)) {
            if (c.ct == 0) fail(c.sy, c.host_error, 4);
            return drain(c, cur);
        }
        if (c.ct == 0)
            for (int i = 0; i < kSlots; i++) S.slot_fill[(cur.k + i) % kSlots] = (int)(cur.k + i);
        norm_quantize(&S, c.ct, g_ffn, cta == 0);
        if (cta == 0)
            for (int i = c.ct; i < DIM; i += kNT) a.b.hidden[i] = S.ns[i];
        // Warp w takes tiles w, w + 16, ... in order (tile t = tile t & 1 of chunk t >> 1),
        // each over all 896 columns, so its lanes hold complete row sums; the warp that
        // finishes the last tile of a chunk starts the copy of the chunk kSlots ahead
        // into its slot.  A chunk's copy waits only for tiles earlier in every warp's
        // order, so the warps never wait on each other in a cycle.  A warp's next chunk
        // is 2 * kSlots chunks on, two fills of the same slot later, and a parity wait is
        // only exact once the chunk's own copy has been issued (the fill before it then
        // has landed and been read): the warp first waits for that on slot_fill.
        int ok = 1;
        {
            const int g = c.lane >> 2, tig = c.lane & 3;
            for (int t = c.cw; t < 2 * nhc; t += kConsumerWarps) {
                const uint32_t k = cur.k + (uint32_t)(t >> 1), slot = k % kSlots;
                if (*(volatile int *)&S.slot_fill[slot] < (int)k) {
                    const long long t0 = clock64();
                    while (*(volatile int *)&S.slot_fill[slot] < (int)k) {
                        if (give_up(c.sy, c.host_error, clock64() - t0, 2)) {
                            ok = 0;
                            break;
                        }
                    }
                    if (!ok) break;
                }
                if (!mbar_wait(&S.full[slot], (k / kSlots) & 1, c.sy, c.host_error)) {
                    ok = 0;
                    break;
                }
                const uint8_t *w = S.ring[slot];
                const ChunkHdr *hd = reinterpret_cast<const ChunkHdr *>(w);
                const int rows = (int)hd->count;
                if (hd->kind != HEAD || rows < 1 || rows > kHeadPerChunk) {
                    if (c.lane == 0) fail(c.sy, c.host_error, 4);
                    ok = 0;
                    break;
                }
                const bool half = rows <= 8;
                const int tin = half ? 1 : (rows + 15) / 16, ti = t & 1;
                if (ti < tin) {
                    const uint8_t *frag = w + sizeof(ChunkHdr);
                    const float *sc = reinterpret_cast<const float *>(frag + (half ? kHalfBytes : tin * kTileBytes)) +
                                      ti * 16 * kGroups;
                    frag += ti * kTileBytes;
                    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 2
                    for (int grp = 0; grp < kGroups; grp++) {
                        int d[4] = {0, 0, 0, 0};
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int ks = 2 * grp + h;
                            uint4 av;
                            if (half) {
                                const uint2 v = *reinterpret_cast<const uint2 *>(frag + ((size_t)ks * 32 + c.lane) * 8);
                                av = make_uint4(v.x, 0u, v.y, 0u);
                            } else {
                                av = *reinterpret_cast<const uint4 *>(frag + ((size_t)ks * 32 + c.lane) * 16);
                            }
                            mma_s8(d, av, S.bf[ks][c.lane]);
                        }
                        float v0, v1;
                        combine(d, v0, v1);
                        const float f = S.sxs[grp];
                        acc0 = fmaf(v0, sc[g * kGroups + grp] * f, acc0);
                        if (!half) acc1 = fmaf(v1, sc[(g + 8) * kGroups + grp] * f, acc1);
                    }
                    if (tig == 0) {
                        const int r0 = 16 * ti + g, r1 = r0 + 8;
                        if (r0 < rows) {
                            a.b.logits[hd->first + r0] = acc0;
                            S.u.hl[hd->first + r0 - lo] = acc0;
                        }
                        if (!half && r1 < rows) {
                            a.b.logits[hd->first + r1] = acc1;
                            S.u.hl[hd->first + r1 - lo] = acc1;
                        }
                    }
                    __syncwarp();
                    if (c.lane == 0) {
                        __threadfence_block();
                        if (atomicAdd(&S.slot_done[slot], 1) + 1 == tin) {
                            S.slot_done[slot] = 0;
                            issue(c, k + kSlots, true);
                        }
                    }
                }
            }
        }
        if (!cbar_and(ok)) return drain(c, cur);
        cur.k += nhc;
        remaining = 0;
        cbar();
        if (decode) {
            // penalty (distinct ids of the history window) and control mask on this
            // CTA's vocabulary slice, then the slice's top k as ordered keys
            const sampling::Params prm = *a.prm;
            if (c.cw == 0) {
                const int count = min(max(a.seq->history_count, 0), sampling::kHistory);
                for (int j = c.lane; j < count; j += 32) {
                    const int id = a.seq->history[j];
                    if (id < lo || id >= lo + n) continue;  // not in this slice: no duplicate scan
                    bool dup = false;
                    for (int t = 0; t < j; t++) dup |= a.seq->history[t] == id;
                    if (!dup) {
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
    stamp(a, cta, c.ct, kTraceHead + 1);
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
    stamp(a, cta, c.ct, kTraceHead + 2);
    if (c.ct == 0) {
        a.b.st->steps++;
        a.sy->done = 0;
        // wraps to 2: the accumulator set (epoch & 1) keeps alternating
        const unsigned next = epoch + 1 >= (1u << 24) ? 2u : epoch + 1;
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

size_t scratch_words()
{
    return (size_t)DIM + (size_t)kReplicas * kStrideKv + kPartWords + 4 * (size_t)kAccRep * LAYERS * kAccCopyWords;
}

void carve_scratch(unsigned long long *base, Scratch *scr)
{
    scr->q = base;
    scr->kv = scr->q + DIM;
    scr->part = scr->kv + kReplicas * kStrideKv;
    scr->dacc = scr->part + kPartWords;
    scr->xacc = scr->dacc + 2 * (size_t)kAccRep * LAYERS * kAccCopyWords;

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

// One 32-column step of a 16-row tile in the A-fragment order of
// mma.m16n8k32.row (lane l = 4 g + tig: rows g and g + 8, columns 4 tig + {0..3} and
// 16 + 4 tig + {0..3}); a null row is zero.  Half tiles keep registers a0 and a2 only.
static void put_step(std::vector<uint8_t> &out, const int8_t *const rows[16], int k0, bool half)
{
    for (int l = 0; l < 32; l++) {
        const int g = l >> 2, tig = l & 3;
        const int8_t *r0 = rows[g], *r1 = rows[g + 8];
        uint8_t b[16];
        for (int j = 0; j < 4; j++) {
            b[j] = r0 ? (uint8_t)r0[k0 + 4 * tig + j] : 0;
            b[4 + j] = r1 ? (uint8_t)r1[k0 + 4 * tig + j] : 0;
            b[8 + j] = r0 ? (uint8_t)r0[k0 + 16 + 4 * tig + j] : 0;
            b[12 + j] = r1 ? (uint8_t)r1[k0 + 16 + 4 * tig + j] : 0;
        }
        if (half) {
            out.insert(out.end(), b, b + 4);
            out.insert(out.end(), b + 8, b + 12);
        } else {
            out.insert(out.end(), b, b + 16);
        }
    }
}

int build_plan(const FileHeader *hdr, const unsigned char *hfile, const unsigned char *dfile, Plan *hplan,
               Chunk **dchunks, uint8_t **dstream, size_t *stream_bytes, cudaStream_t s)
{
    std::vector<Chunk> chunks;
    std::vector<uint8_t> stream;
    stream.reserve((size_t)580 << 20);
    const FileTensor *t = hdr->t;
    auto align16 = [](size_t v) { return (v + 15) & ~(size_t)15; };
    using Row = std::pair<const FileTensor *, int>;  // (matrix, row); null matrix = zero row
    auto row_ptr = [&](const Row &r) -> const int8_t * {
        return r.first ? reinterpret_cast<const int8_t *>(hfile + r.first->data) + (size_t)r.second * r.first->cols
                       : nullptr;
    };
    auto scale = [&](const Row &r, int group) -> float {
        if (!r.first) return 0.f;
        const float *sc = reinterpret_cast<const float *>(hfile + r.first->scales);
        return sc[(size_t)r.second * (r.first->cols / GROUP) + group];
    };
    auto begin = [&](uint32_t kind, uint32_t layer, uint32_t first, uint32_t count) {
        Chunk ch{};
        ch.off = stream.size();
        const ChunkHdr hd{kind, layer, first, count};
        const uint8_t *hb = reinterpret_cast<const uint8_t *>(&hd);
        stream.insert(stream.end(), hb, hb + sizeof hd);
        return ch;
    };
    auto put_floats = [&](const std::vector<float> &v) {
        const uint8_t *b = reinterpret_cast<const uint8_t *>(v.data());
        stream.insert(stream.end(), b, b + v.size() * 4);
    };
    auto finish = [&](Chunk ch, uint32_t gain_off) {
        stream.resize(align16(stream.size()), 0);
        ch.bytes = (uint32_t)(stream.size() - ch.off);
        ch.gain_off = gain_off;
        const uint32_t limit = gain_off ? (uint32_t)kGainOff : (uint32_t)kSlotBytes;
        if (ch.bytes > limit || (gain_off && gain_off % 16)) return false;
        chunks.push_back(ch);
        return true;
    };
    // A chunk of 896-wide rows: tiles of 16 rows (tile_rows.size() a multiple of 16, or 8
    // for a half tile), then the tile rows' 14 scales each, then extra bytes and floats.
    auto emit896 = [&](uint32_t kind, uint32_t layer, uint32_t first, uint32_t count,
                       const std::vector<Row> &tile_rows, const std::vector<uint8_t> &extra_bytes,
                       const std::vector<float> &extra, uint32_t gain_off) {
        const bool half = tile_rows.size() == 8;
        if (!half && tile_rows.size() % 16) return false;
        Chunk ch = begin(kind, layer, first, count);
        const int T = half ? 1 : (int)tile_rows.size() / 16;
        for (int ti = 0; ti < T; ti++) {
            const int8_t *rows[16];
            for (int j = 0; j < 16; j++) rows[j] = half && j >= 8 ? nullptr : row_ptr(tile_rows[16 * ti + j]);
            for (int ks = 0; ks < kSteps; ks++) put_step(stream, rows, 32 * ks, half);
        }
        std::vector<float> sc;
        for (const Row &r : tile_rows)
            for (int g = 0; g < kGroups; g++) sc.push_back(scale(r, g));
        put_floats(sc);
        stream.insert(stream.end(), extra_bytes.begin(), extra_bytes.end());
        put_floats(extra);
        return finish(ch, gain_off);
    };
    const Row none{nullptr, 0};
    for (int c = 0; c < kCTAs; c++) {
        hplan->chunk_begin[c] = (uint32_t)chunks.size();
        for (int l = 0; l < LAYERS; l++) {
            const FileTensor *lt = t + 1 + l * STRIDE;
            int lo, hi;
            // QKV: pair p -> tile rows 2j (dimension i) and 2j + 1 (dimension i + 32)
            std::vector<Row> rows(8, none);
            std::vector<float> bias(8, 0.f);
            split(kQkvPairs, kCTAs, c, lo, hi);
            if (hi - lo > 4) return 1;
            for (int p = lo; p < hi; p++) {
                const FileTensor *m, *b;
                int tt;
                if (p < DIM / 2) { m = &lt[WQ]; b = &lt[BQ]; tt = p; }
                else if (p < DIM / 2 + KV / 2) { m = &lt[WK]; b = &lt[BK]; tt = p - DIM / 2; }
                else { m = &lt[WV]; b = &lt[BV]; tt = p - DIM / 2 - KV / 2; }
                const int r0 = (tt / 32) * HEAD_DIM + tt % 32, j = p - lo;
                rows[2 * j] = {m, r0};
                rows[2 * j + 1] = {m, r0 + 32};
                const float *bv = reinterpret_cast<const float *>(hfile + b->data);
                bias[2 * j] = bv[r0];
                bias[2 * j + 1] = bv[r0 + 32];
            }
            if (!emit896(QKV, l, lo, hi - lo, rows, {}, bias, lt[ATTN_NORM].data)) return 1;
            // gate/up: tiles of 8 gate rows then the 8 up rows of the same hidden units;
            // the CTA's block in two chunks, then its spare piece (one tile, followed by
            // the piece's 8 down-projection columns and their scales)
            const FileTensor *wd = &lt[WDOWN];
            const int8_t *dw = reinterpret_cast<const int8_t *>(hfile + wd->data);
            std::vector<std::pair<int, int>> pieces = {{32 * c, 16}, {32 * c + 16, 16}};
            if (has_spare(c)) pieces.push_back({spare_lo(c), 8});
            for (size_t i = 0; i < pieces.size(); i++) {
                const int h0 = pieces[i].first, n = pieces[i].second;
                rows.clear();
                for (int ti = 0; ti < n / 8; ti++) {
                    for (int j = 0; j < 8; j++) rows.push_back({&lt[WGATE], h0 + 8 * ti + j});
                    for (int j = 0; j < 8; j++) rows.push_back({&lt[WUP], h0 + 8 * ti + j});
                }
                std::vector<uint8_t> pb;
                std::vector<float> psc;
                if (i == 2) {
                    // entry e = 2 g + tig (tig < 2) of tile ti: rows 16 ti + g and 16 ti + g + 8,
                    // columns h0 + 4 tig .. h0 + 4 tig + 3 (registers a0, a1)
                    for (int ti = 0; ti < kDownTiles; ti++)
                        for (int e = 0; e < 16; e++) {
                            const int g = e >> 1, tig = e & 1;
                            for (int rr = 0; rr < 2; rr++)
                                for (int j = 0; j < 4; j++)
                                    pb.push_back((uint8_t)dw[(size_t)(16 * ti + g + 8 * rr) * HIDDEN + h0 + 4 * tig + j]);
                        }
                    for (int r = 0; r < DIM; r++) psc.push_back(scale({wd, r}, h0 / GROUP));
                    if (pb.size() != (size_t)kSpareDownBytes) return 1;
                }
                if (!emit896(GATEUP, l, h0, n, rows, pb, psc, i == 0 ? lt[FFN_NORM].data : 0)) return 1;
            }
            // down: the 32 columns of the CTA's block (one scale group)
            {
                const int k0 = 32 * c;
                std::vector<float> dsc(DIM);
                for (int r = 0; r < DIM; r++) dsc[r] = scale({wd, r}, k0 / GROUP);
                Chunk ch = begin(DOWN, l, 0, 1);
                for (int ti = 0; ti < kDownTiles; ti++) {
                    const int8_t *rr[16];
                    for (int j = 0; j < 16; j++) rr[j] = dw + (size_t)(16 * ti + j) * HIDDEN;
                    put_step(stream, rr, k0, false);
                }
                put_floats(dsc);
                if (!finish(ch, 0)) return 1;
            }
        }
        int lo, hi;
        split(VOCAB, kCTAs, c, lo, hi);
        hplan->head_lo[c] = lo;
        hplan->head_begin[c] = (uint32_t)chunks.size();
        if (hi - lo > kHeadSlice) return 1;
        for (int r0 = lo; r0 < hi; r0 += kHeadPerChunk) {
            const int r1 = r0 + kHeadPerChunk < hi ? r0 + kHeadPerChunk : hi;
            const int n = r1 - r0, padded = n <= 8 ? 8 : (n + 15) / 16 * 16;
            std::vector<Row> rows(padded, none);
            for (int r = r0; r < r1; r++) rows[r - r0] = {&t[0], r};
            if (!emit896(HEAD, LAYERS, r0, n, rows, {}, {}, r0 == lo ? t[TENSORS - 1].data : 0)) return 1;
        }
    }
    // O by head, read by the attention CTAs (not streamed per CTA): for layer l and head
    // h, the two 32-column steps of columns [64 h, 64 h + 64) over all 896 rows in the
    // down projection's tile order, then the rows' scales of that 64-column group
    stream.resize((stream.size() + 255) & ~(size_t)255, 0);
    const size_t o_frag_off = stream.size();
    for (int l = 0; l < LAYERS; l++) {
        const FileTensor *wo = &t[1 + l * STRIDE + WO];
        const int8_t *ow = reinterpret_cast<const int8_t *>(hfile + wo->data);
        for (int h = 0; h < HEADS; h++)
            for (int ks = 0; ks < 2; ks++)
                for (int ti = 0; ti < kDownTiles; ti++) {
                    const int8_t *rr[16];
                    for (int j = 0; j < 16; j++) rr[j] = ow + (size_t)(16 * ti + j) * DIM;
                    put_step(stream, rr, HEAD_DIM * h + 32 * ks, false);
                }
    }
    const size_t o_scale_off = stream.size();
    for (int l = 0; l < LAYERS; l++) {
        const FileTensor *wo = &t[1 + l * STRIDE + WO];
        std::vector<float> osc;
        for (int h = 0; h < HEADS; h++)
            for (int r = 0; r < DIM; r++) osc.push_back(scale({wo, r}, h));
        put_floats(osc);
    }
    if (o_scale_off - o_frag_off != (size_t)LAYERS * HEADS * kOHeadBytes) return 1;
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
    hplan->ofrag = *dstream + o_frag_off;
    hplan->oscale = reinterpret_cast<const float *>(*dstream + o_scale_off);
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
