// Persistent batch-1 decode kernel for the grouped-Q8 model: one cooperative launch
// per token over all 148 SMs.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q8_decode.cuh"
#include "sampling.cuh"

namespace q8p {

constexpr int kCTAs = 148;                // one CTA per SM
constexpr int kConsumerWarps = 16;
constexpr int kThreads = 32 * kConsumerWarps;  // every thread consumes; one also issues the weight copies
constexpr int kSlots = 4;                 // shared-memory ring slots
constexpr int kSlotBytes = 36864;
constexpr int kGainBytes = q8::DIM * 4;   // RMSNorm gain delivered with some chunks
constexpr int kGainOff = kSlotBytes - kGainBytes;
constexpr int kMaxSplit = 10;             // attention splits per query head
constexpr int kAttnTarget = 64;           // positions per split when possible
constexpr int kAttnLenMax = (q8::CONTEXT + kMaxSplit - 1) / kMaxSplit;  // 103

enum Kind : uint32_t { QKV = 0, OPROJ = 1, GATEUP = 2, DOWN = 3, HEAD = 4 };
enum Mode { FORWARD = 0, FORWARD_PROJECT = 1, PREFILL = 2, DECODE = 3 };

// Where the producer finds a chunk of the weight stream.  The chunk itself starts
// with a 16-byte ChunkHdr, so the consumers never read descriptors from global memory.
struct Chunk {
    uint64_t off;       // byte offset in the stream buffer
    uint32_t bytes;     // multiple of 16, header included
    uint32_t gain_off;  // nonzero: byte offset in the model blob of a DIM-float gain
};

struct ChunkHdr {
    uint32_t kind, layer, first, count;  // rows or row pairs [first, first+count)
};

struct Plan {
    const uint8_t *stream;                 // all CTAs' streams back to back
    const Chunk *chunks;                   // all chunks, CTA-major
    const uint8_t *blob;                   // the uploaded model file (gains)
    const uint8_t *ofrag;                  // O by head: [layer][head][2 steps][56 tiles][32 lanes][16 B]
    const float *oscale;                   // [layer][head][896] O scales of the head's 64-column group
    uint32_t chunk_begin[kCTAs + 1];
    uint32_t head_begin[kCTAs];            // first head chunk of each CTA (head chunks are last)
    uint32_t head_lo[kCTAs + 1];           // contiguous vocabulary rows per CTA
};

constexpr int kMaxChunksPerCta = 184;  // >= 24 layers x 6 + 33 head chunks

struct Sync {
    unsigned epoch;  // 1 .. 2^24-1, tags the step's data words
    unsigned done;   // CTAs finished in this step (reset by the last one)
    unsigned error;  // nonzero: a bounded wait expired or an input was invalid
};

// Data words exchanged between CTAs: low 32 bits a float, high 32 bits the tag
// (epoch << 8 | layer << 3 | phase).  A reader polls a word until its tag matches.
// Words that many CTAs read are written to kReplicas copies (replica r at
// base + r * stride) and CTA c reads copy c % kReplicas, so the polling load of one
// exchange is spread over four times as many L2 lines.
constexpr int kReplicas = 4;
constexpr int replica_stride(int words) { return (words + 63) / 64 * 64 + 32; }

struct Scratch {
    unsigned long long *q;        // [DIM] rotated queries
    unsigned long long *kv;       // [kReplicas][KV_HEADS][2][HEAD_DIM] this position's K (rotated) and V
    unsigned long long *part;     // [HEADS][kMaxSplit][2] (max, sum of weights) of every attention split
    unsigned long long *dacc;     // [2][LAYERS][2][DIM, padded] down-projection sums: fixed point (value * 2^32) in
                                  // bits 8..63, additions counted in bits 0..7; two sets used by
                                  // alternating steps (epoch & 1), two copies per layer (writer parity)
    unsigned long long *xacc;     // [2][LAYERS][2][DIM, padded] attention block (O of every head) sums, the same form
    unsigned long long *cand;     // [kCTAs][64] per-CTA candidate keys (plain)
};

size_t scratch_words();  // total 64-bit words of the data-word buffers (q..h)
void carve_scratch(unsigned long long *base, Scratch *scr);  // lay q..h out in `base`

// Host side: build the per-CTA weight streams from the reference-format file in host
// memory, upload them and the chunk table; returns 0 on success.
int build_plan(const q8::FileHeader *hdr, const unsigned char *hfile, const unsigned char *dfile, Plan *hplan,
               Chunk **dchunks, uint8_t **dstream, size_t *stream_bytes, cudaStream_t s);

size_t smem_bytes();

// Enqueue one persistent step (cooperative launch) in `mode`.
int enqueue_step(const q8::Model *dm, const Plan *dplan, const q8::Buffers &b, Sync *sync, const Scratch &scr,
                 int mode, const sampling::Params *prm, sampling::SeqState *seq, int *out_ring, int *out_count,
                 const int *prompt, unsigned *host_error, cudaStream_t s, unsigned long long *trace = nullptr);

// Trace stamps per CTA: [0] start, layer l's points at 2 + kTraceLayer * l + k (k < 23,
// see the stamp() calls in the kernel), the head at kTraceHead + {0, 1, 2}.
constexpr int kTraceLayer = 24;
constexpr int kTraceHead = 2 + kTraceLayer * q8::LAYERS;  // 578
constexpr int kTraceStamps = 640;

int init_device();

}  // namespace q8p
