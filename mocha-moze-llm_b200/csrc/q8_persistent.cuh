// Persistent batch-1 decode kernel for the grouped-Q8 model: one cooperative launch
// per token over all 148 SMs.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "q8_decode.cuh"
#include "sampling.cuh"

namespace q8p {

constexpr int kCTAs = 148;             // one CTA per SM
constexpr int kConsumerWarps = 8;
constexpr int kThreads = 32 * (kConsumerWarps + 1);  // warp 0 streams weights
constexpr int kSlots = 5;              // shared-memory ring slots
constexpr int kSlotBytes = 36864;      // 7 rows of down (5168 B) or 38 rows of 896
constexpr int kAttnChunk = 32;         // positions per attention unit

enum Kind : uint32_t { QKV = 0, OPROJ = 1, GATEUP = 2, DOWN = 3, HEAD = 4 };
enum Phase { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GATEUP = 3, PH_DOWN = 4, kPhases = 5 };
enum Mode { FORWARD = 0, FORWARD_PROJECT = 1, PREFILL = 2, DECODE = 3 };

// One contiguous piece of a CTA's weight stream: `count` rows (or row pairs) starting
// at `first`, stored as int8 rows followed by their fp32 scales, padded to 16 bytes.
struct Chunk {
    uint64_t off;    // byte offset in the stream buffer
    uint32_t bytes;  // multiple of 16
    uint32_t kind;
    uint32_t layer;
    uint32_t first;  // first row / pair index within the matrix
    uint32_t count;  // rows or pairs
    uint32_t pad;
};

struct Plan {
    const uint8_t *stream;                 // all CTAs' streams back to back
    const Chunk *chunks;                   // all chunks, CTA-major
    uint32_t chunk_begin[kCTAs + 1];
    uint32_t head_lo[kCTAs + 1];           // contiguous vocabulary rows per CTA
};

// Global synchronisation words (zeroed once at set-up; targets grow with the epoch).
struct Sync {
    unsigned counters[q8::LAYERS][kPhases];
    unsigned done;
    unsigned epoch;
    unsigned error;                        // nonzero: a bounded wait expired
    unsigned tickets[q8::LAYERS][q8::KV_HEADS];
};

struct Scratch {
    float *o;                              // combined attention output [DIM]
    float *partial;                        // [KV_HEADS][CONTEXT/kAttnChunk][GQA][ATTN_PARTIAL]
    unsigned long long *cand;              // [kCTAs][64] per-CTA candidate keys
};

// Host side: build the per-CTA weight streams from the reference-format file in host
// memory, upload them and the chunk table; returns 0 on success.
int build_plan(const q8::FileHeader *hdr, const unsigned char *hfile, Plan *hplan, Chunk **dchunks,
               uint8_t **dstream, size_t *stream_bytes, cudaStream_t s);

size_t smem_bytes();

// Enqueue one persistent step (cooperative launch) in `mode`.
int enqueue_step(const q8::Model *dm, const Plan *dplan, const q8::Buffers &b, Sync *sync, const Scratch &scr,
                 int mode, const sampling::Params *prm, sampling::SeqState *seq, int *out_ring, int *out_count,
                 const int *prompt, unsigned *host_error, cudaStream_t s);

int init_device();

}  // namespace q8p
