// Repetition penalty, control-token mask, top-k candidates and on-device sampling.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace sampling {

constexpr int kMaxK = 64;           // largest k served by the candidate path
constexpr int kHistory = 64;        // penalty window (src/minimind.cpp:161)
constexpr int kStage1Blocks = 148;  // one CTA per SM

struct Params {
    float penalty;      // >= 1
    float temperature;  // 0 = greedy
    int top_k;          // 1..64
    float top_p;        // (0, 1]
    int eos;            // EOS id, left unmasked
    int control_first;  // ids >= this (except eos) are masked
    int vocab;          // valid token ids are [0, vocab)
};

// Per-sequence sampler state on the device.
struct SeqState {
    int history[kHistory];  // ring of the last kHistory tokens (prompt and generated)
    int history_count;      // entries in the ring (<= kHistory)
    int history_head;       // next write slot
    uint32_t seed;          // xorshift32 state
    int last_token;         // token sampled by the last step
    int finished;           // EOS seen
    int n_out;              // tokens written to the output ring
};

constexpr int kOutRing = 1024;  // output ring entries (index = n_out % kOutRing)

// Top-k candidate keys of logits[0..rows) after penalty (on the distinct ids of
// history[0..*count), device memory, order irrelevant) and mask.  keys_out receives k keys, best first.
// scratch must hold kStage1Blocks*kMaxK keys.
// Params are read from device memory so one captured graph serves every setting.
int enqueue_topk(const float *logits, int rows, const int *history, const int *count, const Params *p,
                 unsigned long long *scratch, unsigned long long *keys_out, cudaStream_t stream);

// Draw the next token from the sorted candidate keys (greedy when temperature == 0),
// exactly as the reference host sampler does (src/minimind.cpp:171-179), then push it
// into the history ring, write it to *token_out and, when out_ring is given, to
// out_ring[n_out % kOutRing] followed (after a system fence) by *out_count = n_out + 1;
// the ring may live in mapped host memory so a host thread can stream tokens.
int enqueue_sample(const unsigned long long *keys, const Params *p, SeqState *st, int *token_out,
                   int *pos_inout, int *out_ring, int *out_count, cudaStream_t stream);

// One-time per-device set-up (shared-memory opt-in of the merge kernel).
int init_device();

// Host helpers for decoding keys.
float key_value_host(unsigned long long k);
int key_id_host(unsigned long long k);

}  // namespace sampling
