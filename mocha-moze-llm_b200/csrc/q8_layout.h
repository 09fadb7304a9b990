// Grouped-Q8 Qwen2.5-0.5B model: shapes, file layout and device-side tensor table.
// Shapes and tensor order are the reference's (src/minimind.h:6-9 with MOCHA_QWEN,
// tools/convert-qwen.py:46-55); everything else is this library's own layout.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace q8 {

constexpr int DIM = 896, HIDDEN = 4864, KV = 128, HEAD_DIM = 64, VOCAB = 151936;
constexpr int CONTEXT = 1024, LAYERS = 24, STRIDE = 12, TENSORS = 290, HEADER_BYTES = 8192;
constexpr int HEADS = DIM / HEAD_DIM;      // 14 query heads
constexpr int KV_HEADS = KV / HEAD_DIM;    // 2 key/value heads
constexpr int GQA = HEADS / KV_HEADS;      // 7 query heads share one KV head
constexpr int GROUP = 64;                  // weights per fp32 scale
constexpr int EOS = 151645, CONTROL_FIRST = 151643;
constexpr float RMS_EPS = 1e-6f;
constexpr uint32_t MAGIC = 0x384D4D4Du;

// per-layer tensor slots relative to 1 + 12*layer
enum Slot { ATTN_NORM, WQ, WK, WV, WO, WGATE, WUP, WDOWN, FFN_NORM, BQ, BK, BV };

struct FileTensor { uint32_t data, scales, rows, cols; };  // src/minimind.h:5
struct FileHeader {                                         // src/minimind.h:15
    uint32_t magic, version, bytes, dim, hidden, layers, vocab, group;
    FileTensor t[TENSORS];
};

// A grouped-Q8 matrix resident in HBM: int8 row-major [rows][cols] and fp32 scales
// [rows][cols/64].
struct Mat {
    const int8_t *w;
    const float *s;
};

struct Layer {
    const float *attn_norm, *ffn_norm, *bq, *bk, *bv;
    Mat q, k, v, o, gate, up, down;
};

struct Model {
    Mat embed;  // also the tied vocabulary head
    const float *final_norm;
    Layer layer[LAYERS];
};

// Header and tensor-table checks of the reference loader plus 16-byte alignment of
// every tensor (head_only: only the embedding needs to be present).
bool valid_file(const void *file, size_t bytes, bool head_only);

// Split-K attention: positions are processed in chunks of ATTN_CHUNK per CTA.
constexpr int ATTN_CHUNK = 32;
constexpr int ATTN_MAX_CHUNKS = CONTEXT / ATTN_CHUNK;
constexpr int ATTN_PARTIAL = HEAD_DIM + 2;  // running max, sum of weights, 64 accumulators

// Per-sequence decode state kept on the device.
struct DecodeState {
    int token;       // input token of the next step
    int pos;         // its position
    int steps;       // forward steps run
    int generated;   // tokens sampled on the device
    uint32_t seed;   // xorshift32 sampler state
    int error;       // nonzero when a device-side check failed
};

}  // namespace q8
