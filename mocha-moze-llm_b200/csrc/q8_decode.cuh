// Batch-1 grouped-Q8 decode step on B200: device buffers and launch entry points.
#pragma once
#include <cuda_runtime.h>

#include "q8_layout.h"

namespace q8 {

struct Buffers {
    float *x;         // residual stream [DIM]
    float *q;         // rotated queries [DIM]
    float *kc, *vc;   // KV cache [LAYERS][KV_HEADS][CONTEXT][HEAD_DIM], fp32
    float *partial;   // split-K attention partials [KV_HEADS][ATTN_MAX_CHUNKS][GQA][ATTN_PARTIAL]
    float *h;         // SwiGLU output [HIDDEN]
    float *logits;    // [VOCAB]
    float *hidden;    // final normalised hidden state [DIM]
    const float *rope_cos, *rope_sin;  // [CONTEXT][HEAD_DIM/2]
    DecodeState *st;  // token / pos of the step
};

// Enqueue one forward step for state->token at state->pos.  When project is set the
// final norm and the tied vocabulary projection run too and buf.logits is filled.
int enqueue_forward(const Model *dmodel, const Model &hmodel, const Buffers &buf, bool project,
                    cudaStream_t stream);

// Vocabulary projection of an already normalised hidden vector (hybrid head mode):
// logits[r] = E[r] . hidden for r < rows.
int enqueue_head_only(const Mat &embed, const float *hidden, float *logits, int rows,
                      cudaStream_t stream);

// Host-side RoPE tables computed exactly as the reference CPU does
// (angle = pos * powf(1e6, -2i/64), cosf/sinf; src/minimind.cpp:63).
void fill_rope_tables(float *cos_table, float *sin_table, int context, int half, float theta);

// Number of kernels enqueue_forward launches.
int forward_launches(bool project);

}  // namespace q8
