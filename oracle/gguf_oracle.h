/* Oracle for the GGUF Q4_K / Q6_K / Q8_0 dequant-matmul bridge.
 *
 * TEST INFRASTRUCTURE ONLY: a plain-C restatement of the reference bridge's scalar
 * dequantisation (src/gguf-cuda.cu:23-44) and of its matmul contract
 * (src/gguf-cuda.cu:110-144).  Pinned bit-exactly against the dequantisers of the
 * gguf Python package 0.19.0 (tests/golden/make_gguf_golden.py). */
#ifndef MOCHA_GGUF_ORACLE_H
#define MOCHA_GGUF_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { GGUF_O_Q8_0 = 8, GGUF_O_Q4_K = 12, GGUF_O_Q6_K = 14 };

float gguf_o_half(uint16_t h);
/* bytes of one row of `cols` weights, or 0 for an unsupported type/shape */
unsigned gguf_o_row_bytes(int type, int cols);
void gguf_o_dequant_row(int type, const uint8_t *row, int cols, float *out);
/* y[v*y_stride + 4r] = sum_c w(r,c) * x[v*x_stride + 4c] (strides in bytes), float
 * accumulation in column order; same argument checks as the bridge (returns 1). */
int gguf_o_matmul(int type, const void *w, int cols, int rows, const float *x, int vectors,
                  unsigned x_stride, float *y, unsigned y_stride);

#ifdef __cplusplus
}
#endif
#endif
