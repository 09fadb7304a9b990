/* GGUF quantised matmul bridge of libmocha_b200.so.
 *
 * Drop-in for the reference bridge (src/gguf-cuda.cu:110-144) that the llama.cpp
 * patch dlopens and calls from ggml_compute_forward_mul_mat
 * (tools/patch-gguf-cuda.py:25-34).  Same signature, argument checks and return codes
 * (0 success, 1 error, message on stderr) and the GGUF_CUDA_STATS line at exit. */
#ifndef MOCHA_GGUF_ABI_H
#define MOCHA_GGUF_ABI_H

#ifdef __cplusplus
extern "C" {
#endif

/* src/gguf-cuda.cu:110 -- y[v*y_stride + 4r] = sum_c W[r][c] * x[v*x_stride + 4c] for
 * v < vectors (<= 32), r < rows.  type is the ggml id: 8 = Q8_0, 12 = Q4_K, 14 = Q6_K;
 * cols % 256 == 0; strides in bytes; w, x, y are host pointers.  Weights stay
 * resident on the device, keyed by (host pointer, size) as the reference's cache is;
 * MOCHA_GGUF_GPU_CACHE_MIB is validated (0..256) as in the reference. */
int mocha_gguf_matmul(int type, const void *w, int cols, int rows, const float *x, int vectors,
                      unsigned x_stride, float *y, unsigned y_stride);

/* Exact (no fused multiply-add) dequantisation of rows x cols file-format weights
 * into out[r*cols + c] through the device layout the matmul uses.  A checking
 * entry point with no counterpart in the reference bridge; it uploads w afresh. */
int mocha_gguf_dequant(int type, const void *w, int cols, int rows, float *out);

#ifdef __cplusplus
}
#endif
#endif
