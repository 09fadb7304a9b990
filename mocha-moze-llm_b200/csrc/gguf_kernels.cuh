// GGUF K-quant / Q8_0 weights on B200: device layout, repack, dequant and GEMV.
//
// Block formats are ggml's.  In HBM every block is stored so that all vector loads
// are 16-byte aligned, with exactly the file's bytes per block:
//   Q4_K: the 144-byte block unchanged (16-byte header d, dmin, 12 scale bytes,
//         then 128 bytes of nibbles);
//   Q6_K: a 208-byte body (ql 128, qh 64, int8 scales 16) per block in one array
//         [rows][blocks][208] and the fp16 d in a second array [rows][blocks];
//   Q8_0: int8 quants [rows][cols] and fp16 d [rows][cols/32].
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gguf {

enum Type { Q8_0 = 8, Q4_K = 12, Q6_K = 14 };

// Bytes of one file row, or 0 when type/cols are unsupported.
inline unsigned row_bytes(int type, int cols)
{
    if (cols <= 0) return 0;
    if (type == Q8_0) return cols % 32 ? 0 : (unsigned)(cols / 32) * 34u;
    if (type == Q4_K) return cols % 256 ? 0 : (unsigned)(cols / 256) * 144u;
    if (type == Q6_K) return cols % 256 ? 0 : (unsigned)(cols / 256) * 210u;
    return 0;
}

// A weight matrix resident in the device layout above.
struct DevMat {
    int type;
    int rows, cols;
    const uint8_t *body;     // Q4_K blocks / Q6_K bodies / Q8_0 quants
    const uint16_t *d;       // Q6_K and Q8_0 fp16 scales (null for Q4_K)
};

// Bytes of device storage for a matrix (same as the file's).
inline size_t dev_bytes(int type, int rows, int cols) { return (size_t)row_bytes(type, cols) * rows; }

// Repack `rows` file rows (raw, already on the device) into `dst` (dev_bytes long).
int enqueue_repack(int type, const uint8_t *raw, int rows, int cols, uint8_t *dst, cudaStream_t s);
DevMat make_devmat(int type, int rows, int cols, uint8_t *dst);

// out[r*cols + c] = dequantised weight, exact (no fused multiply-add), for checking.
int enqueue_dequant(const DevMat &m, float *out, cudaStream_t s);

// y[v*y_stride_f + r] (+)= sum_c W[r][c] * x[v*x_stride_f + c] for v < vectors (fp32
// activations, fp32 accumulation); strides in floats.  With accumulate the dot is added
// to y (residual connections).
int enqueue_gemv(const DevMat &m, const float *x, int vectors, int x_stride_f, float *y, int y_stride_f,
                 cudaStream_t s, bool accumulate = false);

// Fused GEMV of up to three matrices with the same input (q/k/v, gate/up):
// y[i][r] (+)= W_i[r] . xn for r < rows_i, where xn = x, or the RMSNorm of x with `gain`
// and `eps` when gain is non-null.  row_end[i] = rows of matrices 0..i together.
struct MultiGemv {
    DevMat m[3];
    float *y[3];
    int row_end[3];
    int n, cols, accumulate;
    const float *x, *gain;
    float eps;
};
int enqueue_gemv_multi(const MultiGemv &g, cudaStream_t s);

// out[c] = exact dequantised weight (row *row_index, read on the device), c < cols.
int enqueue_dequant_row(const DevMat &m, const int *row_index, float *out, cudaStream_t s);

// ---- tensor-core layout for the engine's GEMVs (csrc/gguf_mma.cu) ----------------------
//
// A matrix (rows a multiple of 16, cols a multiple of 256) repacked into 16-row tiles in
// the A-fragment order of mma.sync, with the file's bytes per weight.
struct MmaMat {
    int type;
    int rows, cols;
    const uint8_t *body;
};

// bytes of one 16-row tile, 0 when type/cols are unsupported
__host__ __device__ inline size_t mma_tile_bytes(int type, int cols)
{
    if (cols <= 0 || cols % 256) return 0;
    if (type == Q4_K) return (size_t)(cols / 256) * 2368;  // 64 B d|dmin, 256 B unpacked scales, 2048 B nibbles
    if (type == Q6_K) return (size_t)(cols / 256) * 3360;
    if (type == Q8_0) return (size_t)(cols / 32) * 544;
    return 0;
}
inline size_t mma_bytes(int type, int rows, int cols) { return rows % 16 ? 0 : mma_tile_bytes(type, cols) * (rows / 16); }

// Repack `rows` file rows (raw file bytes, on the device) into `dst` (mma_bytes long).
int enqueue_repack_mma(int type, const uint8_t *raw, int rows, int cols, uint8_t *dst, cudaStream_t s);

// y[i][r] (+)= W_i[r] . xn for up to three matrices with the same input, as MultiGemv.
struct MultiGemvMma {
    MmaMat m[3];
    float *y[3];
    int n, cols, accumulate;
    const float *x, *gain;
    const float *up;  // non-null: the input is silu(x) * up (SwiGLU folded into the down GEMV)
    float eps;
};
int enqueue_gemv_mma(const MultiGemvMma &g, cudaStream_t s);
// 1 (with a message) when a staged GEMV's bounded wait for its weights expired since the
// last call; clears the flag.
int gemv_take_timeout();

}  // namespace gguf
