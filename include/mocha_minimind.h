/* Grouped-Q8 engine device ABI of libmocha_b200.so.
 *
 * Drop-in for the reference engine's device entry points (src/minimind.h:16-22,
 * implemented in src/minimind.cu:163-223): same names, argument meaning, return
 * codes (0 success, 1 any CUDA or argument error, message on stderr) and stderr
 * metric lines, so the reference host src/minimind.cpp links against this library
 * unchanged.  Differences: a B200 (compute capability 10.x) is required instead of
 * GK20A; MOCHA_LLM_CUDA_THREADS is validated (256/512/1024) but does not change the
 * kernels; gpu_collect returns the exact global top-k, a subset of the reference's
 * 64 partitions x k union that contains the same top k.
 * One model per process, single host thread, like the reference. The device is
 * MOCHA_DEVICE (default 0). */
#ifndef MOCHA_MINIMIND_ABI_H
#define MOCHA_MINIMIND_ABI_H

#ifdef __cplusplus
extern "C" {
#endif

/* src/minimind.cu:163 -- upload the whole grouped-Q8 file (validated like
 * src/minimind.cpp:89-93), allocate the KV cache, print
 * "BACKEND=cuda DEVICE=<name> Q8_GROUP=64 GPU_WEIGHTS=<bytes> GPU_KV=<bytes>". */
int gpu_init(const void *file, unsigned bytes);

/* src/minimind.cu:172 -- one decode step for `token` at `pos`; the KV cache is owned
 * by the library.  When project && readback, logits receives 151936 floats. */
int gpu_forward(float *logits, int token, int pos, int project, int readback);

/* src/minimind.cu:218 -- free everything, print CUDA_FORWARD_STEPS / CUDA_KERNEL_CALLS;
 * returns 1 when no step ran. */
int gpu_finish(void);

/* src/minimind.cu:197 -- hybrid mode: upload only the tied embedding / head t[0]. */
int gpu_head_init(const void *file);

/* src/minimind.cu:209 -- start the head projection of an already normalised hidden
 * vector (896 floats) over vocabulary rows [0, rows). */
int gpu_head_start(const float *input, int rows);

/* src/minimind.cu:215 -- wait for the head; copy rows logits when readback. */
int gpu_head_finish(float *logits, int rows, int readback);

/* src/minimind.cu:186 -- penalty (on the distinct ids of history[0..count)) + control
 * mask + top-k candidates of the last projected logits over ids [0, rows); on return
 * logits[0..rows) is -FLT_MAX except the candidates.  k in [1,64], count in [0,64]. */
int gpu_collect(float *logits, const int *history, int count, float penalty, int k, int rows);

#ifdef __cplusplus
}
#endif
#endif
