/* Oracle for the grouped-Q8 Qwen2.5-0.5B token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * engine's CPU path (src/minimind.cpp) used to check the CUDA library.  Only the
 * tests, the smoke check and the CPU-baseline leg of the benchmark may load it;
 * nothing in the product library links or calls it.
 *
 * Parity pin: running the reference host (src/minimind.cpp, compiled from the
 * reference sources) with its gpu_* entry points served by this restatement and
 * --check enabled compares every logit of every step with the reference's own
 * cpu(); the recorded maximum absolute difference is 0 (bit-exact).  See
 * oracle/q8_oracle_shim.c and tests/test_oracle_q8.py.
 */
#ifndef MOCHA_Q8_ORACLE_H
#define MOCHA_Q8_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    Q8O_DIM = 896, Q8O_HIDDEN = 4864, Q8O_KV = 128, Q8O_HEAD = 64, Q8O_VOCAB = 151936,
    Q8O_CONTEXT = 1024, Q8O_LAYERS = 24, Q8O_STRIDE = 12, Q8O_TENSORS = 290,
    Q8O_EOS = 151645, Q8O_CONTROL_FIRST = 151643, Q8O_HEADER_BYTES = 8192
};

typedef struct { uint32_t data, scales, rows, cols; } q8o_tensor;
typedef struct q8o_model q8o_model;

/* Validate the header (src/minimind.cpp:89-93) and allocate the fp32 KV cache. */
q8o_model *q8o_create(const void *file, size_t bytes);
void q8o_destroy(q8o_model *m);
void q8o_reset(q8o_model *m);
const q8o_tensor *q8o_tensors(const q8o_model *m);
const uint8_t *q8o_base(const q8o_model *m);

/* One decode step (src/minimind.cpp:51-82).  When project is set, out receives
 * the 151936 logits, or the 896 normalised hidden values when hidden_only is set. */
void q8o_forward(q8o_model *m, int token, int pos, int project, int hidden_only, float *out);

/* y[r] (+)= sum_g s[r,g] * (sum_{j<64} w[r,64g+j] * x[64g+j]), rows [first, rows). */
void q8o_matvec(const int8_t *w, const float *s, unsigned rows, unsigned cols,
                const float *x, float *y, int add, unsigned first);
void q8o_rmsnorm(const float *x, const float *gain, int n, float eps, float *y);

/* Host sampler (src/minimind.cpp:160-179).  Modifies logits in place exactly as the
 * reference does: repetition penalty on the distinct ids of the last <=64 history
 * entries unless skip_penalty, control-token mask, then greedy (temp == 0) or
 * top-k / top-p with the xorshift32 state in *seed. */
int q8o_sample(float *logits, int vocab, const int *history, int history_len, float penalty,
               float temp, int top_k, float top_p, uint32_t *seed, int skip_penalty);

/* Candidate selection (src/minimind.cu:135-162 plus the host scatter at :193-194):
 * penalty + mask + per-partition top-k over 64 interleaved partitions.  Fills
 * out[0..rows) with -FLT_MAX except the selected candidates. Returns 1 on bad k/count. */
int q8o_collect(const float *logits, float *out, const int *recent, int count, float penalty,
                int k, int rows);

#ifdef __cplusplus
}
#endif
#endif
