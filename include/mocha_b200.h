/* Handle-based entry points of libmocha_b200.so for the B200 token loop.
 *
 * These run the reference host's whole token loop (src/minimind.cpp:110-182: prompt
 * steps that only fill the KV cache, projection at the last prompt position,
 * penalty + control mask + greedy or top-k/top-p/xorshift32 sampling, EOS stop) on
 * the device, with an explicit device index so several replicas can run in one
 * process.  They sit alongside the reference ABI (mocha_minimind.h), which stays
 * the drop-in boundary; there is no reference counterpart for the handles
 * themselves.  All functions return 0 on success and 1 on error (message on
 * stderr). */
#ifndef MOCHA_B200_H
#define MOCHA_B200_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mocha_q8 mocha_q8;

/* Sampling settings with the reference CLI's meaning (mocha-llm:69-73):
 * temperature 0 = greedy; top_k in [1,64] on the device path; top_p in (0,1];
 * repeat_penalty >= 1 over the last 64 tokens; seed = xorshift32 start state. */
typedef struct {
    float temperature;
    int top_k;
    float top_p;
    float repeat_penalty;
    unsigned seed;
} mocha_sampling;

typedef struct {
    double prefill_s;  /* prompt positions, measured with CUDA events */
    double decode_s;   /* generated tokens after the first, CUDA events */
    int generated;     /* tokens before EOS (EOS itself is not counted) */
} mocha_timing;

/* Number of visible CUDA devices with compute capability 10.x. */
int mocha_b200_device_count(void);

/* Upload a grouped-Q8 Qwen2.5-0.5B file (reference format) to `device`. */
int mocha_q8_open(int device, const void *file, unsigned long long bytes, mocha_q8 **out);
int mocha_q8_close(mocha_q8 *h);

/* One step for `token` at `pos` (same as gpu_forward on a handle). */
int mocha_q8_forward(mocha_q8 *h, int token, int pos, int project, float *logits);

/* Run the token loop: n_prompt prompt tokens, then up to n_new sampled tokens,
 * written to out_tokens (capacity n_new); *n_out = tokens before EOS.
 * n_prompt + n_new <= 1024 as in the reference (src/minimind.cpp:98). */
int mocha_q8_generate(mocha_q8 *h, const int *prompt, int n_prompt, int n_new, const mocha_sampling *s,
                      int *out_tokens, int *n_out, mocha_timing *timing);

/* Streaming form of mocha_q8_generate for hosts that print tokens as they come
 * (the reference host prints one id per line, src/minimind.cpp:181).  begin enqueues
 * the prompt steps and a few decode steps; each next returns the next sampled token
 * (EOS included, once) and keeps a fixed number of steps in flight; *token = -1 once
 * the stream has ended.  end waits for the steps still in flight. */
int mocha_q8_stream_begin(mocha_q8 *h, const int *prompt, int n_prompt, int n_new, const mocha_sampling *s);
int mocha_q8_stream_next(mocha_q8 *h, int *token);
int mocha_q8_stream_end(mocha_q8 *h);

/* Device-timed decode: after the KV cache holds positions [0, pos0), run `warmup`
 * then `steps` greedy steps with the token fed back on the device, starting at
 * (token, pos0) and restarting at pos0 whenever the position reaches pos_end.
 * *ms = CUDA-event time of the timed steps. */
int mocha_q8_bench_decode(mocha_q8 *h, int token, int pos0, int pos_end, int warmup, int steps, float *ms);

/* Number of this library's kernel launches per decode step (projection + sampling). */
int mocha_q8_launches_per_step(mocha_q8 *h);

/* Diagnostic: one persistent step (forward + projection) for `token` at `pos` that
 * records %globaltimer stamps of every CTA into stamps[148][640] (0 = not reached):
 * [0] start; per layer l at 2 + 24 l: +0 x_in gathered, +11 QKV chunk taken, +12 its
 * input normalised and quantized, +13 QKV products done, +1 QKV done, +14 query and
 * K/V words arrived (attention CTAs), +15 past K/V resident, +16 split softmax and
 * P.V done, +2 attention done, +17 partials gathered, +3 attention combined, +4 O
 * done, +5 x_mid gathered, +9 gate/up chunks resident, +10 gate/up input quantized,
 * +18 gate/up products done, +7 SwiGLU done, +19 SwiGLU slice quantized, +20 down
 * chunk taken, +21 down products done, +6 down partials stored, +22 own rows polled,
 * +8 own rows reduced; [578] head start, [579] head done, [580] token drawn.
 * Fails on the per-phase graph path. */
int mocha_q8_trace_step(mocha_q8 *h, int token, int pos, unsigned long long *stamps);

/* Penalty + control mask + top-k candidates (the selection gpu_collect performs)
 * for callers that cannot allocate device memory at call time: a host that has
 * reserved the whole GPU memory budget in its own pool, or a latency-critical loop
 * that must not take cudaMalloc's implicit device synchronisation.  No counterpart
 * in the reference.  logits[0..rows) and history[0..count) are host arrays; the k
 * best (value, id) pairs, penalised values and ties to the lower id first, go to
 * host values[k] / ids[k]; the call waits for `stream` (may be NULL) before it
 * returns.  The control mask is Qwen2.5's: ids >= 151643 other than EOS 151645 are
 * set to -1e30 (it only touches rows past 151643).  All device buffers live in one
 * fixed ~672 KiB __device__ array, so 1 <= k <= min(64, rows) and rows <= 151936;
 * other requests fail with a message.  The first call on a device looks the array's
 * address up (make it before any stream capture on that device); a call on a stream
 * that is being captured fails with a message; calls that overlap on the GPU share
 * the array and race. */
int mocha_topk_static(const float *logits, int rows, const int *history, int count, float penalty, int k,
                      float *values, int *ids, void *stream);

/* Forward steps and kernel launches issued on this handle so far (the counters the
 * reference prints at exit as CUDA_FORWARD_STEPS / CUDA_KERNEL_CALLS). */
int mocha_q8_counters(mocha_q8 *h, unsigned long long *steps, unsigned long long *launches);

/* ---- GGUF models (llama / qwen2, Q4_K / Q6_K / Q8_0 weights) --------------------
 * The forward of the reference's GGUF path (llama.cpp's graph for these
 * architectures, whose matmuls the reference bridge offloads) with attention,
 * RoPE, norms, KV cache and sampling on the device as well.  No counterpart handle
 * exists in the reference; the matmul bridge itself is mocha_gguf_matmul. */
typedef struct mocha_gguf mocha_gguf;

typedef struct {
    int arch;           /* 0 = llama, 1 = qwen2 */
    int layers, dim, ffn, heads, kv_heads, head_dim, vocab, context;
    float eps, rope_base;
    int rope_neox;      /* 1: split-half pairs (qwen2); 0: interleaved pairs (llama) */
    int rope_factors;   /* 1 when rope_freqs.weight (llama3 scaling) is present */
    int eos;            /* tokenizer.ggml.eos_token_id, or -1 */
} mocha_gguf_info;

/* Parse a GGUF v2/v3 file in host memory and upload it to `device`. */
int mocha_gguf_open(int device, const void *file, unsigned long long bytes, mocha_gguf **out);
int mocha_gguf_close(mocha_gguf *m);
int mocha_gguf_get_info(mocha_gguf *m, mocha_gguf_info *info);
/* One step for `token` at `pos`; with project, logits (vocab floats) are returned. */
int mocha_gguf_forward(mocha_gguf *m, int token, int pos, int project, float *logits);
/* Device-side token loop as mocha_q8_generate (no control-token mask; EOS from the file). */
int mocha_gguf_generate(mocha_gguf *m, const int *prompt, int n_prompt, int n_new, const mocha_sampling *s,
                        int *out_tokens, int *n_out, mocha_timing *timing);
/* Device-timed greedy decode as mocha_q8_bench_decode. */
int mocha_gguf_bench_decode(mocha_gguf *m, int token, int pos0, int pos_end, int warmup, int steps, float *ms);
int mocha_gguf_launches_per_step(mocha_gguf *m);

/* ---- batched engine: prefill and multi-sequence decode on tensor cores ------------
 * The batched extension of the reference ABI (gpu_forward_batch / gpu_sample_batch /
 * gpu_prefill with an explicit device index; no reference counterpart).  A handle owns
 * the model file as stored (int8 weights + fp32 scales), row-fused int8 copies of
 * q|k|v and gate|up for the tcgen05 GEMMs (248 MB), activation
 * buffers for `max_rows` rows and the fp32 KV cache of `slots` sequences
 * ([slot][layer][kv head][pos][64]). */
typedef struct mocha_q8b mocha_q8b;

int mocha_q8b_open(int device, const void *file, unsigned long long bytes, int max_rows, int slots, mocha_q8b **out);
int mocha_q8b_close(mocha_q8b *h);

/* One forward over n rows: row i runs tokens[i] at position pos[i] of KV slot
 * slots[i] (keys 0..pos[i] of that slot must already hold earlier positions; rows of
 * one slot run in increasing position order within the call).  Logits of the
 * n_project rows listed in project_rows go to logits[n_project][151936] when non-NULL
 * (n_project <= slots). */
int mocha_q8b_forward(mocha_q8b *h, int n, const int *tokens, const int *pos, const int *slots, int n_project,
                      const int *project_rows, float *logits);

/* Prompt prefill of one slot: positions 0..n-1; logits of the last position. */
int mocha_q8b_prefill(mocha_q8b *h, int slot, const int *tokens, int n, float *logits);

/* The reference token loop for nseq sequences of prompt_len tokens each: n_new tokens
 * per sequence (fewer if EOS comes first; EOS not reported), sampling as in
 * mocha_sampling with seed seed_base + sequence index.  out_tokens[nseq][n_new],
 * out_counts[nseq].  Continuous batching: min(slots, max_rows / prompt_len) sequences
 * decode together, one row per slot; a slot whose sequence finishes is refilled with
 * the next waiting sequence (its prompt pass, then it joins the decode steps). */
int mocha_q8b_generate(mocha_q8b *h, int nseq, const int *prompts, int prompt_len, int n_new,
                       const mocha_sampling *sampling, unsigned seed_base, int *out_tokens, int *out_counts,
                       mocha_timing *timing);

/* mocha_q8b_generate with a token budget per sequence, n_new[i] <= out_stride:
 * out_tokens[nseq][out_stride].  Sequences with smaller budgets leave their slots
 * early, and waiting sequences take them mid-stream. */
int mocha_q8b_generate_each(mocha_q8b *h, int nseq, const int *prompts, int prompt_len, const int *n_new,
                            const mocha_sampling *sampling, unsigned seed_base, int *out_tokens, int out_stride,
                            int *out_counts, mocha_timing *timing);

/* Device-timed prefill of an n-token seeded random prompt in slot 0 (head on the
 * last position): warmup passes, then *ms = CUDA-event time of `steps` passes. */
int mocha_q8b_bench_prefill(mocha_q8b *h, int n, unsigned seed, int warmup, int steps, float *ms);

/* Kernels launched by one decode step of the batched loop. */
int mocha_q8b_launches_per_step(mocha_q8b *h);

/* The batched sampler alone on caller logits[n][151936]: history[n][64] with counts
 * (penalty window), seeds[n]; writes tokens[n]. */
int mocha_q8b_sample_check(mocha_q8b *h, int n, const float *logits, const int *history, const int *history_counts,
                           const mocha_sampling *sampling, const unsigned *seeds, int *tokens);

/* ---- tensor-core GEMM check (no reference counterpart) ----------------------------
 * y[n][rows] = x[n][cols] . dequant(q, scales)^T for one grouped-Q8 matrix (int8
 * [rows][cols] row-major, fp32 scale per 64 consecutive weights), computed by the
 * tcgen05 GEMM of the batched paths.  rows % 128 == 0, cols % 64 == 0, 1 <= n <= 1024;
 * splits = 0 lets the kernel choose its K split.  Allocates and frees its own device
 * buffers; for tests. */
int mocha_tc_gemm_check(int device, int rows, int n, int cols, const signed char *q, const float *scales,
                        const float *x, float *y, int splits);

/* The same product through the int8 tcgen05 GEMM of the batched engine: x split into
 * three int8 limbs per 64-group, exact int32 group sums, fp32 promotion.
 * rows % 128 == 0, cols % 128 == 0, 1 <= n <= 1024.  No reference counterpart. */
int mocha_tq_gemm_check(int device, int rows, int n, int cols, const signed char *q, const float *scales,
                        const float *x, float *y, int splits);

#ifdef __cplusplus
}
#endif
#endif
