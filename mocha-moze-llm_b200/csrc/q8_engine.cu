// Grouped-Q8 engine state and C ABI: the reference device entry points
// (src/minimind.h:16-22) and the handle-based token-loop API of mocha_b200.h.
//
// One engine per device: the whole reference-format file lives in HBM as uploaded
// (tensor offsets from the header), the fp32 KV cache is [layer][kv head][pos][64],
// and every per-token sequence of kernels is captured once into a CUDA graph whose
// kernels read the token and position from device memory.
#include <cuda_runtime.h>
#include <float.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "mb_common.cuh"
#include "mocha_b200.h"
#include "mocha_minimind.h"
#include "q8_decode.cuh"
#include "q8_persistent.cuh"
#include "sampling.cuh"

namespace {

using q8::CONTEXT;
using q8::DIM;
using q8::VOCAB;

double now_s()
{
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

__global__ void k_advance_prompt(q8::DecodeState *st, const int *prompt)
{
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        st->steps++;
        st->pos++;
        st->token = prompt[st->pos];
    }
}

__global__ void k_count_step(q8::DecodeState *st)
{
    if (threadIdx.x == 0 && blockIdx.x == 0) st->steps++;
}

}  // namespace

namespace q8 {

// Header and tensor-table checks of src/minimind.cpp:89-93, plus the 16-byte
// alignment the vector loads need.
bool valid_file(const void *file, size_t bytes, bool head_only)
{
    if (!file || bytes < (size_t)q8::HEADER_BYTES) return false;
    const q8::FileHeader *h = (const q8::FileHeader *)file;
    if (h->magic != q8::MAGIC || h->version != 1 || (!head_only && h->bytes != bytes) || h->dim != (uint32_t)DIM ||
        h->hidden != (uint32_t)q8::HIDDEN || h->layers != (uint32_t)q8::LAYERS || h->vocab != (uint32_t)VOCAB ||
        h->group != 64)
        return false;
    const size_t limit = head_only ? (size_t)h->bytes : bytes;
    for (int i = 0; i < q8::TENSORS; i++) {
        const q8::FileTensor t = h->t[i];
        const uint64_t size = (uint64_t)t.rows * (t.scales ? t.cols : 4);
        if (t.data < (uint32_t)q8::HEADER_BYTES || t.data + size > limit) return false;
        if (t.scales && (t.cols % 64 || t.scales + size / 64 * 4 > limit)) return false;
        if (t.data % 16 || t.scales % 16) return false;
    }
    return true;
}

}  // namespace q8

struct mocha_q8 {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool head_only = false;
    unsigned char *d_file = nullptr;
    size_t bytes = 0;
    q8::Model hm{};
    q8::Model *dm = nullptr;
    q8::Buffers b{};
    q8::DecodeState *h_state = nullptr;  // pinned staging for token/pos
    sampling::SeqState *d_seq = nullptr;
    sampling::Params *d_params = nullptr, *h_params = nullptr;
    int *d_hist = nullptr, *h_hist = nullptr;  // [64 ids][count]
    unsigned long long *d_scratch = nullptr, *d_keys = nullptr, *h_keys = nullptr;
    float *h_logits = nullptr;
    int *d_prompt = nullptr, *h_pos0 = nullptr;
    int *h_out = nullptr, *h_out_count = nullptr;  // mapped pinned ring written by the sampler
    int *d_out = nullptr, *d_out_count = nullptr;  // their device addresses
    int stream_total = 0, stream_enqueued = 0, stream_read = 0;
    bool stream_done = true;
    cudaGraphExec_t g_forward[2] = {nullptr, nullptr};
    cudaGraphExec_t g_prefill = nullptr, g_decode = nullptr;
    // kStepsPerGraph consecutive prompt / decode steps in one graph: each step reads the
    // token and position the previous one wrote, as with separate launches, and the
    // steps follow each other as kernel nodes of one graph instead of graph launches
    cudaGraphExec_t g_prefill_n = nullptr, g_decode_n = nullptr;
    cudaEvent_t ev[4] = {};
    // persistent one-launch-per-token path (default) and its state
    bool persistent = true;
    q8p::Plan hplan{};
    q8p::Plan *dplan = nullptr;
    q8p::Chunk *dchunks = nullptr;
    uint8_t *dstream = nullptr;
    size_t stream_bytes = 0;
    q8p::Sync *dsync = nullptr;
    q8p::Scratch scr{};
    unsigned long long *dwords = nullptr;  // data words exchanged between CTAs
    unsigned *h_err = nullptr, *d_err = nullptr;  // mapped error word of the bounded waits
    unsigned long long calls = 0, kernel_calls = 0;
    double transformer_s = 0, head_s = 0, copy_s = 0;
};

namespace {

#define TRY(x)                                                                                   \
    do {                                                                                         \
        cudaError_t e_ = (x);                                                                    \
        if (e_ != cudaSuccess) {                                                                 \
            fprintf(stderr, "CUDA %s: %d %s\n", #x, (int)e_, cudaGetErrorString(e_));           \
            return 1;                                                                            \
        }                                                                                        \
    } while (0)

int reset_persistent(mocha_q8 *h);

int check_device(int device, cudaDeviceProp *p)
{
    int n = 0;
    TRY(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) {
        fprintf(stderr, "MOCHA_B200: device %d not present (%d visible)\n", device, n);
        return 1;
    }
    TRY(cudaGetDeviceProperties(p, device));
    if (p->major != 10) {
        fprintf(stderr, "MOCHA_B200: requires a compute capability 10.x (B200) device, found %d.%d\n", p->major,
                p->minor);
        return 1;
    }
    TRY(cudaSetDevice(device));
    return 0;
}

q8::Mat mat_of(const unsigned char *base, const q8::FileTensor &t)
{
    return q8::Mat{(const int8_t *)(base + t.data), (const float *)(base + t.scales)};
}

constexpr int kStepsPerGraph = 8;
int enqueue_one(mocha_q8 *h, int kind);

int capture(mocha_q8 *h, cudaGraphExec_t *out, int kind, int steps = 1)
{
    cudaGraph_t g = nullptr;
    TRY(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    int rc = 0;
    for (int i = 0; i < steps && !rc; i++) rc = enqueue_one(h, kind);
    const cudaError_t end = cudaStreamEndCapture(h->stream, &g);
    if (rc || end != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        fprintf(stderr, "CUDA graph capture failed: %s\n", cudaGetErrorString(end));
        return 1;
    }
    const cudaError_t inst = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    TRY(inst);
    return 0;
}

// Launch `count` prompt (kind 2) or decode (kind 3) steps: whole graphs of
// kStepsPerGraph, then single steps.
int launch_steps(mocha_q8 *h, int kind, int count)
{
    cudaGraphExec_t one = kind == 2 ? h->g_prefill : h->g_decode, many = kind == 2 ? h->g_prefill_n : h->g_decode_n;
    for (; count >= kStepsPerGraph; count -= kStepsPerGraph) TRY(cudaGraphLaunch(many, h->stream));
    for (; count > 0; count--) TRY(cudaGraphLaunch(one, h->stream));
    return 0;
}

// One step of `kind` into the stream being captured.
int enqueue_one(mocha_q8 *h, int kind)
{
    int rc = 0;
    if (h->persistent) {
        static const int modes[4] = {q8p::FORWARD, q8p::FORWARD_PROJECT, q8p::PREFILL, q8p::DECODE};
        rc = q8p::enqueue_step(h->dm, h->dplan, h->b, h->dsync, h->scr, modes[kind], h->d_params, h->d_seq, h->d_out,
                               h->d_out_count, h->d_prompt, h->d_err, h->stream);
    } else if (kind == 0 || kind == 1) {  // bare forward without / with projection
        rc = q8::enqueue_forward(h->dm, h->hm, h->b, kind == 1, h->stream);
        if (!rc) k_count_step<<<1, 1, 0, h->stream>>>(h->b.st);
    } else if (kind == 2) {  // prompt step: fill KV, advance to the next prompt token
        rc = q8::enqueue_forward(h->dm, h->hm, h->b, false, h->stream);
        if (!rc) k_advance_prompt<<<1, 1, 0, h->stream>>>(h->b.st, h->d_prompt);
    } else {  // decode step: project, select, sample, feed the token back
        rc = q8::enqueue_forward(h->dm, h->hm, h->b, true, h->stream);
        if (!rc) k_count_step<<<1, 1, 0, h->stream>>>(h->b.st);
        if (!rc)
            rc = sampling::enqueue_topk(h->b.logits, VOCAB, h->d_seq->history, &h->d_seq->history_count,
                                        h->d_params, h->d_scratch, h->d_keys, h->stream);
        if (!rc)
            rc = sampling::enqueue_sample(h->d_keys, h->d_params, h->d_seq, &h->b.st->token, &h->b.st->pos,
                                          h->d_out, h->d_out_count, h->stream);
    }
    return rc;
}

int alloc_common(mocha_q8 *h)
{
    TRY(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    for (auto &e : h->ev) TRY(cudaEventCreate(&e));
    TRY(cudaMalloc(&h->b.logits, sizeof(float) * VOCAB));
    TRY(cudaMalloc(&h->b.hidden, sizeof(float) * DIM));
    TRY(cudaMalloc(&h->d_seq, sizeof(sampling::SeqState)));
    TRY(cudaMemset(h->d_seq, 0, sizeof(sampling::SeqState)));
    TRY(cudaMalloc(&h->d_params, sizeof(sampling::Params)));
    TRY(cudaMallocHost(&h->h_params, sizeof(sampling::Params)));
    TRY(cudaMalloc(&h->d_hist, sizeof(int) * 65));
    TRY(cudaMallocHost(&h->h_hist, sizeof(int) * 65));
    TRY(cudaMalloc(&h->d_scratch, sizeof(unsigned long long) * sampling::kStage1Blocks * sampling::kMaxK));
    TRY(cudaMalloc(&h->d_keys, sizeof(unsigned long long) * sampling::kMaxK));
    TRY(cudaMallocHost(&h->h_keys, sizeof(unsigned long long) * sampling::kMaxK));
    TRY(cudaMallocHost(&h->h_logits, sizeof(float) * VOCAB));
    if (sampling::init_device()) return 1;
    return 0;
}

int open_full(mocha_q8 *h, int device, const void *file, size_t bytes)
{
    cudaDeviceProp p;
    if (check_device(device, &p)) return 1;
    h->device = device;
    h->bytes = bytes;
    if (alloc_common(h)) return 1;
    TRY(cudaMalloc(&h->d_file, bytes));
    TRY(cudaMemcpy(h->d_file, file, bytes, cudaMemcpyHostToDevice));
    const q8::FileHeader *hd = (const q8::FileHeader *)file;
    h->hm.embed = mat_of(h->d_file, hd->t[0]);
    h->hm.final_norm = (const float *)(h->d_file + hd->t[q8::TENSORS - 1].data);
    for (int l = 0; l < q8::LAYERS; l++) {
        const q8::FileTensor *t = hd->t + 1 + l * q8::STRIDE;
        q8::Layer &L = h->hm.layer[l];
        L.attn_norm = (const float *)(h->d_file + t[q8::ATTN_NORM].data);
        L.ffn_norm = (const float *)(h->d_file + t[q8::FFN_NORM].data);
        L.bq = (const float *)(h->d_file + t[q8::BQ].data);
        L.bk = (const float *)(h->d_file + t[q8::BK].data);
        L.bv = (const float *)(h->d_file + t[q8::BV].data);
        L.q = mat_of(h->d_file, t[q8::WQ]);
        L.k = mat_of(h->d_file, t[q8::WK]);
        L.v = mat_of(h->d_file, t[q8::WV]);
        L.o = mat_of(h->d_file, t[q8::WO]);
        L.gate = mat_of(h->d_file, t[q8::WGATE]);
        L.up = mat_of(h->d_file, t[q8::WUP]);
        L.down = mat_of(h->d_file, t[q8::WDOWN]);
    }
    TRY(cudaMalloc(&h->dm, sizeof(q8::Model)));
    TRY(cudaMemcpy(h->dm, &h->hm, sizeof(q8::Model), cudaMemcpyHostToDevice));

    const size_t kv = (size_t)q8::LAYERS * q8::KV_HEADS * CONTEXT * q8::HEAD_DIM;
    TRY(cudaMalloc(&h->b.x, sizeof(float) * DIM));
    TRY(cudaMalloc(&h->b.q, sizeof(float) * DIM));
    TRY(cudaMalloc(&h->b.kc, sizeof(float) * kv));
    TRY(cudaMalloc(&h->b.vc, sizeof(float) * kv));
    TRY(cudaMemset(h->b.kc, 0, sizeof(float) * kv));
    TRY(cudaMemset(h->b.vc, 0, sizeof(float) * kv));
    TRY(cudaMalloc(&h->b.partial,
                   sizeof(float) * q8::KV_HEADS * q8::ATTN_MAX_CHUNKS * q8::GQA * q8::ATTN_PARTIAL));
    TRY(cudaMalloc(&h->b.h, sizeof(float) * q8::HIDDEN));
    float *rope = nullptr;
    TRY(cudaMalloc(&rope, sizeof(float) * CONTEXT * 32 * 2));
    {
        float *tab = (float *)malloc(sizeof(float) * CONTEXT * 32 * 2);
        if (!tab) return 1;
        q8::fill_rope_tables(tab, tab + CONTEXT * 32, CONTEXT, 32, 1000000.f);
        const cudaError_t e = cudaMemcpy(rope, tab, sizeof(float) * CONTEXT * 64, cudaMemcpyHostToDevice);
        free(tab);
        TRY(e);
    }
    h->b.rope_cos = rope;
    h->b.rope_sin = rope + CONTEXT * 32;
    q8::DecodeState *st = nullptr;
    TRY(cudaMalloc(&st, sizeof(q8::DecodeState)));
    TRY(cudaMemset(st, 0, sizeof(q8::DecodeState)));
    h->b.st = st;
    TRY(cudaMallocHost(&h->h_state, sizeof(q8::DecodeState)));
    memset(h->h_state, 0, sizeof(q8::DecodeState));
    TRY(cudaMallocHost(&h->h_pos0, sizeof(int) * 2));
    TRY(cudaMalloc(&h->d_prompt, sizeof(int) * CONTEXT));
    TRY(cudaHostAlloc(&h->h_out, sizeof(int) * sampling::kOutRing, cudaHostAllocMapped));
    TRY(cudaHostAlloc(&h->h_out_count, sizeof(int), cudaHostAllocMapped));
    TRY(cudaHostGetDevicePointer(&h->d_out, h->h_out, 0));
    TRY(cudaHostGetDevicePointer(&h->d_out_count, h->h_out_count, 0));
    *h->h_out_count = 0;
    const char *mode = getenv("MOCHA_B200_DECODE");
    h->persistent = !(mode && strcmp(mode, "graph") == 0);
    if (h->persistent) {
        if (q8p::init_device()) return 1;
        if (q8p::build_plan(hd, (const unsigned char *)file, h->d_file, &h->hplan, &h->dchunks, &h->dstream,
                            &h->stream_bytes, h->stream))
            return 1;
        TRY(cudaMalloc(&h->dplan, sizeof(q8p::Plan)));
        TRY(cudaMemcpy(h->dplan, &h->hplan, sizeof(q8p::Plan), cudaMemcpyHostToDevice));
        TRY(cudaMalloc(&h->dsync, sizeof(q8p::Sync)));
        TRY(cudaMalloc(&h->dwords, sizeof(unsigned long long) * q8p::scratch_words()));
        q8p::carve_scratch(h->dwords, &h->scr);
        TRY(cudaMalloc(&h->scr.cand, sizeof(unsigned long long) * q8p::kCTAs * sampling::kMaxK));
        if (reset_persistent(h)) return 1;
    }
    TRY(cudaHostAlloc(&h->h_err, sizeof(unsigned), cudaHostAllocMapped));
    TRY(cudaHostGetDevicePointer(&h->d_err, h->h_err, 0));
    *h->h_err = 0;
    if (capture(h, &h->g_forward[0], 0) || capture(h, &h->g_forward[1], 1) || capture(h, &h->g_prefill, 2) ||
        capture(h, &h->g_decode, 3) || capture(h, &h->g_prefill_n, 2, kStepsPerGraph) ||
        capture(h, &h->g_decode_n, 3, kStepsPerGraph))
        return 1;
    TRY(cudaStreamSynchronize(h->stream));
    return 0;
}

void release(mocha_q8 *h)
{
    if (!h) return;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    for (auto g : h->g_forward)
        if (g) cudaGraphExecDestroy(g);
    if (h->g_prefill) cudaGraphExecDestroy(h->g_prefill);
    if (h->g_decode) cudaGraphExecDestroy(h->g_decode);
    if (h->g_prefill_n) cudaGraphExecDestroy(h->g_prefill_n);
    if (h->g_decode_n) cudaGraphExecDestroy(h->g_decode_n);
    for (auto e : h->ev)
        if (e) cudaEventDestroy(e);
    void *dev[] = {h->d_file, h->dm, h->b.x, h->b.q, h->b.kc, h->b.vc, h->b.partial, h->b.h, h->b.logits,
                   h->b.hidden, (void *)h->b.rope_cos, h->b.st, h->d_seq, h->d_params, h->d_hist,
                   h->d_scratch, h->d_keys, h->d_prompt, h->dplan, h->dchunks, h->dstream, h->dsync, h->dwords,
                   h->scr.cand};
    for (void *p : dev)
        if (p) cudaFree(p);
    void *host[] = {h->h_state, h->h_params, h->h_hist, h->h_keys, h->h_logits, h->h_pos0, h->h_out,
                    h->h_out_count, h->h_err};
    for (void *p : host)
        if (p) cudaFreeHost(p);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

int set_params(mocha_q8 *h, float penalty, float temperature, int top_k, float top_p)
{
    sampling::Params *p = h->h_params;
    p->penalty = penalty;
    p->temperature = temperature;
    p->top_k = temperature == 0.f ? 1 : top_k;
    p->top_p = top_p;
    p->eos = q8::EOS;
    p->control_first = q8::CONTROL_FIRST;
    p->vocab = VOCAB;
    TRY(cudaMemcpyAsync(h->d_params, p, sizeof(*p), cudaMemcpyHostToDevice, h->stream));
    return 0;
}

// Synchronisation words to their start state: epoch 1 (tag 0 never matches), data
// words cleared so no stale tag can be mistaken for this step's.
int reset_persistent(mocha_q8 *h)
{
    q8p::Sync s{1u, 0u, 0u};
    TRY(cudaMemcpy(h->dsync, &s, sizeof s, cudaMemcpyHostToDevice));
    TRY(cudaMemset(h->dwords, 0, sizeof(unsigned long long) * q8p::scratch_words()));
    return 0;
}

// A bounded wait inside the persistent kernel expired: report it, clear the
// synchronisation words so the next step starts from a clean state, and fail.
int check_device_error(mocha_q8 *h)
{
    if (!h->h_err) return 0;
    const unsigned code = __atomic_load_n(h->h_err, __ATOMIC_ACQUIRE);
    if (!code) return 0;
    fprintf(stderr, "MOCHA_B200: persistent decode step aborted (wait expired, code %u)\n", code);
    cudaStreamSynchronize(h->stream);
    if (h->dsync) reset_persistent(h);
    __atomic_store_n(h->h_err, 0u, __ATOMIC_RELEASE);
    return 1;
}

int launches_per_forward(const mocha_q8 *h, bool project)
{
    return h->persistent ? 1 : q8::forward_launches(project) + 1;
}

int forward_step(mocha_q8 *h, float *logits, int token, int pos, int project, int readback, bool profile)
{
    if (token < 0 || token >= VOCAB || pos < 0 || pos >= CONTEXT) {
        fprintf(stderr, "MOCHA_B200: token %d / pos %d out of range\n", token, pos);
        return 1;
    }
    h->h_state->token = token;
    h->h_state->pos = pos;
    TRY(cudaMemcpyAsync(h->b.st, h->h_state, 2 * sizeof(int), cudaMemcpyHostToDevice, h->stream));
    if (profile) TRY(cudaEventRecord(h->ev[0], h->stream));
    TRY(cudaGraphLaunch(h->g_forward[project ? 1 : 0], h->stream));
    if (profile) TRY(cudaEventRecord(h->ev[1], h->stream));
    const bool copy = project && readback && logits;
    if (copy) TRY(cudaMemcpyAsync(h->h_logits, h->b.logits, sizeof(float) * VOCAB, cudaMemcpyDeviceToHost, h->stream));
    TRY(cudaStreamSynchronize(h->stream));
    if (check_device_error(h)) return 1;
    if (profile) {
        float ms = 0.f;
        TRY(cudaEventElapsedTime(&ms, h->ev[0], h->ev[1]));
        h->transformer_s += ms * 1e-3;
    }
    if (copy) {
        const double t0 = now_s();
        memcpy(logits, h->h_logits, sizeof(float) * VOCAB);
        h->copy_s += now_s() - t0;
    }
    h->calls++;
    h->kernel_calls += launches_per_forward(h, project);
    return 0;
}

mocha_q8 *g_engine = nullptr;  // the reference ABI's single per-process model
constexpr int kStreamAhead = 8;  // decode steps kept enqueued ahead of the host reader

int env_device()
{
    const char *d = getenv("MOCHA_DEVICE");
    return d ? atoi(d) : 0;
}

}  // namespace

// ---------------------------------------------------------------------------
// Reference device ABI (src/minimind.h:16-22)
// ---------------------------------------------------------------------------

extern "C" int gpu_init(const void *file, unsigned bytes)
{
    if (g_engine || !q8::valid_file(file, bytes, false)) {
        fprintf(stderr, "MOCHA_B200: gpu_init: invalid grouped-Q8 file or already initialised\n");
        return 1;
    }
    mocha_q8 *h = new mocha_q8();
    if (open_full(h, env_device(), file, bytes)) {
        release(h);
        return 1;
    }
    g_engine = h;
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, h->device);
    fprintf(stderr, "BACKEND=cuda DEVICE=%s Q8_GROUP=64 GPU_WEIGHTS=%u GPU_KV=%u\n", p.name, bytes,
            (unsigned)(2u * q8::LAYERS * CONTEXT * q8::KV * 4u));
    return 0;
}

extern "C" int gpu_forward(float *logits, int token, int pos, int project, int readback)
{
    mocha_q8 *h = g_engine;
    if (!h || h->head_only) return 1;
    const char *option = getenv("MOCHA_LLM_CUDA_THREADS");
    const int threads = option ? atoi(option) : 512;
    if (threads != 256 && threads != 512 && threads != 1024) return 1;
    TRY(cudaSetDevice(h->device));
    return forward_step(h, logits, token, pos, project, readback, getenv("MOCHA_LLM_PROFILE") != nullptr);
}

extern "C" int gpu_collect(float *logits, const int *history, int count, float penalty, int k, int rows)
{
    mocha_q8 *h = g_engine;
    if (!h || k < 1 || k > 64 || count < 0 || count > 64 || rows < 1 || rows > VOCAB || !logits) return 1;
    if (count && !history) return 1;
    TRY(cudaSetDevice(h->device));
    for (int i = 0; i < count; i++) h->h_hist[i] = history[i];
    h->h_hist[64] = count;
    TRY(cudaMemcpyAsync(h->d_hist, h->h_hist, sizeof(int) * 65, cudaMemcpyHostToDevice, h->stream));
    sampling::Params *p = h->h_params;
    p->penalty = penalty;
    p->temperature = 0.f;
    p->top_k = k;
    p->top_p = 1.f;
    p->eos = q8::EOS;
    p->control_first = q8::CONTROL_FIRST;
    p->vocab = VOCAB;
    TRY(cudaMemcpyAsync(h->d_params, p, sizeof(*p), cudaMemcpyHostToDevice, h->stream));
    if (sampling::enqueue_topk(h->b.logits, rows, h->d_hist, h->d_hist + 64, h->d_params, h->d_scratch, h->d_keys,
                               h->stream))
        return 1;
    TRY(cudaMemcpyAsync(h->h_keys, h->d_keys, sizeof(unsigned long long) * k, cudaMemcpyDeviceToHost, h->stream));
    TRY(cudaStreamSynchronize(h->stream));
    h->kernel_calls += 2;
    for (int i = 0; i < rows; i++) logits[i] = -FLT_MAX;
    for (int r = 0; r < k; r++) {
        const int id = sampling::key_id_host(h->h_keys[r]);
        if (id >= 0 && id < rows) logits[id] = sampling::key_value_host(h->h_keys[r]);
    }
    return 0;
}

extern "C" int gpu_head_init(const void *file)
{
    if (g_engine || !file) return 1;
    const q8::FileHeader *hd = (const q8::FileHeader *)file;
    if (hd->magic != q8::MAGIC || hd->t[0].rows != (uint32_t)VOCAB || hd->t[0].cols != (uint32_t)DIM) return 1;
    mocha_q8 *h = new mocha_q8();
    h->head_only = true;
    cudaDeviceProp p;
    if (check_device(env_device(), &p)) {
        delete h;
        return 1;
    }
    h->device = env_device();
    const size_t n = (size_t)VOCAB * DIM;
    if (alloc_common(h) || cudaMalloc(&h->d_file, n + n / 16) != cudaSuccess ||
        cudaMemcpy(h->d_file, (const unsigned char *)file + hd->t[0].data, n, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(h->d_file + n, (const unsigned char *)file + hd->t[0].scales, n / 16, cudaMemcpyHostToDevice) !=
            cudaSuccess) {
        fprintf(stderr, "MOCHA_B200: gpu_head_init failed\n");
        release(h);
        return 1;
    }
    h->hm.embed = q8::Mat{(const int8_t *)h->d_file, (const float *)(h->d_file + n)};
    g_engine = h;
    fprintf(stderr, "BACKEND=hybrid DEVICE=%s GPU_WEIGHTS=%u\n", p.name, (unsigned)(n + n / 16));
    return 0;
}

extern "C" int gpu_head_start(const float *input, int rows)
{
    mocha_q8 *h = g_engine;
    if (!h || !input || rows < 1 || rows > VOCAB) return 1;
    TRY(cudaSetDevice(h->device));
    TRY(cudaMemcpyAsync(h->b.hidden, input, sizeof(float) * DIM, cudaMemcpyHostToDevice, h->stream));
    if (q8::enqueue_head_only(h->hm.embed, h->b.hidden, h->b.logits, rows, h->stream)) return 1;
    h->calls++;
    h->kernel_calls++;
    return 0;
}

extern "C" int gpu_head_finish(float *logits, int rows, int readback)
{
    mocha_q8 *h = g_engine;
    if (!h || rows < 1 || rows > VOCAB) return 1;
    TRY(cudaSetDevice(h->device));
    TRY(cudaStreamSynchronize(h->stream));
    if (readback) TRY(cudaMemcpy(logits, h->b.logits, sizeof(float) * rows, cudaMemcpyDeviceToHost));
    return 0;
}

extern "C" int gpu_finish(void)
{
    mocha_q8 *h = g_engine;
    if (!h) return 1;
    if (getenv("MOCHA_LLM_PROFILE"))
        fprintf(stderr, "CUDA_PROFILE TRANSFORMER_S=%.6f HEAD_S=%.6f COPY_S=%.6f\n", h->transformer_s, h->head_s,
                h->copy_s);
    const unsigned long long calls = h->calls, kernels = h->kernel_calls;
    release(h);
    g_engine = nullptr;
    fprintf(stderr, "CUDA_FORWARD_STEPS=%llu CUDA_KERNEL_CALLS=%llu\n", calls, kernels);
    return calls ? 0 : 1;
}

// ---------------------------------------------------------------------------
// Handle API (mocha_b200.h)
// ---------------------------------------------------------------------------

extern "C" int mocha_b200_device_count(void)
{
    int n = 0, ok = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    for (int d = 0; d < n; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) ok++;
    }
    return ok;
}

extern "C" int mocha_q8_open(int device, const void *file, unsigned long long bytes, mocha_q8 **out)
{
    if (!out || !q8::valid_file(file, (size_t)bytes, false)) {
        fprintf(stderr, "MOCHA_B200: mocha_q8_open: invalid grouped-Q8 file\n");
        return 1;
    }
    mocha_q8 *h = new mocha_q8();
    if (open_full(h, device, file, (size_t)bytes)) {
        release(h);
        return 1;
    }
    *out = h;
    return 0;
}

extern "C" int mocha_q8_close(mocha_q8 *h)
{
    if (!h) return 1;
    release(h);
    return 0;
}

extern "C" int mocha_q8_forward(mocha_q8 *h, int token, int pos, int project, float *logits)
{
    if (!h || h->head_only) return 1;
    TRY(cudaSetDevice(h->device));
    return forward_step(h, logits, token, pos, project, 1, false);
}

extern "C" int mocha_q8_trace_step(mocha_q8 *h, int token, int pos, unsigned long long *stamps)
{
    if (!h || !h->persistent || !stamps || token < 0 || token >= VOCAB || pos < 0 || pos >= CONTEXT) return 1;
    TRY(cudaSetDevice(h->device));
    const size_t n = (size_t)q8p::kCTAs * q8p::kTraceStamps;
    unsigned long long *d = nullptr;
    TRY(cudaMalloc(&d, n * sizeof(unsigned long long)));
    int rc = cudaMemsetAsync(d, 0, n * sizeof(unsigned long long), h->stream) != cudaSuccess;
    h->h_state->token = token;
    h->h_state->pos = pos;
    rc = rc || cudaMemcpyAsync(h->b.st, h->h_state, 2 * sizeof(int), cudaMemcpyHostToDevice, h->stream) != cudaSuccess;
    rc = rc || q8p::enqueue_step(h->dm, h->dplan, h->b, h->dsync, h->scr, q8p::FORWARD_PROJECT, h->d_params,
                                 h->d_seq, h->d_out, h->d_out_count, h->d_prompt, h->d_err, h->stream, d);
    rc = rc || cudaMemcpyAsync(stamps, d, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost, h->stream) !=
                   cudaSuccess;
    rc = rc || cudaStreamSynchronize(h->stream) != cudaSuccess;
    cudaFree(d);
    if (rc || check_device_error(h)) return 1;
    h->calls++;
    return 0;
}

extern "C" int mocha_q8_counters(mocha_q8 *h, unsigned long long *steps, unsigned long long *launches)
{
    if (!h) return 1;
    if (steps) *steps = h->calls;
    if (launches) *launches = h->kernel_calls;
    return 0;
}

extern "C" int mocha_q8_launches_per_step(mocha_q8 *h)
{
    if (!h) return 0;
    // persistent: one kernel; graph path: forward + step counter + top-k (2) + sample
    return h->persistent ? 1 : q8::forward_launches(true) + 1 + 3;
}

namespace {

bool valid_sampling(const mocha_sampling *s)
{
    return s && s->temperature >= 0.f && s->temperature < 1e30f && s->repeat_penalty >= 1.f &&
           s->repeat_penalty < 1e30f && (s->temperature == 0.f || (s->top_k >= 1 && s->top_k <= sampling::kMaxK)) &&
           s->top_p > 0.f && s->top_p <= 1.f;
}

// Sequence set-up shared by generate and the stream: history ring = last <= 64
// prompt tokens, xorshift seed, prompt upload, state at (prompt[0], 0), ring reset.
int begin_sequence(mocha_q8 *h, const int *prompt, int n_prompt, const mocha_sampling *s)
{
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= VOCAB) return 1;
    TRY(cudaSetDevice(h->device));
    TRY(cudaStreamSynchronize(h->stream));
    sampling::SeqState seq;
    memset(&seq, 0, sizeof seq);
    const int first = n_prompt > sampling::kHistory ? n_prompt - sampling::kHistory : 0;
    for (int i = first; i < n_prompt; i++) seq.history[i - first] = prompt[i];
    seq.history_count = n_prompt - first;
    seq.history_head = seq.history_count % sampling::kHistory;
    seq.seed = s->seed;
    TRY(cudaMemcpyAsync(h->d_seq, &seq, sizeof seq, cudaMemcpyHostToDevice, h->stream));
    if (set_params(h, s->repeat_penalty, s->temperature, s->top_k, s->top_p)) return 1;
    TRY(cudaMemcpyAsync(h->d_prompt, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice, h->stream));
    h->h_state->token = prompt[0];
    h->h_state->pos = 0;
    TRY(cudaMemcpyAsync(h->b.st, h->h_state, 2 * sizeof(int), cudaMemcpyHostToDevice, h->stream));
    TRY(cudaStreamSynchronize(h->stream));  // the seq copy above reads a stack buffer
    __atomic_store_n(h->h_out_count, 0, __ATOMIC_SEQ_CST);
    return 0;
}

}  // namespace

extern "C" int mocha_q8_generate(mocha_q8 *h, const int *prompt, int n_prompt, int n_new, const mocha_sampling *s,
                                 int *out_tokens, int *n_out, mocha_timing *timing)
{
    if (!h || h->head_only || !prompt || !out_tokens || n_prompt < 1 || n_new < 1 || n_prompt + n_new > CONTEXT ||
        !valid_sampling(s)) {
        fprintf(stderr, "MOCHA_B200: mocha_q8_generate: invalid arguments\n");
        return 1;
    }
    if (begin_sequence(h, prompt, n_prompt, s)) return 1;
    TRY(cudaEventRecord(h->ev[0], h->stream));
    if (launch_steps(h, 2, n_prompt - 1)) return 1;
    TRY(cudaEventRecord(h->ev[1], h->stream));
    TRY(cudaGraphLaunch(h->g_decode, h->stream));  // first sampled token (not in DECODE_TPS)
    TRY(cudaEventRecord(h->ev[2], h->stream));
    if (launch_steps(h, 3, n_new - 1)) return 1;
    TRY(cudaEventRecord(h->ev[3], h->stream));
    TRY(cudaStreamSynchronize(h->stream));
    if (check_device_error(h)) return 1;
    int n = 0;
    for (int i = 0; i < n_new; i++) out_tokens[i] = h->h_out[i];
    while (n < n_new && out_tokens[n] != q8::EOS) n++;
    if (n_out) *n_out = n;
    if (timing) {
        float a = 0, b = 0;
        TRY(cudaEventElapsedTime(&a, h->ev[0], h->ev[1]));
        TRY(cudaEventElapsedTime(&b, h->ev[2], h->ev[3]));
        timing->prefill_s = a * 1e-3;
        timing->decode_s = b * 1e-3;
        timing->generated = n;
    }
    h->calls += n_prompt - 1 + n_new;
    h->kernel_calls += (uint64_t)(n_prompt - 1) * launches_per_forward(h, false) +
                       (uint64_t)n_new * mocha_q8_launches_per_step(h);
    return 0;
}

extern "C" int mocha_q8_stream_begin(mocha_q8 *h, const int *prompt, int n_prompt, int n_new,
                                     const mocha_sampling *s)
{
    if (!h || h->head_only || !prompt || n_prompt < 1 || n_new < 1 || n_prompt + n_new > CONTEXT ||
        !valid_sampling(s)) {
        fprintf(stderr, "MOCHA_B200: mocha_q8_stream_begin: invalid arguments\n");
        return 1;
    }
    if (begin_sequence(h, prompt, n_prompt, s)) return 1;
    if (launch_steps(h, 2, n_prompt - 1)) return 1;
    h->stream_total = n_new;
    h->stream_read = 0;
    h->stream_enqueued = 0;
    h->stream_done = false;
    const int ahead = n_new < kStreamAhead ? n_new : kStreamAhead;
    for (int i = 0; i < ahead; i++) TRY(cudaGraphLaunch(h->g_decode, h->stream));
    h->stream_enqueued = ahead;
    h->calls += n_prompt - 1;
    h->kernel_calls += (uint64_t)(n_prompt - 1) * launches_per_forward(h, false);
    return 0;
}

extern "C" int mocha_q8_stream_next(mocha_q8 *h, int *token)
{
    if (!h || !token) return 1;
    if (h->stream_done || h->stream_read >= h->stream_total) {
        *token = -1;
        return 0;
    }
    // wait for the sampler's write to the mapped ring; poll the stream for errors
    long spins = 0;
    while (__atomic_load_n(h->h_out_count, __ATOMIC_ACQUIRE) <= h->stream_read) {
        if (++spins % 4096 == 0) {
            if (check_device_error(h)) {
                h->stream_done = true;
                return 1;
            }
            const cudaError_t e = cudaStreamQuery(h->stream);
            if (e != cudaSuccess && e != cudaErrorNotReady) {
                fprintf(stderr, "CUDA decode stream: %d %s\n", (int)e, cudaGetErrorString(e));
                h->stream_done = true;
                return 1;
            }
            if (e == cudaSuccess && __atomic_load_n(h->h_out_count, __ATOMIC_ACQUIRE) <= h->stream_read) {
                fprintf(stderr, "MOCHA_B200: decode stream idle without a token\n");
                h->stream_done = true;
                return 1;
            }
        }
    }
    const int t = h->h_out[h->stream_read % sampling::kOutRing];
    h->stream_read++;
    h->calls++;
    h->kernel_calls += mocha_q8_launches_per_step(h);
    if (t == q8::EOS || h->stream_read >= h->stream_total) {
        h->stream_done = true;
    } else if (h->stream_enqueued < h->stream_total) {
        TRY(cudaGraphLaunch(h->g_decode, h->stream));
        h->stream_enqueued++;
    }
    *token = t;
    return 0;
}

extern "C" int mocha_q8_stream_end(mocha_q8 *h)
{
    if (!h) return 1;
    h->stream_done = true;
    TRY(cudaSetDevice(h->device));
    TRY(cudaStreamSynchronize(h->stream));
    return check_device_error(h);
}

extern "C" int mocha_q8_bench_decode(mocha_q8 *h, int token, int pos0, int pos_end, int warmup, int steps, float *ms)
{
    if (!h || h->head_only || !ms || token < 0 || token >= VOCAB || pos0 < 0 || pos_end <= pos0 ||
        pos_end > CONTEXT || warmup < 0 || steps < 1)
        return 1;
    TRY(cudaSetDevice(h->device));
    if (set_params(h, 1.f, 0.f, 1, 1.f)) return 1;
    h->h_pos0[0] = token;
    h->h_pos0[1] = pos0;
    TRY(cudaMemcpyAsync(h->b.st, h->h_pos0, 2 * sizeof(int), cudaMemcpyHostToDevice, h->stream));
    int pos = pos0;
    for (int i = 0; i < warmup + steps; i++) {
        if (i == warmup) TRY(cudaEventRecord(h->ev[0], h->stream));
        if (pos == pos_end) {
            TRY(cudaMemcpyAsync(&h->b.st->pos, h->h_pos0 + 1, sizeof(int), cudaMemcpyHostToDevice, h->stream));
            pos = pos0;
        }
        TRY(cudaGraphLaunch(h->g_decode, h->stream));
        pos++;
    }
    TRY(cudaEventRecord(h->ev[1], h->stream));
    TRY(cudaStreamSynchronize(h->stream));
    if (check_device_error(h)) return 1;
    TRY(cudaEventElapsedTime(ms, h->ev[0], h->ev[1]));
    h->calls += warmup + steps;
    return 0;
}
