// mocha_topk_static: candidate selection that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the moment they want candidates: a serving
// host that has reserved the whole GPU memory budget in its own pool (an extra
// allocation fails or fragments it), or a latency-critical loop where cudaMalloc's
// implicit device synchronisation would stall the other streams.  This
// entry point runs the same penalty / control-mask / top-k kernels as gpu_collect
// (sampling.cu), but every device-side buffer it needs -- the staged logits and
// history, the parameters, the per-CTA partial keys and the merged keys -- lives in
// one file-scope __device__ array of fixed size.  The caller passes host inputs and
// host outputs; the call waits for its stream before it returns.
//
// Limits and sharing rules:
//   * 1 <= k <= min(64, rows) and rows <= kMaxRows (151,936, one Qwen2.5
//     vocabulary); other requests fail with a message.  The array occupies ~672 KiB on every GPU that loads the library,
//     until the process exits.
//   * Every call reuses the same array, which keeps the previous call's contents;
//     everything a call reads is written by that call first.  Calls that overlap on
//     the GPU (from several host threads or streams) race on the array and must not
//     be issued concurrently.
//   * The control mask is Qwen2.5's (src/minimind.cu:143-144): ids >= 151643 other
//     than EOS 151645 are set to -1e30 before selection, so it only touches callers
//     whose rows extend past 151643.
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (and sets the merge kernel's shared-memory limit); make
//     that first call before starting any stream capture on that device.
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "mocha_b200.h"
#include "sampling.cuh"

namespace {

constexpr int kMaxRows = 151936;
constexpr size_t kLogitsOff = 0;
constexpr size_t kHistOff = kLogitsOff + (size_t)kMaxRows * sizeof(float);         // 64 ids + count
constexpr size_t kParamsOff = kHistOff + 272;
constexpr size_t kStage1Off = kParamsOff + 256;                                      // 148 x 64 keys
constexpr size_t kKeysOff = kStage1Off + (size_t)sampling::kStage1Blocks * sampling::kMaxK * 8;
constexpr size_t kScratchBytes = kKeysOff + (size_t)sampling::kMaxK * 8;

static __device__ __align__(256) unsigned char g_topk_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
unsigned char *g_scratch_addr[kMaxDevices];  // device address of g_topk_scratch per device

int report(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return 0;
    fprintf(stderr, "mocha_topk_static: %s: %d %s\n", what, (int)e, cudaGetErrorString(e));
    return 1;
}

// Once per device, with that device current: the array's device address.  The host
// symbol itself is only a stand-in and must never be handed to a kernel.
unsigned char *scratch_for_current_device()
{
    int dev = -1;
    if (report(cudaGetDevice(&dev), "cudaGetDevice")) return nullptr;
    if (dev < 0 || dev >= kMaxDevices) {
        fprintf(stderr, "mocha_topk_static: device %d out of range\n", dev);
        return nullptr;
    }
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        if (report(cudaGetSymbolAddress(&p, g_topk_scratch), "cudaGetSymbolAddress")) return nullptr;
        if (sampling::init_device()) return nullptr;
        g_scratch_addr[dev] = static_cast<unsigned char *>(p);
    }
    return g_scratch_addr[dev];
}

}  // namespace

extern "C" int mocha_topk_static(const float *logits, int rows, const int *history, int count, float penalty, int k,
                                 float *values, int *ids, void *stream)
{
    if (!logits || !values || !ids || (count && !history)) {
        fprintf(stderr, "mocha_topk_static: null argument\n");
        return 1;
    }
    if (rows < 1 || rows > kMaxRows) {
        fprintf(stderr, "mocha_topk_static: rows=%d outside [1, %d] (fixed scratch size)\n", rows, kMaxRows);
        return 1;
    }
    if (k < 1 || k > sampling::kMaxK || count < 0 || count > sampling::kHistory) {
        fprintf(stderr, "mocha_topk_static: k must be 1..64 and count 0..64\n");
        return 1;
    }
    if (k > rows) {  // fewer candidates than asked for: the merge would return empty keys
        fprintf(stderr, "mocha_topk_static: k=%d exceeds rows=%d\n", k, rows);
        return 1;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the call copies to and from host stack buffers and waits for the stream: inside a
    // capture it would invalidate the capture, so it refuses instead
    cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &capturing) != cudaSuccess || capturing != cudaStreamCaptureStatusNone) {
        fprintf(stderr, "mocha_topk_static: the stream is being captured (the call waits for it); call it outside a capture\n");
        return 1;
    }
    unsigned char *base = scratch_for_current_device();
    if (!base) return 1;
    float *d_logits = reinterpret_cast<float *>(base + kLogitsOff);
    int *d_hist = reinterpret_cast<int *>(base + kHistOff);
    sampling::Params *d_params = reinterpret_cast<sampling::Params *>(base + kParamsOff);
    unsigned long long *d_stage1 = reinterpret_cast<unsigned long long *>(base + kStage1Off);
    unsigned long long *d_keys = reinterpret_cast<unsigned long long *>(base + kKeysOff);

    int hist[sampling::kHistory + 1];
    for (int i = 0; i < count; i++) hist[i] = history[i];
    hist[sampling::kHistory] = count;
    sampling::Params p{};
    p.penalty = penalty;
    p.temperature = 0.f;
    p.top_k = k;
    p.top_p = 1.f;
    p.eos = 151645;
    p.control_first = 151643;
    p.vocab = rows;
    unsigned long long keys[sampling::kMaxK];
    // every byte the kernels read is written here first; nothing else needs clearing
    if (report(cudaMemcpyAsync(d_logits, logits, sizeof(float) * rows, cudaMemcpyHostToDevice, s), "copy logits") ||
        report(cudaMemcpyAsync(d_hist, hist, sizeof hist, cudaMemcpyHostToDevice, s), "copy history") ||
        report(cudaMemcpyAsync(d_params, &p, sizeof p, cudaMemcpyHostToDevice, s), "copy params"))
        return 1;
    if (sampling::enqueue_topk(d_logits, rows, d_hist, d_hist + sampling::kHistory, d_params, d_stage1, d_keys, s))
        return 1;
    if (report(cudaMemcpyAsync(keys, d_keys, sizeof(unsigned long long) * k, cudaMemcpyDeviceToHost, s),
               "copy keys") ||
        report(cudaStreamSynchronize(s), "synchronize"))
        return 1;
    for (int r = 0; r < k; r++) {
        values[r] = sampling::key_value_host(keys[r]);
        ids[r] = sampling::key_id_host(keys[r]);
    }
    return 0;
}
