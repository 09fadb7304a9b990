// mocha-qwen-engine: the grouped-Q8 Qwen2.5-0.5B token-loop host for B200.
//
// Command-line protocol, exit codes and output lines are the reference engine's
// (src/minimind.cpp:84-191), so the unchanged Python launcher (mocha-llm:136-147) can
// drive it:
//
//   mocha-qwen-engine MODEL TOKEN_IDS NEW_TOKENS cuda TEMPERATURE SEED CHECK
//                     REPEAT_PENALTY TOP_K TOP_P
//
// stdout: one sampled token id per line (EOS stops the loop and is not printed);
// stderr: BACKEND=... PROMPT_TOKENS GENERATED STARTUP_S PREFILL_S DECODE_TPS WALL_S
// CHECKED MAX_ABS_ERROR, RSS_KIB PEAK_RSS_KIB, CUDA_FORWARD_STEPS CUDA_KERNEL_CALLS.
// Exit codes: 2 bad arguments / model file, 3 device error.
//
// The whole loop runs on the device (library handle API): prompt positions only
// fill the KV cache, sampling happens on the device and tokens stream back through
// mapped host memory.  top_k above 64 at T > 0 uses the full-logit path with the
// host sampler, as the reference does for k > 64 (src/minimind.cpp:104).  There is
// no CPU transformer: backends cpu/hybrid and CHECK=1 are served by the reference
// host linked against libmocha_b200.so (gpu_* ABI), not by this binary.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "mocha_b200.h"

namespace {

constexpr int kDim = 896, kHidden = 4864, kLayers = 24, kVocab = 151936, kContext = 1024, kEos = 151645;
constexpr int kControlFirst = 151643, kHeaderBytes = 8192, kTensors = 290;

double now() { return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count(); }

struct FileTensor { uint32_t data, scales, rows, cols; };

bool header_ok(const unsigned char *base, size_t size)
{
    if (size < (size_t)kHeaderBytes) return false;
    uint32_t h[8];
    std::memcpy(h, base, sizeof h);
    if (h[0] != 0x384D4D4Du || h[1] != 1 || h[2] != (uint32_t)size || h[3] != (uint32_t)kDim ||
        h[4] != (uint32_t)kHidden || h[5] != (uint32_t)kLayers || h[6] != (uint32_t)kVocab || h[7] != 64)
        return false;
    for (int i = 0; i < kTensors; i++) {
        FileTensor t;
        std::memcpy(&t, base + 32 + 16 * i, sizeof t);
        const uint64_t bytes = (uint64_t)t.rows * (t.scales ? t.cols : 4);
        if (t.data < (uint32_t)kHeaderBytes || t.data + bytes > size) return false;
        if (t.scales && (t.cols % 64 || t.scales + bytes / 64 * 4 > size)) return false;
    }
    return true;
}

// Host sampler for top_k > 64 on full logits, with the reference's semantics:
// penalty on distinct ids of the last 64 history tokens, control mask, top-k by
// (value desc, id asc), softmax with temperature, top-p cutoff, xorshift32 draw.
int sample_full(std::vector<float> &logits, const std::vector<int> &history, float penalty, float temp, int top_k,
                float top_p, unsigned &seed)
{
    std::vector<char> seen(kVocab, 0);
    for (size_t j = history.size() > 64 ? history.size() - 64 : 0; j < history.size(); j++) {
        const int id = history[j];
        if (!seen[id]) {
            logits[id] = logits[id] < 0 ? logits[id] * penalty : logits[id] / penalty;
            seen[id] = 1;
        }
    }
    for (int id = kControlFirst; id < kVocab; id++)
        if (id != kEos) logits[id] = -1e30f;
    std::vector<int> order(kVocab);
    for (int i = 0; i < kVocab; i++) order[i] = i;
    std::partial_sort(order.begin(), order.begin() + top_k, order.end(),
                      [&](int a, int b) { return logits[a] > logits[b] || (logits[a] == logits[b] && a < b); });
    const float largest = logits[order[0]];
    float sum = 0;
    for (int j = 0; j < top_k; j++) {
        float &v = logits[order[j]];
        v = std::exp((v - largest) / temp);
        sum += v;
    }
    float cutoff = 0;
    int kept = 0;
    while (kept < top_k && cutoff < sum * top_p) cutoff += logits[order[kept++]];
    seed ^= seed << 13;
    seed ^= seed >> 17;
    seed ^= seed << 5;
    float r = (float)((seed / 4294967296.0) * cutoff);
    int token = order[kept - 1];
    for (int j = 0; j < kept; j++) {
        r -= logits[order[j]];
        if (r <= 0) {
            token = order[j];
            break;
        }
    }
    return token;
}

void print_rss()
{
    unsigned long rss = 0, peak = 0;
    char line[256];
    if (FILE *f = std::fopen("/proc/self/status", "r")) {
        while (std::fgets(line, sizeof line, f)) {
            std::sscanf(line, "VmRSS: %lu kB", &rss);
            std::sscanf(line, "VmHWM: %lu kB", &peak);
        }
        std::fclose(f);
    }
    std::fprintf(stderr, "RSS_KIB=%lu PEAK_RSS_KIB=%lu\n", rss, peak);
}

}  // namespace

int main(int argc, char **argv)
{
    if (argc != 11) {
        std::fprintf(stderr,
                     "usage: engine MODEL TOKEN_IDS NEW_TOKENS cuda TEMPERATURE SEED CHECK REPEAT_PENALTY TOP_K TOP_P\n");
        return 2;
    }
    const int fd = open(argv[1], O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st)) return 2;
    const size_t size = (size_t)st.st_size;
    void *map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return 2;
    const unsigned char *base = (const unsigned char *)map;
    if (!header_ok(base, size)) return 2;

    std::vector<int> prompt;
    FILE *f = std::fopen(argv[2], "r");
    if (!f) return 2;
    int token;
    while (std::fscanf(f, "%d", &token) == 1) {
        if (token < 0 || token >= kVocab) {
            std::fclose(f);
            return 2;
        }
        prompt.push_back(token);
    }
    std::fclose(f);
    const int count = std::atoi(argv[3]);
    const float temp = (float)std::atof(argv[5]);
    unsigned seed = (unsigned)std::strtoul(argv[6], nullptr, 10);
    const int check = std::atoi(argv[7]);
    const float penalty = (float)std::atof(argv[8]), top_p = (float)std::atof(argv[10]);
    const int top_k = std::atoi(argv[9]);
    if (prompt.empty() || count < 1 || prompt.size() + count > (size_t)kContext || temp < 0 || !std::isfinite(temp) ||
        !std::isfinite(penalty) || penalty < 1 || top_k < 1 || top_k > kVocab || !(top_p > 0 && top_p <= 1))
        return 2;
    if (std::strcmp(argv[4], "cuda") != 0 || check) {
        std::fprintf(stderr, "mocha-qwen-engine runs the cuda backend only; cpu/hybrid/--check are served by the "
                             "reference host linked against libmocha_b200.so\n");
        return 2;
    }

    const double start = now();
    const char *dev = std::getenv("MOCHA_DEVICE");
    mocha_q8 *h = nullptr;
    if (mocha_q8_open(dev ? std::atoi(dev) : 0, base, size, &h)) return 3;
    std::fprintf(stderr, "BACKEND=cuda DEVICE=B200 Q8_GROUP=64 GPU_WEIGHTS=%zu GPU_KV=%u\n", size,
                 2u * kLayers * kContext * 128u * 4u);
    madvise(map, size, MADV_DONTNEED);
    const double ready = now();
    double decode_start = 0;
    int generated = 0;

    const bool full_logits = temp > 0 && top_k > 64;
    if (!full_logits) {
        mocha_sampling s{temp, temp == 0 ? 1 : top_k, top_p, penalty, seed};
        if (mocha_q8_stream_begin(h, prompt.data(), (int)prompt.size(), count, &s)) return 3;
        for (;;) {
            int t;
            if (mocha_q8_stream_next(h, &t)) return 3;
            if (t < 0) break;
            if (!decode_start) decode_start = now();
            if (t == kEos) break;
            std::printf("%d\n", t);
            std::fflush(stdout);
            generated++;
        }
        if (mocha_q8_stream_end(h)) return 3;
    } else {
        std::vector<float> logits(kVocab);
        std::vector<int> history = prompt;
        token = prompt[0];
        for (int pos = 0; pos < (int)prompt.size() + count - 1; pos++) {
            const bool project = pos + 1 >= (int)prompt.size();
            if (mocha_q8_forward(h, token, pos, project, logits.data())) return 3;
            if (!project) {
                token = prompt[pos + 1];
                continue;
            }
            if (!decode_start) decode_start = now();
            token = sample_full(logits, history, penalty, temp, top_k, top_p, seed);
            if (token == kEos) break;
            std::printf("%d\n", token);
            std::fflush(stdout);
            generated++;
            history.push_back(token);
        }
    }
    const double done = now();
    std::fprintf(stderr,
                 "BACKEND=cuda PROMPT_TOKENS=%zu GENERATED=%d STARTUP_S=%.3f PREFILL_S=%.3f DECODE_TPS=%.3f "
                 "WALL_S=%.3f CHECKED=0 MAX_ABS_ERROR=0\n",
                 prompt.size(), generated, ready - start, (decode_start ? decode_start : done) - ready,
                 generated > 1 ? (generated - 1) / (done - decode_start) : 0.0, done - start);
    print_rss();
    unsigned long long steps = 0, launches = 0;
    mocha_q8_counters(h, &steps, &launches);
    mocha_q8_close(h);
    std::fprintf(stderr, "CUDA_FORWARD_STEPS=%llu CUDA_KERNEL_CALLS=%llu\n", steps, launches);
    munmap(map, size);
    return 0;
}
