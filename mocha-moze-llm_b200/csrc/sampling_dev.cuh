// Device-side token draw shared by the sampling kernels and the persistent decode
// kernel: greedy or the reference host's top-k / temperature / top-p / xorshift32
// sampler (src/minimind.cpp:171-179) over candidate keys sorted best first.
#pragma once
#include "mb_common.cuh"
#include "sampling.cuh"

namespace sampling {

MB_DEV int draw_token(const unsigned long long *keys, const Params &p, uint32_t &seed)
{
    if (p.temperature == 0.f) return mb::key_id(keys[0]);
    float prob[kMaxK];
    int ids[kMaxK];
    const int k = min(max(p.top_k, 1), kMaxK);
    const float largest = mb::key_value(keys[0]);
    float sum = 0.f;
    for (int j = 0; j < k; j++) {
        ids[j] = mb::key_id(keys[j]);
        prob[j] = expf((mb::key_value(keys[j]) - largest) / p.temperature);
        sum += prob[j];
    }
    float cutoff = 0.f;
    int kept = 0;
    while (kept < k && cutoff < sum * p.top_p) cutoff += prob[kept++];
    uint32_t s = seed;
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    seed = s;
    float r = (float)((s / 4294967296.0) * (double)cutoff);
    int token = ids[kept - 1];
    for (int j = 0; j < kept; j++) {
        r -= prob[j];
        if (r <= 0.f) {
            token = ids[j];
            break;
        }
    }
    return token;
}

// Record a sampled token: history ring, EOS flag, output ring (optionally in mapped
// host memory, count published after a system fence).
MB_DEV void record_token(int token, const Params &p, SeqState *st, int *out_ring, int *out_count)
{
    st->history[st->history_head] = token;
    st->history_head = (st->history_head + 1) % kHistory;
    if (st->history_count < kHistory) st->history_count++;
    st->last_token = token;
    if (token == p.eos) st->finished = 1;
    if (out_ring) {
        const int n = st->n_out;
        out_ring[n % kOutRing] = token;
        st->n_out = n + 1;
        __threadfence_system();
        *(volatile int *)out_count = n + 1;
    }
}

}  // namespace sampling
