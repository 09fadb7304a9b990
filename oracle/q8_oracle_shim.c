/* The reference's device entry points (src/minimind.h:16-22) served by the CPU
 * restatement in q8_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * Linked with the reference host (src/minimind.cpp) this pins the restatement:
 * with --check the host compares every logit of every step against its own cpu()
 * and prints MAX_ABS_ERROR, which must be exactly 0. */
#include "q8_oracle.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static q8o_model *model;
static unsigned char *copy;
static float *logits_buf;
static const q8o_tensor *head;
static unsigned long long calls;

int gpu_init(const void *file, unsigned bytes)
{
    copy = (unsigned char *)malloc(bytes);
    logits_buf = (float *)malloc(sizeof(float) * Q8O_VOCAB);
    if (!copy || !logits_buf) return 1;
    memcpy(copy, file, bytes);
    model = q8o_create(copy, bytes);
    if (!model) return 1;
    head = &q8o_tensors(model)[0];
    fprintf(stderr, "BACKEND=cuda DEVICE=cpu-oracle Q8_GROUP=64 GPU_WEIGHTS=%u GPU_KV=%u\n", bytes,
            2u * Q8O_LAYERS * Q8O_CONTEXT * Q8O_KV * 4u);
    return 0;
}

int gpu_forward(float *logits, int token, int pos, int project, int readback)
{
    if (!model || token < 0 || token >= Q8O_VOCAB || pos < 0 || pos >= Q8O_CONTEXT) return 1;
    q8o_forward(model, token, pos, project, 0, logits_buf);
    if (project && readback) memcpy(logits, logits_buf, sizeof(float) * Q8O_VOCAB);
    calls++;
    return 0;
}

int gpu_collect(float *logits, const int *history, int count, float penalty, int k, int rows)
{
    return q8o_collect(logits_buf, logits, history, count, penalty, k, rows);
}

int gpu_head_init(const void *file)
{
    const q8o_tensor *t = (const q8o_tensor *)((const unsigned *)file + 8);
    size_t n = (size_t)t[0].rows * t[0].cols;
    copy = (unsigned char *)malloc(n + n / 16);
    logits_buf = (float *)malloc(sizeof(float) * Q8O_VOCAB);
    if (!copy || !logits_buf) return 1;
    memcpy(copy, (const unsigned char *)file + t[0].data, n);
    memcpy(copy + n, (const unsigned char *)file + t[0].scales, n / 16);
    static q8o_tensor local;
    local = t[0];
    local.data = 0;
    local.scales = (unsigned)n;
    head = &local;
    return 0;
}

int gpu_head_start(const float *input, int rows)
{
    q8o_matvec((const int8_t *)copy + head->data, (const float *)(copy + head->scales), (unsigned)rows,
               head->cols, input, logits_buf, 0, 0);
    calls++;
    return 0;
}

int gpu_head_finish(float *logits, int rows, int readback)
{
    if (readback) memcpy(logits, logits_buf, sizeof(float) * (size_t)rows);
    return 0;
}

int gpu_finish(void)
{
    fprintf(stderr, "CUDA_FORWARD_STEPS=%llu CUDA_KERNEL_CALLS=%llu\n", calls, calls);
    q8o_destroy(model);
    free(copy);
    free(logits_buf);
    return calls ? 0 : 1;
}
